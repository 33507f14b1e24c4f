"""The reference's own residency suite (tests/test_eahmmf.cpp of the reference: 204 checks over the
ExpertStore / ExpertPager / ExpertLease API, tier matrix, fault injection, VRAM pressure, lease
lifecycle), compiled unmodified by oracle/Makefile (oracle/_ref/test_eahmmf) and run on the reference's
tiny model (tests/golden/ref_tiny.gguf). It must still pass as-is next to this project's adapters: the
C++ API the adapters implement is the one it checks. CPU only (the suite's devices are host stand-ins);
the same tiers on the real backend are tests/test_gpu_store.py's.
"""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "test_eahmmf")
TINY = os.path.join(ROOT, "tests", "golden", "ref_tiny.gguf")
REF = os.environ.get("EAHMMF_REF", os.path.normpath(os.path.join(ROOT, "..", "reference")))


def test_reference_residency_suite_passes(tmp_path):
    logits = os.path.join(REF, "baseline", "logits.txt")
    if not os.path.exists(BIN) or not os.path.exists(logits):
        pytest.skip("needs oracle/_ref/test_eahmmf and the reference tree (build container)")
    os.makedirs(tmp_path / "baseline")
    with open(logits) as f, open(tmp_path / "baseline" / "logits.txt", "w") as g:
        g.write(f.read())  # the suite reads its golden logits from ./baseline
    r = subprocess.run([BIN, TINY], cwd=tmp_path, capture_output=True, timeout=600,
                       env=dict(os.environ, OMP_NUM_THREADS="4"))
    err = r.stderr.decode()
    m = re.search(r"^(\d+) checks, (\d+) failed$", err, re.M)
    assert m, err[-2000:]
    assert int(m.group(1)) == 204 and int(m.group(2)) == 0, err[-3000:]
    assert r.returncode == 0
