"""The reference engine's ExpertStore on eahmmf::B200Device, and eahmmf_cuda_moe_layer fed from the
layer tables that eahmmf::B200LayerTable builds out of ExpertLeases (include/eahmmf_b200_device.hpp).

Runs oracle/_ref/b200_store_check (built with the reference engine compiled unmodified) on the
reference's tiny model:
  * the store places every expert in VRAM through B200Device with --verify checksums on, and the bytes
    read back through the backend equal the GGUF source;
  * decode with every expert matmul on the GPU gives the reference CPU logits within 2e-6 and the same
    12 greedy ids;
  * per layer, the table holds one pin per expert while it lives and none after clear(); the MoE layer
    on those tables routes bit-exactly and matches the reference MoE block within rel-L2 1e-5.
"""
import os
import re
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "b200_store_check")
TINY = os.path.join(ROOT, "tests", "golden", "ref_tiny.gguf")


@pytest.fixture(scope="module")
def report(golden):
    if not os.path.exists(BIN):
        pytest.fail(f"{BIN} missing: `make -C oracle storecheck` in the build container")
    g = golden("ref_tiny.npz")
    ids = ",".join(str(int(t)) for t in g["prompt"])
    r = subprocess.run([BIN, TINY, ids, "12", "5"], capture_output=True, timeout=300,
                       env=dict(os.environ, OMP_NUM_THREADS="4"))
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    return r.stdout.decode(), g


def test_backend_decode_matches_reference(report):
    out, g = report
    assert re.search(r"^backend_name cuda$", out, re.M)
    lg = np.array(re.search(r"^logits (.*)$", out, re.M).group(1).split(), np.float64)
    assert np.abs(lg - g["logits"]).max() < 2e-6
    greedy = [int(v) for v in re.search(r"^greedy (.*)$", out, re.M).group(1).split()]
    assert greedy == [int(v) for v in g["gen12"]]
    assert re.search(r"^store_pinned_after_decode 0$", out, re.M)


def test_layer_tables_from_leases(report):
    out, _ = report
    n_layer = len(re.findall(r"^layer \d+ table", out, re.M))
    n_expert = int(re.search(r"^n_expert (\d+)$", out, re.M).group(1))
    assert n_layer >= 2
    for l in range(n_layer):
        m = re.search(rf"^layer {l} table (\d) pinned (\d+)$", out, re.M)
        assert m and m.group(1) == "1"
        assert int(m.group(2)) == n_expert  # one pin per expert while the table lives
        m = re.search(rf"^layer {l} bytes_equal (\d) status (-?\d+) ids_equal (\d) rel_l2 (\S+)$", out, re.M)
        assert m, out[-2000:]
        assert m.group(1) == "1" and m.group(2) == "0" and m.group(3) == "1"
        assert float(m.group(4)) < 1e-5
        assert re.search(rf"^layer {l} released pinned 0$", out, re.M)
    assert re.search(r"^done 1$", out, re.M)
