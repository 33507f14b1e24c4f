"""GGUF -> HBM staging checked by the residency layer's checksum (hash64, eahmmf.h:64-76) on the device:

* eahmmf_cuda_hash64 over device ranges of every length modulo 8 and unaligned starts equals the
  reference's hash64 of the same bytes (compiled from its sources);
* eahmmf_engine_verify after loading a model finds every expert component equal to the file, and after
  one byte of one expert is changed in the file (the source the copy must match), exactly that
  component differs -- the --verify contract of Config::verify (eahmmf.h:203-214, :1014).
"""
import os
import shutil

import numpy as np
import pytest

import eahmmf_b200 as eb
import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    eb.lib()
    return torch.device("cuda", 0)


def test_device_hash64_matches_reference(dev, ref):
    import torch
    rng = np.random.default_rng(5)
    host = rng.integers(0, 256, 3 << 20, dtype=np.uint8)
    d = torch.from_numpy(host).to(dev)
    ranges = [(0, 0), (0, 1), (3, 7), (8, 8), (5, 1000), (16, 884736), (1, 1290240), (7, 2 << 20), (0, 3 << 20)]
    got = eb.cuda_hash64([(d, o, n) for o, n in ranges])
    want = [ref.hash64(host[o:o + n]) for o, n in ranges]
    assert got == want


def _expert_offset(path, name):
    import gguf
    r = gguf.GGUFReader(path)
    for t in r.tensors:
        if t.name == name:
            return int(t.data_offset)
    raise KeyError(name)


def test_engine_verify_detects_a_changed_expert(dev, tmp_path):
    path = synth.write_gguf(str(tmp_path / "c1.gguf"), synth.config1_tiny())
    e = eb.Engine(path, 64)
    try:
        rc, n, bad = e.verify()
        assert rc == 0 and bad == 0
        assert n == 2 * 8 * 3  # layers x experts x gate/up/down
        off = _expert_offset(path, "blk.1.ffn_up_exps.weight")
        per = 256 * 144  # one expert's Q4_K up matrix: 256 rows of 144 bytes
        with open(path, "r+b") as f:  # one byte inside expert 5 of layer 1
            f.seek(off + 5 * per + 1234)
            b = f.read(1)
            f.seek(off + 5 * per + 1234)
            f.write(bytes([b[0] ^ 0x40]))
        rc, n, bad = e.verify()
        assert rc == 0 and bad == 1
    finally:
        e.close()
