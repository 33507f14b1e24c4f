"""Pins the CPU oracle (oracle/oracle.c) before it is trusted as the parity checker.

Pins, in order of independence:
  * gguf-py's dequantizer (an independent implementation of the GGUF block formats),
  * the reference engine compiled from its own sources (fixtures recorded by tests/golden/make_fixtures.py),
  * through the reference engine, the reference's golden vectors (baseline/logits.txt and
    baseline/gen_greedy.bin, checked when the fixtures were made; recorded in fixtures.json).
"""
import hashlib
import json
import os

import numpy as np
import pytest

import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("qtype", [synth.Q4_K, synth.Q5_K, synth.Q6_K, synth.Q8_0])
def test_dequant_matches_gguf_py(orc, qtype):
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize
    blck, nb = synth.BLOCK[qtype]
    rows, K = 6, blck * 4
    raw = synth.quant_blocks(qtype, rows * 4, synth._rng(42, qtype), 0.01).reshape(rows, -1)
    mine = orc.dequant(qtype, raw, K, rows)
    theirs = dequantize(raw, GGMLQuantizationType(qtype)).reshape(rows, K).astype(np.float32)
    np.testing.assert_allclose(mine, theirs, rtol=2e-6, atol=1e-9)


def test_f16_edge_values(orc):
    import ctypes
    f = orc.lib.orc_f16
    f.restype, f.argtypes = ctypes.c_float, [ctypes.c_uint16]
    for h in (0x0000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x8001, 0xFC00, 0x7C00):
        want = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        assert f(h) == want or (np.isinf(want) and np.isinf(f(h)))


@pytest.mark.parametrize("qtype,K", [(12, 1024), (13, 512), (14, 768), (8, 288), (0, 320)])
@pytest.mark.parametrize("nb", [1, 5])
def test_matmul_matches_reference(orc, golden, qtype, K, nb):
    g = golden("matmul.npz")
    raw, x, want = g[f"w{qtype}"], g[f"x{qtype}_{nb}"], g[f"y{qtype}_{nb}"]
    got = orc.matmul(raw, qtype, K, 40, synth.row_bytes(qtype, K), x)
    assert _rel_l2(got, want) < 2e-6
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5 * np.abs(want).max())


@pytest.mark.parametrize("T", [1, 3, 8])
def test_moe_layer_config2_matches_reference(orc, golden, experts_c2, T):
    ex = experts_c2
    g = golden("moe_c2.npz")
    x = synth.activations(T, ex.D, seed=100 + T)
    xn = synth.activations(T, ex.D, seed=200 + T)
    lg = synth.router_logits(T, ex.n_expert, seed=300 + T)
    y, ids, w = orc.moe_layer(x, xn, lg, list(ex.gate), list(ex.up), list(ex.down), ex.types, ex.row_bytes, 8)
    np.testing.assert_array_equal(ids, g[f"ids{T}"])
    np.testing.assert_array_equal(w.view(np.uint32), g[f"w{T}"].view(np.uint32))  # bit-exact routing weights
    assert _rel_l2(y - x, g[f"y{T}"] - x) < 1e-5


def test_moe_layer_mixed_types_with_router_matrix(orc, golden):
    mx = synth.expert_set(D=256, FF=256, n_expert=8, types=(13, 12, 14), seed=7, d_sigma=0.002)
    g = golden("moe_mixed.npz")
    T = 11
    x = synth.activations(T, 256, seed=17)
    xn = synth.activations(T, 256, seed=18)
    rw = (synth._rng(19).normal(0, 0.3, (8, 256))).astype(np.float32)
    y, ids, w = orc.moe_layer(x, xn, None, list(mx.gate), list(mx.up), list(mx.down), mx.types, mx.row_bytes, 2,
                              router_w=rw)
    # router logits come from different fp32 summation orders, so ids are compared exactly but the
    # weights only to the logits' rounding
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_allclose(w, g["w"], rtol=1e-5)
    assert _rel_l2(y - x, g["y"] - x) < 1e-5


def test_routing_ties_prefer_lower_index(orc):
    # equal logits -> equal expf values -> the reference's comparator ranks the lower index first
    lg = np.zeros((3, 16), np.float32)
    lg[0, [3, 9, 12]] = 2.0
    lg[1, :] = 1.0
    lg[2, [15, 14, 1]] = [5.0, 5.0, 4.0]
    ids, w = orc.route(lg, 4)
    assert ids[0].tolist() == [3, 9, 12, 0]
    assert ids[1].tolist() == [0, 1, 2, 3]
    assert ids[2].tolist() == [14, 15, 1, 0]
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)


def test_routing_ties_match_reference(orc, ref):
    mx = synth.expert_set(D=256, FF=256, n_expert=8, types=(12, 12, 12), seed=8, d_sigma=0.002)
    T = 6
    lg = np.round(synth.router_logits(T, 8, seed=5) * 2) / 2  # many exact ties
    x = synth.activations(T, 256, seed=1)
    y1, i1, w1 = orc.moe_layer(x, x, lg, list(mx.gate), list(mx.up), list(mx.down), mx.types, mx.row_bytes, 3)
    y2, i2, w2 = ref.moe_layer(x, x, lg, list(mx.gate), list(mx.up), list(mx.down), mx.types, mx.row_bytes, 3)
    np.testing.assert_array_equal(i1, i2)
    np.testing.assert_array_equal(w1.view(np.uint32), w2.view(np.uint32))
    assert _rel_l2(y1 - x, y2 - x) < 1e-5


def test_fixture_files_are_pinned():
    meta = json.load(open(os.path.join(GOLDEN, "fixtures.json")))
    h = hashlib.sha256(open(os.path.join(GOLDEN, "ref_tiny.gguf"), "rb").read()).hexdigest()
    assert h == meta["ref_tiny_sha256"]
    assert meta["baseline_gen_greedy"] == "byte-exact" and meta["baseline_logits_maxdiff"] < 2e-6


def test_config1_generator_is_deterministic(tmp_path):
    meta = json.load(open(os.path.join(GOLDEN, "fixtures.json")))
    p = synth.write_gguf(str(tmp_path / "c1.gguf"), synth.config1_tiny())
    assert hashlib.sha256(open(p, "rb").read()).hexdigest() == meta["config1_sha256"]


def test_reference_engine_reproduces_fixtures(ref, golden):
    g = golden("ref_tiny.npz")
    eng = ref.engine(os.path.join(GOLDEN, "ref_tiny.gguf"), 128)
    try:
        lg = eng.eval(g["prompt"], 0, 32)
        np.testing.assert_allclose(lg, g["logits"], atol=2e-6)
        gen, _ = eng.greedy(g["hello_ids"], 24, 32)
        np.testing.assert_array_equal(gen, g["hello_gen"])
    finally:
        eng.close()
