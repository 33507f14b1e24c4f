"""The device-resident engine (eahmmf_engine_*, engine.cu + decode.cu) against the reference engine.

Pins: the reference tiny model's golden outputs (ref_tiny.npz: prompt logits, 24-token greedy
generation of "hello world ab ab", the routing trace of a prompt + 12 decode steps) and the config-1
synthetic model's golden outputs (config1.npz: 32 greedy tokens, first logits, routing trace) and a
small all-K-quant model's (kquant_small.npz: prompt logits and routing trace, 16 greedy tokens), all
produced by the reference engine (tests/golden/make_fixtures.py). Expected: greedy token ids and
routed expert ids bit-exact; logits within 1e-4 of the largest |logit| (the reference's own GPU/CPU
tolerance, qwen3moe.cpp:449-458) with the same argmax; routing weights within 1e-5 relative or 1e-6
absolute (a weight w = r / sum r inherits the logits' absolute rounding as relative error, which
dominates for small w).
"""
import hashlib
import json
import os

import numpy as np
import pytest

import eahmmf_b200 as eb
import synth

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = os.path.join(ROOT, "tests", "golden", "ref_tiny.gguf")
ST_OK, ST_BAD_ARG = 0, 1


@pytest.fixture(scope="module")
def gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    eb.lib()


def rel_max(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


@pytest.fixture(scope="module")
def tiny(gpu):
    e = eb.Engine(TINY, 128)
    yield e
    e.close()


@pytest.fixture(scope="module")
def config1(gpu, tmp_path_factory):
    cfg = synth.config1_tiny()
    path = synth.write_gguf(str(tmp_path_factory.mktemp("c1") / "c1.gguf"), cfg)
    meta = json.load(open(os.path.join(ROOT, "tests", "golden", "fixtures.json")))
    h = hashlib.sha256(open(path, "rb").read()).hexdigest()
    assert h == meta["config1_sha256"], "synthetic config-1 GGUF differs from the one the fixture was made from"
    e = eb.Engine(path, 512)
    yield e
    e.close()


def test_engine_dims(tiny):
    assert tiny.dims == dict(n_layer=2, D=256, n_head=4, n_kv=2, hd=64, n_expert=8, n_used=2, FF=256, n_vocab=260,
                             n_ctx=128, n_embd=260)


def test_engine_prompt_logits_match_reference(tiny, golden):
    g = golden("ref_tiny.npz")
    rc, lg = tiny.eval(g["prompt"], 0, 32)
    assert rc == ST_OK
    assert rel_max(lg, g["logits"]) < 1e-4
    assert int(lg.argmax()) == int(g["logits"].argmax())


def test_engine_logits_independent_of_batching(tiny, golden):
    """Per-token results do not depend on how the prompt is split into forward passes."""
    g = golden("ref_tiny.npz")
    ref = None
    for nb in (32, 4, 1, 7):
        rc, lg = tiny.eval(g["prompt"], 0, nb)
        assert rc == ST_OK
        if ref is None:
            ref = lg
        else:
            np.testing.assert_array_equal(lg, ref)
    assert rel_max(ref, g["logits_b4"]) < 1e-4


def test_engine_greedy_hello_matches_reference(tiny, golden):
    g = golden("ref_tiny.npz")
    rc, out, lg = tiny.greedy(g["hello_ids"], 24, 32, want_logits=True)
    assert rc == ST_OK
    np.testing.assert_array_equal(out, g["hello_gen"])


def test_engine_routing_trace_matches_reference(tiny, golden):
    """Prompt in passes of 4 tokens, then 12 single-token steps, as the residency suite's inference
    (tests/test_eahmmf.cpp:36-54); the routing trace of every layer and pass, bit-exact ids."""
    g = golden("ref_tiny.npz")
    tiny.trace(True)
    try:
        rc, lg = tiny.eval(g["prompt"], 0, 4)
        assert rc == ST_OK
        ids, pos = [], len(g["prompt"])
        for _ in range(12):
            t = int(lg.argmax())
            ids.append(t)
            rc, lg = tiny.eval([t], pos, 1)
            assert rc == ST_OK
            pos += 1
        tr_ids, tr_w = tiny.trace_get()
    finally:
        tiny.trace(False)
    np.testing.assert_array_equal(ids, g["gen12"])
    np.testing.assert_array_equal(tr_ids, g["trace_ids"])
    np.testing.assert_allclose(tr_w, g["trace_w"], rtol=1e-5, atol=1e-6)


def test_engine_decode_continues_greedy(tiny, golden):
    g = golden("ref_tiny.npz")
    rc, first, _ = tiny.greedy(g["hello_ids"], 10, 32)
    assert rc == ST_OK
    rc, more, ms = tiny.decode(14)
    assert rc == ST_OK and ms > 0
    np.testing.assert_array_equal(np.concatenate([first, more]), g["hello_gen"])


def test_engine_config1_greedy_and_trace(config1, golden):
    g = golden("config1.npz")
    config1.trace(True)
    try:
        rc, out, lg = config1.greedy(g["prompt"], 32, 16, want_logits=True)
        tr_ids, tr_w = config1.trace_get()
    finally:
        config1.trace(False)
    assert rc == ST_OK
    assert rel_max(lg, g["logits"]) < 1e-4
    np.testing.assert_array_equal(out, g["gen"])
    np.testing.assert_array_equal(tr_ids, g["trace_ids"])
    np.testing.assert_allclose(tr_w, g["trace_w"], rtol=1e-5, atol=1e-6)


def test_engine_graph_and_eager_steps_agree(config1, golden):
    """The captured decode step (greedy without trace) and eager steps (with trace) give the same tokens."""
    g = golden("config1.npz")
    rc, out, _ = config1.greedy(g["prompt"], 32, 16)
    assert rc == ST_OK
    np.testing.assert_array_equal(out, g["gen"])


@pytest.fixture(scope="module")
def kquant(gpu, tmp_path_factory):
    cfg = synth.config_kquant_small()
    path = synth.write_gguf(str(tmp_path_factory.mktemp("ks") / "ks.gguf"), cfg)
    meta = json.load(open(os.path.join(ROOT, "tests", "golden", "fixtures.json")))
    h = hashlib.sha256(open(path, "rb").read()).hexdigest()
    assert h == meta["kquant_small_sha256"], "synthetic K-quant GGUF differs from the one the fixture was made from"
    e = eb.Engine(path, 256)
    yield e
    e.close()


def test_engine_kquant_prompt_matches_reference(kquant, golden):
    """Every projection K-quant: prompt passes of 32 tokens go through the many-token tensor-core GEMM,
    single tokens through the GEMV; logits, routing trace and greedy ids against the reference engine."""
    g = golden("kquant_small.npz")
    kquant.trace(True)
    try:
        rc, lg = kquant.eval(g["prompt"], 0, 32)
        tr_ids, tr_w = kquant.trace_get()
    finally:
        kquant.trace(False)
    assert rc == ST_OK
    assert rel_max(lg, g["logits"]) < 1e-4
    assert int(lg.argmax()) == int(g["logits"].argmax())
    np.testing.assert_array_equal(tr_ids, g["trace_ids"])
    np.testing.assert_allclose(tr_w, g["trace_w"], rtol=1e-5, atol=1e-6)
    rc, out, _ = kquant.greedy(g["prompt"], 16, 32)
    assert rc == ST_OK
    np.testing.assert_array_equal(out, g["gen"])


def test_engine_kquant_logits_independent_of_batching(kquant, golden):
    """Per-token results are bitwise the same whether a token goes through the many-token GEMM (passes
    of 5..64 tokens) or the GEMV (passes of 1..4)."""
    g = golden("kquant_small.npz")
    ref = None
    for nb in (40, 4, 1, 13, 64, 5):
        rc, lg = kquant.eval(g["prompt"], 0, nb)
        assert rc == ST_OK
        if ref is None:
            ref = lg
        else:
            np.testing.assert_array_equal(lg, ref, err_msg=f"passes of {nb}")


def test_engine_rejects_bad_arguments(tiny):
    assert tiny.eval([1, 2, 3], 0, 0)[0] == ST_BAD_ARG
    assert tiny.eval([1, 2, 3], 127, 4)[0] == ST_BAD_ARG  # past n_ctx
    assert tiny.greedy([1], 200, 4)[0] == ST_BAD_ARG
    with pytest.raises(RuntimeError, match="cannot open"):
        eb.Engine(os.path.join(ROOT, "does-not-exist.gguf"), 64)
