"""Expert residency beyond HBM (eahmmf_engine_load_budget): the engine with only a device cache of whole
experts -- one layer's worth, or a few layers' -- against the fully resident engine on the same model and
prompt: the prompt logits bitwise equal and the greedy tokens exact (the kernels read the same expert
bytes from cache slots), with the cache counters showing misses and, where the small model's layers
cannot all stay resident, evictions, prefetch fills and hits on prefetched experts; the resident copies pass the hash64 verify. Models: the small all-K-quant model and
the Qwen3-30B-A3B shape reduced to 4 layers.
"""
import os

import numpy as np
import pytest

import eahmmf_b200 as eb
import synth

pytestmark = pytest.mark.gpu


def footprint(cfg):
    a256 = lambda v: (v + 255) // 256 * 256  # noqa: E731
    tg, tu, td = cfg.expert_types
    g = cfg.FF * synth.row_bytes(tg, cfg.D)
    u = cfg.FF * synth.row_bytes(tu, cfg.D)
    d = cfg.D * synth.row_bytes(td, cfg.FF)
    return a256(a256(a256(g) + u) + d)


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    d = tmp_path_factory.mktemp("res")
    ks = synth.config_kquant_small()
    c4 = synth.config4_30b(n_layer=4)
    return {"kquant": (synth.write_gguf(str(d / "ks.gguf"), ks), ks),
            "c4": (synth.cached_gguf(c4, str(d), workers=max(1, min(16, os.cpu_count() or 1))), c4)}


@pytest.mark.parametrize("model,layers_worth", [("kquant", 1.0), ("kquant", 2.5), ("c4", 1.0), ("c4", 1.5)])
def test_budgeted_engine_matches_resident(models, model, layers_worth):
    path, cfg = models[model]
    vocab = min(cfg.n_vocab, 1000)
    prompt = synth._rng(11, 3).integers(0, vocab, 40).astype(np.int32)
    n_gen = 20
    full = eb.Engine(path, 128)
    rc, want, want_lg = full.greedy(prompt, n_gen, 32, want_logits=True)
    assert rc == 0
    full.close()
    budget = int(layers_worth * cfg.n_expert * footprint(cfg))
    e = eb.Engine(path, 128, expert_vram_bytes=budget)
    try:
        rc, got, got_lg = e.greedy(prompt, n_gen, 32, want_logits=True)
        assert rc == 0
        np.testing.assert_array_equal(got_lg, want_lg)  # bitwise: the same kernels over the same bytes
        np.testing.assert_array_equal(got, want)
        st = e.cache_stats()
        assert st["slots"] == int(layers_worth * cfg.n_expert)
        assert st["misses"] > 0 and st["bytes_h2d"] > 0
        if model == "kquant" and layers_worth == 1.0:  # its layers' routed experts cannot all stay at once
            assert st["evictions"] > 0 and st["prefetched"] > 0
        # a second generation: the decode steps' prefetches of the next layer's last routed experts hit
        rc, got2, _ = e.greedy(prompt, n_gen, 32)
        assert rc == 0
        np.testing.assert_array_equal(got2, want)
        if model == "kquant" and layers_worth == 1.0:
            assert e.cache_stats()["prefetch_hits"] > 0
        rc, n, bad = e.verify()
        assert rc == 0 and n > 0 and bad == 0
    finally:
        e.close()


def test_budget_below_one_layer_is_refused(models):
    path, cfg = models["kquant"]
    with pytest.raises(RuntimeError, match="below one layer"):
        eb.Engine(path, 64, expert_vram_bytes=(cfg.n_expert - 1) * footprint(cfg))
