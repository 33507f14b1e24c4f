"""The GPU sampler (sample.cu: eahmmf_cuda_sample, and the engine's sampled generation) against the
reference's Sampler::sample (qwen3moe.cpp:1090-1130) compiled from its sources (oracle/_ref).

* One row at a time: seeded random logits (vocabularies of 512 and 151,936; planted ties at the top for
  the first-maximum case; repeated history tokens), every parameter path (greedy, top-k 1..256, top-p, min-p, temperature,
  repetition penalty with duplicate history entries): the token exact and the penalised logits bitwise
  equal. The uniform u is the first draw of the reference's stream for the same seed (eahmmf_rng).
* The engine's generate loop with the sampler against the reference's generate loop on the same model,
  prompt and seed: the generated ids exact (the logits themselves agree to ~1e-6, far inside the gaps the
  draws land in).
"""
import os

import numpy as np
import pytest

import eahmmf_b200 as eb
import synth

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = os.path.join(ROOT, "tests", "golden", "ref_tiny.gguf")

CASES = [
    dict(temp=0.0, top_p=0.8, min_p=0.0, rep=1.05, top_k=20, rep_n=64),
    dict(temp=0.7, top_p=0.8, min_p=0.0, rep=1.05, top_k=20, rep_n=64),
    dict(temp=1.0, top_p=1.0, min_p=0.0, rep=1.0, top_k=40, rep_n=64),
    dict(temp=0.6, top_p=0.95, min_p=0.05, rep=1.3, top_k=256, rep_n=16),
    dict(temp=1.5, top_p=0.5, min_p=0.0, rep=0.9, top_k=1, rep_n=64),
    dict(temp=0.3, top_p=1.0, min_p=0.2, rep=1.1, top_k=128, rep_n=200),
]


@pytest.fixture(scope="module")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    eb.lib()
    return torch.device("cuda", 0)


@pytest.mark.parametrize("n", [512, 151936])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_sample_row_matches_reference(dev, ref, n, case):
    import torch
    P = CASES[case]
    params = eb.sampler_params(**P)
    rng = np.random.default_rng(1000 * case + n)
    ws = torch.empty(int(eb.lib().eahmmf_cuda_sample_workspace_bytes(n)), dtype=torch.uint8, device=dev)
    tok_d = torch.zeros(1, dtype=torch.int32, device=dev)
    for trial in range(12):
        lg = (rng.normal(0, 2.0, n) * (1 + trial % 3)).astype(np.float32)
        if trial % 4 == 1 and P["temp"] <= 0:
            # ties at the top: the first maximum is defined (std::max_element); std::partial_sort leaves the
            # order of equal logits unspecified, so sampled cases keep distinct values
            lg[rng.integers(0, n, 5)] = lg.max()
        hist = rng.integers(0, n, int(rng.integers(0, 3 * P["rep_n"] // 2 + 2))).astype(np.int32)
        if len(hist) > 3:
            hist[1] = hist[0] = int(np.argmax(lg))  # a repeated, top-ranked history token
        seed = 7919 * trial + case
        u = float(eb.Rng(seed).uniform())
        want_tok, want_lg = ref.sample(lg, hist, P["temp"], P["top_p"], P["min_p"], P["rep"], P["top_k"], P["rep_n"],
                                       seed)
        d_lg = torch.from_numpy(lg.copy()).to(dev)
        d_h = torch.from_numpy(hist).to(dev) if len(hist) else None
        rc = eb.sample(d_lg, d_h, params, u, tok_d, ws)
        torch.cuda.synchronize()
        assert rc == 0
        np.testing.assert_array_equal(d_lg.cpu().numpy(), want_lg, err_msg=f"penalised logits, trial {trial}")
        assert int(tok_d.item()) == want_tok, (trial, P)


def test_sample_rejects_unsupported_top_k(dev):
    import torch
    d_lg = torch.zeros(100, device=dev)
    tok = torch.zeros(1, dtype=torch.int32, device=dev)
    assert eb.sample(d_lg, None, eb.sampler_params(top_k=0), 0.5, tok) == eb.ST_BAD_ARG
    assert eb.sample(d_lg, None, eb.sampler_params(top_k=257), 0.5, tok) == eb.ST_BAD_ARG
    assert eb.sample(d_lg, None, eb.sampler_params(temp=0.0, top_k=0), 0.5, tok) == 0  # greedy: any top_k


@pytest.fixture(scope="module")
def kquant_path(tmp_path_factory):
    return synth.write_gguf(str(tmp_path_factory.mktemp("ks") / "ks.gguf"), synth.config_kquant_small())


@pytest.mark.parametrize("model", ["tiny", "kquant"])
@pytest.mark.parametrize("case", [1, 3])
def test_engine_sampled_generation_matches_reference(dev, ref, kquant_path, model, case):
    path = TINY if model == "tiny" else kquant_path
    P = CASES[case]
    g = synth._rng(77, case).integers(0, 250, 20).astype(np.int32)
    want = ref.engine(path, 128)
    want_ids = want.generate(g, 40, P, seed=42 + case, n_batch=32)
    want.close()
    e = eb.Engine(path, 128)
    try:
        assert e.sampler(seed=42 + case, **P) == 0
        assert e.greedy(g, 4, 32)[0] == eb.ST_BAD_ARG  # greedy refuses while a sampler is configured
        rc, got = e.generate(g, 40, 32)
        assert rc == 0
        np.testing.assert_array_equal(got, want_ids)
        assert e.graph_nodes() > 0  # the sampled steps ran as the captured graph
        # back to the first maximum: the greedy generation of before
        assert e.sampler() == 0
        rc, gg, _ = e.greedy(g, 8, 32)
        assert rc == 0
        want2 = ref.engine(path, 128)
        ref_greedy, _ = want2.greedy(g, 8, 32)
        want2.close()
        np.testing.assert_array_equal(gg, ref_greedy)
    finally:
        e.close()
