"""Host side of the GPU sampler: the random stream the library draws its uniforms from
(eahmmf_rng_create / eahmmf_rng_uniform) is the reference sampler's -- std::mt19937_64 seeded as
Sampler::rng.seed(seed) (qwen3moe.cpp:1231), one std::uniform_real_distribution<float>(0, 1) draw per
sampled token (:1125) -- checked bit for bit against the compiled reference's own draws. No GPU needed."""
import numpy as np
import pytest

import eahmmf_b200 as eb


@pytest.mark.parametrize("seed", [0, 42, 1234567890123, 2**63 + 5])
def test_rng_matches_reference_stream(ref, seed):
    want = ref.uniform(seed, 200)
    r = eb.Rng(seed)
    got = np.array([r.uniform() for _ in range(200)], np.float32)
    np.testing.assert_array_equal(got, want)
    assert np.all((got >= 0) & (got <= 1))


def test_sampler_defaults_are_the_reference_cli_defaults():
    p = eb.sampler_params()
    assert (round(p.temp, 6), round(p.top_p, 6), p.min_p, round(p.rep, 6), p.top_k, p.rep_n) == (0.7, 0.8, 0.0, 1.05, 20, 64)
