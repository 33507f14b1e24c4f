"""eahmmf_cuda_gemv_static (the GEMV whose workspace is a fixed device array) against eahmmf_cuda_gemv.

Collected last (file name) so it also runs after every other test has used the device; it creates all
of its own buffers, so it passes alone as well. Two calls in a row go through the same static array:
the second call (another type and row length) must not see anything the first one left behind.
"""
import numpy as np
import pytest

import eahmmf_b200 as eb
import synth

pytestmark = pytest.mark.gpu


def _matrix(qtype, K, rows, seed):
    blck, _ = synth.BLOCK[qtype]
    return synth.quant_blocks(qtype, rows * K // blck, synth._rng(seed, qtype), 0.01).reshape(rows, -1)


def _pair(torch, qtype, K, rows, nb, seed):
    W = _matrix(qtype, K, rows, seed)
    x = synth.activations(nb, K, seed=seed + 1)
    return torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda(), W.shape[1]


def test_static_workspace_matches_gemv_on_two_calls_in_a_row():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    # call 1: Q4_K, long rows, 7 tokens (two passes); call 2: Q6_K, shorter rows, 3 tokens, accumulate
    cases = [(synth.Q4_K, 4096, 512, 7, False, 11), (synth.Q6_K, 768, 2048, 3, True, 12)]
    for qtype, K, rows, nb, acc, seed in cases:
        dw, dx, rb = _pair(torch, qtype, K, rows, nb, seed)
        base = torch.from_numpy(synth.activations(nb, rows, seed=seed + 2)).cuda()
        want = base.clone()
        got = base.clone()
        assert eb.gemv(dw, qtype, K, rows, rb, dx, want, accumulate=acc) == eb.ST_OK
        assert eb.gemv_static(dw, qtype, K, rows, rb, dx, got, accumulate=acc) == eb.ST_OK
        torch.cuda.synchronize()
        assert torch.equal(got, want), (qtype, K, float((got - want).abs().max()))


def test_static_workspace_rejects_rows_longer_than_its_limit():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    K = eb.GEMV_STATIC_MAX_NE0 + 256
    dw = torch.zeros(4 * (K // 256) * 144, dtype=torch.uint8, device="cuda")
    dx = torch.zeros((1, K), device="cuda")
    dy = torch.full((1, 4), 7.0, device="cuda")
    assert eb.gemv_static(dw, synth.Q4_K, K, 4, (K // 256) * 144, dx, dy) == eb.ST_CAPACITY
    torch.cuda.synchronize()
    assert bool((dy == 7.0).all())  # nothing was launched
