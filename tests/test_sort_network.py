"""The routing's warp sorting network (moe.cu: warp_bitonic, warp_merge_runs8, run8_slot), modelled
lane by lane on the CPU.

Top-k routing of one token sorts 32 keys per warp, then merges the four warps' top-8 runs with only the
network's last two levels (16, 32), the runs stored in the lane layout the network has after level 8
(run w in lanes 8w..8w+7, reversed for odd w); the k <= 8 picks are then ordered by levels 2..8 alone.
Both shortcuts must give exactly the sequence a full 32-key sort gives: the top-k ids and weights depend
on it bit for bit.
"""
import numpy as np
import pytest


def bitonic(keys, k0, k1):
    """Levels k0..k1 of the network as the kernel runs them: lane l exchanges with lane l ^ j, keeps the
    larger key when (l & j == 0) == (l & k == 0), else the smaller."""
    v = list(keys)
    k = k0
    while k <= k1:
        j = k >> 1
        while j > 0:
            o = [v[l ^ j] for l in range(32)]
            v = [(max if ((l & j) == 0) == ((l & k) == 0) else min)(v[l], o[l]) for l in range(32)]
            j >>= 1
        k <<= 1
    return v


def run8_slot(w, i):
    return 8 * w + (7 - i if w & 1 else i)


@pytest.mark.parametrize("seed", range(40))
def test_merge_of_four_sorted_runs_is_a_full_sort(seed):
    rng = np.random.default_rng(seed)
    # 4 warps x 32 keys: distinct 64-bit-style keys, with exact duplicates and zeros (absent entries)
    keys = [int(x) for x in rng.integers(0, 1 << 20, 128)]
    keys[:10] = [keys[10]] * 10
    keys[100:] = [0] * 28
    runs = [bitonic(keys[32 * w: 32 * w + 32], 2, 32)[:8] for w in range(4)]
    assert all(r == sorted(r, reverse=True) for r in runs)
    cand = [0] * 32
    for w in range(4):
        for i in range(8):
            cand[run8_slot(w, i)] = runs[w][i]
    merged = bitonic(cand, 16, 32)
    assert merged == bitonic(cand, 2, 32) == sorted(cand, reverse=True)
    assert merged[:8] == sorted(keys, reverse=True)[:8]  # the token's top 8 of all 128 entries


@pytest.mark.parametrize("k", [1, 2, 4, 7, 8])
@pytest.mark.parametrize("seed", range(10))
def test_first_three_levels_sort_up_to_eight_keys(k, seed):
    rng = np.random.default_rng(100 + seed)
    keys = [int(x) + 1 for x in rng.integers(0, 1 << 30, k)] + [0] * (32 - k)
    out = bitonic(keys, 2, 8)
    assert out[:8] == bitonic(keys, 2, 32)[:8] == sorted(keys, reverse=True)[:8]
