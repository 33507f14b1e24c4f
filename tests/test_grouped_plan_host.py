"""The grouped tensor-core path's work plan (moe.cu: k_route_big's slot counts, k_plan_big; gemm.cu:
tc_tile, k_pack_groups, k_pack_slots; capi.cu: the launch bounds), modelled on the CPU.

k_plan_big turns the per-expert slot counts into slot offsets and the two GEMMs' tile prefixes (row
tiles fastest, then 128-slot tiles); every GEMM CTA finds its tile by binary search over a prefix, and
the pack kernels find the slot tile of their 8-slot row group the same way. The model checks that the
gate/up tiles cover every (slot, 128 FF rows) once and the down tiles every (slot, 256 D rows) once,
that a slot's packed row sits where the GEMM reads it (tile btile, row slot - m0), and that the grids
the host sizes from S / 128 + E slot tiles cover the plan.
"""
import numpy as np
import pytest

GU_TILE_ROWS, DN_TILE_ROWS = 128, 256


def plan(cnt, D, FF):
    """k_plan_big: exclusive prefixes of the counts and of ceil(count / 128), times the row tiles."""
    cnt = np.asarray(cnt, np.int64)
    nt = (cnt + 127) // 128
    offsets = np.concatenate([[0], np.cumsum(cnt)])
    toff = np.concatenate([[0], np.cumsum(nt)])
    return offsets, (FF // GU_TILE_ROWS) * toff, (D // DN_TILE_ROWS) * toff


def find(prefix, b, E):
    """largest e with prefix[e] <= b (the kernels' binary search over [0, E))"""
    lo, hi = 0, E
    while hi - lo > 1:
        mid = (lo + hi) >> 1
        if prefix[mid] <= b:
            lo = mid
        else:
            hi = mid
    return lo


def tc_tile(mode, b, offsets, tiles_gu, tiles_dn, E, D, FF):
    off = tiles_gu if mode == 0 else tiles_dn
    if b >= off[E]:
        return None
    e = find(off, b, E)
    RT = FF // GU_TILE_ROWS if mode == 0 else D // DN_TILE_ROWS
    local = b - off[e]
    st = local // RT
    m0 = offsets[e] + 128 * st
    return dict(e=e, rt=local - st * RT, m0=m0, mc=min(128, offsets[e + 1] - m0),
                btile=tiles_gu[e] // (FF // GU_TILE_ROWS) + st)


def pack_rows(gw, offsets, tiles_gu, E, FF):
    """k_pack_groups / k_pack_slots warp gw: (slot, tile, row) of its 8 rows, None past the expert's slots"""
    RT = FF // GU_TILE_ROWS
    bt, grp = gw >> 4, gw & 15
    if bt * RT >= tiles_gu[E]:
        return []
    e = find(tiles_gu, bt * RT, E)
    cnt = offsets[e + 1] - offsets[e]
    j0 = 128 * (bt - tiles_gu[e] // RT) + 8 * grp
    if j0 >= cnt:
        return []
    return [(offsets[e] + j0 + r if j0 + r < cnt else None, bt, 8 * grp + r) for r in range(8)]


CASES = {
    "zipf_128": (128, 2048, 768, None),
    "empty_and_edges": (16, 512, 256, [0, 1, 127, 128, 129, 0, 255, 256, 257, 0, 0, 383, 1, 2, 0, 500]),
    "wide_235b": (128, 4096, 1536, None),
    "odd_expert_count": (100, 1024, 512, None),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_tiles_cover_every_slot_once_and_packed_rows_sit_where_the_gemm_reads(name):
    E, D, FF, cnt = CASES[name]
    rng = np.random.default_rng(7)
    if cnt is None:  # top-8 of log-Zipf(1.1)-biased logits over 2,048 tokens
        T, K = 2048, 8
        bias = -1.1 * np.log(np.arange(1, E + 1))
        lg = rng.normal(size=(T, E)) + bias[rng.permutation(E)]
        top = np.argsort(-lg, axis=1)[:, :K]
        cnt = np.bincount(top.ravel(), minlength=E)
    cnt = np.asarray(cnt, np.int64)
    S = int(cnt.sum())
    offsets, tiles_gu, tiles_dn = plan(cnt, D, FF)

    slot_tiles = (S + 127) // 128 + E  # capi.cu's bound on the sum over experts of ceil(m_e / 128)
    assert tiles_gu[E] <= (FF // GU_TILE_ROWS) * slot_tiles  # the launch bounds cover the plan
    assert tiles_dn[E] <= (D // DN_TILE_ROWS) * slot_tiles

    # gate/up and down tiles: every (slot, row tile) exactly once
    for mode, RT, prefix in ((0, FF // GU_TILE_ROWS, tiles_gu), (1, D // DN_TILE_ROWS, tiles_dn)):
        seen = np.zeros((S, RT), np.int32)
        b = 0
        while True:
            t = tc_tile(mode, b, offsets, tiles_gu, tiles_dn, E, D, FF)
            if t is None:
                break
            assert 0 < t["mc"] <= 128
            assert offsets[t["e"]] <= t["m0"] and t["m0"] + t["mc"] <= offsets[t["e"] + 1]
            seen[t["m0"]: t["m0"] + t["mc"], t["rt"]] += 1
            b += 1
        assert b == prefix[E]
        assert (seen == 1).all(), name

    # the pack kernels' rows: every slot once, at (btile, slot - m0) of the gate/up tiles that read it
    where = {}
    for gw in range(slot_tiles * 16):
        for slot, bt, row in pack_rows(gw, offsets, tiles_gu, E, FF):
            if slot is not None:
                assert slot not in where
                where[slot] = (bt, row)
    assert sorted(where) == list(range(S))
    for b in range(int(tiles_gu[E])):
        t = tc_tile(0, b, offsets, tiles_gu, tiles_dn, E, D, FF)
        for sl in range(t["mc"]):
            assert where[t["m0"] + sl] == (t["btile"], sl)
    # the down tiles read the same packed tiles (h rows, packed by k_pack_slots with the same map)
    for b in range(int(tiles_dn[E])):
        t = tc_tile(1, b, offsets, tiles_gu, tiles_dn, E, D, FF)
        for sl in range(t["mc"]):
            assert where[t["m0"] + sl] == (t["btile"], sl)


def test_block_gathered_slot_counts_give_every_slot_a_place():
    """k_route_big: each block of 4 tokens counts its slots per expert with shared-memory atomics, then
    reserves its range of each expert's slots with one global atomic; a slot's place is the block's base
    plus its place in the block. Whatever order the atomics land in, k_scatter_big's slots
    offsets[e] + local are a permutation of 0..S-1 and each expert's slots hold exactly its tokens."""
    rng = np.random.default_rng(11)
    E, K, T, TPB = 64, 8, 203, 4  # T not a multiple of the block's 4 tokens
    bias = -1.1 * np.log(np.arange(1, E + 1))
    ids = np.argsort(-(rng.normal(size=(T, E)) + bias), axis=1)[:, :K]
    for trial in range(5):
        cnt = np.zeros(E, np.int64)  # the global counters
        local = np.full((T, K), -1, np.int64)
        blocks = list(range((T + TPB - 1) // TPB))
        rng.shuffle(blocks)  # blocks reach their global atomics in any order
        for blk in blocks:
            toks = range(blk * TPB, min(T, (blk + 1) * TPB))
            s_cnt = np.zeros(E, np.int64)
            pos = {}
            order = [(t, k) for t in toks for k in range(K)]
            rng.shuffle(order)  # shared-memory atomics in any order
            for t, k in order:
                pos[t, k] = s_cnt[ids[t, k]]
                s_cnt[ids[t, k]] += 1
            base = np.zeros(E, np.int64)
            for e in rng.permutation(E):  # one global atomic per expert with slots in the block
                if s_cnt[e]:
                    base[e] = cnt[e]
                    cnt[e] += s_cnt[e]
            for (t, k), p in pos.items():
                local[t, k] = base[ids[t, k]] + p
        offsets = np.concatenate([[0], np.cumsum(cnt)])
        slot = offsets[ids] + local
        assert sorted(slot.ravel().tolist()) == list(range(T * K))
        for e in range(E):
            mine = slot[ids == e]
            assert mine.min(initial=offsets[e]) >= offsets[e] and mine.max(initial=offsets[e + 1] - 1) < offsets[e + 1]
