"""The grouped tensor-core path's data flow (gemm.cu: k_gemm_tc's operand stages and epilogue, with the
layouts of k_dequant_f16, k_pack_groups and k_pack_slots), modelled on the CPU in float64.

Weights and slot rows are placed tile-major exactly as the kernels place them; every GEMM tile reads
its A stages from the slot tile and its B stages from two weight blocks, forms the 128 x 256
accumulator, and the epilogue maps accumulator columns back to FF / D rows with the row and slot scales
the kernels load: gate/up columns c and c + 64 of each 128-column half are a gate/up pair, down column n
is D row 256 rt + n. The result must equal the same projections computed directly from the unpacked
rows (up to float64 rounding), for every slot of every expert, with an expert that has no slots and
tiles that are partly filled.
"""
import numpy as np

from test_grouped_plan_host import plan, tc_tile, pack_rows
from test_tile_layout_host import tile_off

IDX = np.array([[tile_off(r, k) for k in range(64)] for r in range(128)], np.int64)  # one 128 x 64 stage
assert all((IDX[r] == np.array([tile_off(r, k) for k in range(64)])).all() for r in (0, 77, 127))


def row_offsets(r, K):
    """tile_off(r, i) for i < K, vectorised"""
    i = np.arange(K)
    return (i >> 6) * 8192 + ((r >> 3) * 8 + ((i & 63) >> 3)) * 64 + (r & 7) * 8 + (i & 7)


def untile(buf, base, K):
    """a 128-row tile of K columns stored as K / 64 consecutive core-matrix stages"""
    return np.concatenate([buf[base + kt * 8192 + IDX] for kt in range(K // 64)], axis=1)


def silu_mul(g, u):
    return g / (1.0 + np.exp(-g)) * u


def test_tiles_and_epilogue_reproduce_the_projections():
    rng = np.random.default_rng(5)
    E, D, FF, T = 3, 512, 256, 100
    cnt = np.array([130, 0, 77])
    S = int(cnt.sum())
    offsets, tiles_gu, tiles_dn = plan(cnt, D, FF)
    slot_token = rng.integers(0, T, S)

    # experts as the dequantization leaves them: f16 values, a power-of-two scale per row
    vals = [[(rng.normal(size=shape) / np.sqrt(shape[1])).astype(np.float16) for shape in ((FF, D), (FF, D), (D, FF))]
            for _ in range(E)]
    rs = [2.0 ** rng.integers(-3, 4, 2 * FF + D) for _ in range(E)]  # gate, up, down rows
    w_expert = 3 * FF * D
    wf = np.zeros(E * w_expert, np.float16)
    for e in range(E):
        for c, (m, K) in enumerate(((vals[e][0], D), (vals[e][1], D), (vals[e][2], FF))):
            for row in range(m.shape[0]):
                if c < 2:
                    base, ar = e * w_expert + (row >> 6) * 128 * K, (0 if c == 0 else 64) + (row & 63)
                else:
                    base, ar = e * w_expert + 2 * FF * D + (row >> 7) * 128 * K, row & 127
                wf[base + row_offsets(ar, K)] = m[row]
    true_w = [[vals[e][c].astype(np.float64) * rs[e][c * FF: c * FF + vals[e][c].shape[0], None] for c in range(3)]
              for e in range(E)]

    # token rows as k_token_scale leaves them, packed per slot by the 8-slot row groups
    xh = rng.normal(size=(T, D)).astype(np.float16)
    tscale = 2.0 ** rng.integers(-2, 3, T)
    slot_tiles = (S + 127) // 128 + E

    def pack(rows, scale, K):
        bhi = np.zeros(slot_tiles * 128 * K, np.float16)
        for gw in range(slot_tiles * 16):
            for slot, bt, row in pack_rows(gw, offsets, tiles_gu, E, FF):
                bhi[bt * 128 * K + row_offsets(row, K)] = (
                    rows[slot] if slot is not None else 0)
        return bhi, scale

    bhi, bscale = pack(xh[slot_token], tscale[slot_token], D)

    def run(mode, bhi, bscale):
        K, ncol = (D, FF) if mode == 0 else (FF, D)
        out = np.full((S, ncol), np.nan)
        b = 0
        while (t := tc_tile(mode, b, offsets, tiles_gu, tiles_dn, E, D, FF)) is not None:
            b += 1
            e, rt = t["e"], t["rt"]
            A = untile(bhi, t["btile"] * 128 * K, K).astype(np.float64)
            wb = e * w_expert + (0 if mode == 0 else 2 * FF * D)
            B = np.concatenate([untile(wf, wb + blk * 128 * K, K) for blk in (2 * rt, 2 * rt + 1)]).astype(np.float64)
            acc = A @ B.T  # 128 slots x 256 columns
            r = rs[e]
            for sl in range(t["mc"]):
                bs = bscale[t["m0"] + sl]
                if mode == 0:
                    for qq in range(4):
                        fr, gcol = 128 * rt + 32 * qq, (qq >> 1) * 128 + (qq & 1) * 32
                        for j in range(32):
                            g = acc[sl, gcol + j] * r[fr + j] * bs
                            u = acc[sl, gcol + 64 + j] * r[FF + fr + j] * bs
                            out[t["m0"] + sl, fr + j] = silu_mul(g, u)
                else:
                    for p in range(8):
                        dr = 256 * rt + 32 * p
                        out[t["m0"] + sl, dr: dr + 32] = acc[sl, 32 * p: 32 * p + 32] * r[2 * FF + dr: 2 * FF + dr + 32] * bs
        return out

    h = run(0, bhi, bscale)
    expert_of = np.repeat(np.arange(E), cnt)
    x = xh[slot_token].astype(np.float64) * tscale[slot_token][:, None]
    h_ref = np.stack([silu_mul(true_w[e][0] @ x[s], true_w[e][1] @ x[s]) for s, e in enumerate(expert_of)])
    np.testing.assert_allclose(h, h_ref, rtol=1e-9, atol=1e-12)

    # the down GEMM over h as k_pack_slots leaves it: a power-of-two scale per slot, f16 of h / s
    hs = 2.0 ** np.ceil(np.log2(np.abs(h).max(axis=1) / 2.0 ** 14 + 1e-300))
    hh = (h / hs[:, None]).astype(np.float16)
    bhi_h, _ = pack(hh, None, FF)
    y = run(1, bhi_h, hs)
    hq = hh.astype(np.float64) * hs[:, None]
    y_ref = np.stack([true_w[e][2] @ hq[s] for s, e in enumerate(expert_of)])
    np.testing.assert_allclose(y, y_ref, rtol=1e-9, atol=1e-12)
