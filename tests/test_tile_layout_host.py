"""The grouped tensor-core path's expert layout and decode (gemm.cu: k_dequant_f16, dq_sb_k45, dq_sb_q6k,
kq_bound, tile_off), modelled lane by lane on the CPU.

Every active expert's rows are decoded once to f16, each row scaled by a power of two taken from a bound
read off its super-block headers, and stored tile-major in the tensor cores' K-major core-matrix order: a
128-row tile's 64-element K stages are consecutive 128 x 64 blocks, element (r, k) of a stage at
((r / 8) * 8 + (k % 64) / 8) * 64 + (r % 8) * 8 + k % 8. A warp decodes 8 rows; lane l takes row l / 4
and the 16 elements 16 (l % 4) .. +15 of each 64-element chunk, a whole super-block (four chunks) at a
time, the header's scale and min picked by shifts of its words. The model follows that order and those
shifts and must give, bit for bit, the f16 of the oracle's decoder (qwen3moe.cpp:133-202) times the
row's scale, at the place the tensor cores read it: gate/up blocks of 64 gate rows then the same 64 up
rows, down blocks of 128 rows.
"""
import numpy as np
import pytest

import synth

F32 = np.float32


def words(b: np.ndarray, off: int, n: int = 4) -> list:
    """n little-endian 32-bit words at byte off (any alignment)."""
    return [int.from_bytes(bytes(b[off + 4 * i: off + 4 * i + 4]), "little") for i in range(n)]


def f16_bits(v: int) -> F32:
    return F32(np.array([v & 0xFFFF], np.uint16).view(np.float16)[0])


def fma32(a: F32, b: F32, c: F32) -> F32:
    # a * b is exact in fp32 here (<= 22 significant bits), so one rounding of the exact sum is the fma
    return F32(np.float64(a) * np.float64(b) + np.float64(c))


def lane_sb_k45(b: np.ndarray, q5: bool, kq: int, inv: F32) -> dict:
    """dq_sb_k45: this lane's 4 x 16 values of a Q4_K / Q5_K super-block, by element index."""
    hi, l0 = kq >> 5, kq & 31
    x, y, z, w = words(b, 0)
    dh, mh = f16_bits(x), f16_bits(x >> 16)
    ha = words(b, 16 + l0) if q5 else [0, 0, 0, 0]
    out = {}
    for c in range(4):
        j, sh = 2 * c + hi, 16 * (c & 1) + 8 * hi
        if c < 2:
            sc, mn = (y >> sh) & 63, (z >> sh) & 63
        else:
            bw, by, bz = (w >> sh) & 0xFF, (y >> sh) & 0xFF, (z >> sh) & 0xFF
            sc, mn = (bw & 0x0F) | ((by >> 6) << 4), (bw >> 4) | ((bz >> 6) << 4)
        d = F32(F32(dh * F32(sc)) * inv)
        mo = -F32(F32(mh * F32(mn)) * inv)
        qa = words(b, (48 if q5 else 16) + 32 * c + l0)
        for wi in range(4):
            nib = (qa[wi] >> (4 * hi)) & 0x0F0F0F0F
            if q5:
                nib |= ((ha[wi] >> j) & 0x01010101) << 4
            for k in range(4):
                out[64 * c + kq + 4 * wi + k] = fma32(d, F32((nib >> (8 * k)) & 0xFF), mo)
    return out


def lane_sb_q6k(b: np.ndarray, kq: int, inv: F32) -> dict:
    """dq_sb_q6k: chunks 2 h and 2 h + 1 from the same low-bit and high-bit words."""
    hi, l0 = kq >> 5, kq & 31
    dd = f16_bits(int(b[208]) | int(b[209]) << 8)
    scl = b[192:208].view(np.int8)
    out = {}
    for h in range(2):
        lw = words(b, 64 * h + kq)
        hw = words(b, 128 + 32 * h + l0)
        for cl in range(2):
            c, quad = 2 * h + cl, 2 * cl + hi
            ds = F32(F32(dd * F32(scl[8 * h + (l0 >> 4) + 2 * quad])) * inv)
            for wi in range(4):
                v = ((lw[wi] >> 4) if cl else lw[wi]) & 0x0F0F0F0F
                v |= ((hw[wi] >> (2 * quad)) & 0x03030303) << 4
                for k in range(4):
                    out[64 * c + kq + 4 * wi + k] = F32(ds * F32(((v >> (8 * k)) & 0xFF) - 32))
    return out


def kq_bound(b: np.ndarray, qtype: int) -> F32:
    """kq_bound: an upper bound of |y| over the super-block, from its header alone."""
    if qtype == synth.Q6_K:
        ms = int(np.max(np.abs(b[192:208].view(np.int8).astype(np.int32))))
        return F32(F32(abs(f16_bits(int(b[208]) | int(b[209]) << 8)) * F32(ms)) * F32(32))
    x, y, z, w = words(b, 0)
    d, dm = abs(f16_bits(x)), abs(f16_bits(x >> 16))
    qmax = F32(31 if qtype == synth.Q5_K else 15)
    scales = [int(v) for v in b[4:16]]
    m = F32(0)
    for j in range(8):
        if j < 4:
            sc, mn = scales[j] & 63, scales[j + 4] & 63
        else:
            sc = (scales[j + 4] & 0x0F) | ((scales[j - 4] >> 6) << 4)
            mn = (scales[j + 4] >> 4) | ((scales[j] >> 6) << 4)
        m = max(m, F32(F32(F32(d * F32(sc)) * qmax) + F32(dm * F32(mn))))
    return m


def pow2_scale(m: F32) -> F32:
    """The power of two that brings max|y| into [2^13, 2^14) (1 for a zero row)."""
    if not (m > 0) or not np.isfinite(m):
        return F32(1)
    _, e = np.frexp(m)
    return F32(np.ldexp(1.0, int(e) - 14))


def tile_off(r: int, k: int) -> int:
    return (k >> 6) * (128 * 64) + ((r >> 3) * 8 + ((k & 63) >> 3)) * 64 + (r & 7) * 8 + (k & 7)


def decode_rows(raw: np.ndarray, qtype: int, K: int):
    """The rows of one matrix as k_dequant_f16 leaves them: f16 values and their scales."""
    bsz = synth.BLOCK[qtype][1]
    rows = raw.shape[0]
    vals = np.zeros((rows, K), np.float16)
    scales = np.zeros(rows, np.float32)
    for r in range(rows):
        row = raw[r]
        s = pow2_scale(max(kq_bound(row[sb * bsz:(sb + 1) * bsz], qtype) for sb in range(K // 256)))
        inv, scales[r] = F32(1) / s, s
        for lane4 in range(4):  # the row's four lanes
            kq = 16 * lane4
            for sb in range(K // 256):
                blk = row[sb * bsz:(sb + 1) * bsz]
                got = lane_sb_q6k(blk, kq, inv) if qtype == synth.Q6_K else lane_sb_k45(blk, qtype == synth.Q5_K, kq, inv)
                for e, v in got.items():
                    vals[r, 256 * sb + e] = np.float16(v)
    return vals, scales


@pytest.mark.parametrize("qtype", [synth.Q4_K, synth.Q5_K, synth.Q6_K])
@pytest.mark.parametrize("seed", [0, 1])
def test_lane_decode_is_the_oracle_value_times_the_row_scale(orc, qtype, seed):
    rows, K = 8, 512
    bsz = synth.BLOCK[qtype][1]
    raw = synth.quant_blocks(qtype, rows * K // 256, synth._rng(seed, qtype), 0.02).reshape(rows, -1)
    assert raw.shape[1] == K // 256 * bsz
    vals, scales = decode_rows(raw, qtype, K)
    y = orc.dequant(qtype, raw, K, rows)
    want = (y * (F32(1) / scales)[:, None]).astype(np.float32).astype(np.float16)
    np.testing.assert_array_equal(vals.view(np.uint16), want.view(np.uint16))
    # the header bound holds: every scaled value below 2^14, so f16 never overflows and keeps 11 bits
    assert np.all(np.abs(y / scales[:, None]) < 2.0 ** 14)
    # on rows of uniform random quants the bound is also tight: every row's largest value above 2^12
    assert np.all(np.abs(y / scales[:, None]).max(axis=1) >= 2.0 ** 12)


def test_tile_major_blocks_are_what_the_tensor_cores_read():
    """Gate/up block b: tile rows 0..63 = gate rows 64 b + 0..63, 64..127 = the same up rows; down block b:
    tile rows 0..127 = down rows 128 b + 0..127; each 64-element K stage a contiguous 128 x 64 block."""
    D, FF = 512, 256
    gate = np.arange(FF * D, dtype=np.int64).reshape(FF, D)
    up = gate + FF * D
    down = np.arange(D * FF, dtype=np.int64).reshape(D, FF) + 2 * FF * D
    expert = np.full(3 * FF * D, -1, np.int64)
    # placement as k_dequant_f16 computes it for component c, row, element i
    for c, (m, K) in enumerate(((gate, D), (up, D), (down, FF))):
        for row in range(m.shape[0]):
            if c < 2:
                base, ar = (row >> 6) * 128 * K, (0 if c == 0 else 64) + (row & 63)
            else:
                base, ar = 2 * FF * D + (row >> 7) * 128 * K, row & 127
            for i in range(K):
                expert[base + tile_off(ar, i)] = m[row, i]
    assert (expert >= 0).all()  # a permutation: every place written once
    assert len(np.unique(expert)) == expert.size
    # the GEMM's view: stage kt of block b is the 128 x 64 block at b * 128 K + kt * 8192, core matrix
    # (row group g, k octet o) at (g * 8 + o) * 64, its row i at + 8 i
    def stage(base, K, b, kt):
        blk = expert[base + b * 128 * K + kt * 8192: base + b * 128 * K + (kt + 1) * 8192]
        out = np.zeros((128, 64), np.int64)
        for g in range(16):
            for o in range(8):
                cm = blk[(g * 8 + o) * 64:(g * 8 + o + 1) * 64].reshape(8, 8)
                out[8 * g: 8 * g + 8, 8 * o: 8 * o + 8] = cm
        return out
    for b in range(FF // 64):
        for kt in range(D // 64):
            s = stage(0, D, b, kt)
            np.testing.assert_array_equal(s[:64], gate[64 * b: 64 * b + 64, 64 * kt: 64 * kt + 64])
            np.testing.assert_array_equal(s[64:], up[64 * b: 64 * b + 64, 64 * kt: 64 * kt + 64])
    for b in range(D // 128):
        for kt in range(FF // 64):
            s = stage(2 * FF * D, FF, b, kt)
            np.testing.assert_array_equal(s, down[128 * b: 128 * b + 128, 64 * kt: 64 * kt + 64])
