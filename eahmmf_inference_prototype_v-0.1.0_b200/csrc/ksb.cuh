// ksb.cuh -- one super-block (16 rows x 256 weights) of the expert GEMV with NS MMA column sets (two
// tokens each; the weights decoded once), the inner loop of the MoE kernels (moe.cu).
//
// Same arithmetic as kq_task (kq.cuh) on both halves of a super-block at once, written for the
// instruction budget of a kernel that must decode ~40 weight bytes per cycle per SM: all operands are
// addressed from a few per-super-block base pointers with constant offsets, group scales are pulled
// out of their packed words with byte permutes, and the int32 sums of all eight (Q4_K/Q5_K) or sixteen
// (Q6_K) groups stay in one accumulator per row until the super-block's fp32 scale is applied.
//
// Operands, per lane (g, t) of the warp:
//   r0, r1   the super-block in MMA rows g and g+8 (shared memory; Q4_K/Q5_K: 16-byte aligned)
//   bq[s]    set s's B fragments of this super-block for the lane: Q4_K/Q5_K: XF row base + 8t + sb * 768,
//            Q6_K: XF row base + 4t + sb * 768 (kq.cuh: 96 bytes per 32-k block)
//   mq[s]    Q4_K/Q5_K: set s's B operand for the lane of the minimum-term MMA at this super-block: in the XF
//            group sums of token g/2 (g < 4; token 0 otherwise), f16 high parts (g even) or residues
//            (g odd), + 4t
//   out      d-scaled sums of rows g, g+8 for the lane's two digit columns (accumulated)
//   mn       dmin-scaled minimum terms of rows g, g+8 for token t (t < 2), in units of the token's
//            scale s (accumulated)
//
// The minimum term sum_g m_g * (sum of x over group g) of a Q4_K/Q5_K super-block is one f16 MMA
// (m16n8k8): A = the rows' eight 6-bit mins (exact in f16), B = the group sums / s as f16 high part and
// residue (columns 2i, 2i+1 for token i), f32 accumulation; lane t (t < 2) holds token t's two
// columns.
#pragma once
#include "kq.cuh"

namespace eb {

// C = A (16x8 f16) x B (8x8 f16), f32, fresh accumulator
__device__ __forceinline__ void hmma8(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
        : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
        : "r"(a0), "r"(a1), "r"(b0), "f"(0.f));
}
// Bytes (k0, k1) of w as an exact f16 pair (values < 1024): 0x6400 | v is the f16 1024 + v.
__device__ __forceinline__ uint32_t u8pair_f16(uint32_t w, uint32_t sel) {
    const uint32_t h = __byte_perm(w, 0u, sel) | 0x64006400u;
    const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h), __floats2half2_rn(1024.f, 1024.f));
    return *reinterpret_cast<const uint32_t*>(&r);
}

// 32-bit word at p; M: p is 2 bytes past a 4-byte boundary (Q6_K rows of 630 bytes)
template <bool M>
__device__ __forceinline__ uint32_t ld32m(const uint8_t* p) {
    if constexpr (M) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(p - 2);
        return __funnelshift_r(w[0], w[1], 16);
    } else {
        return *reinterpret_cast<const uint32_t*>(p);
    }
}

// ---- NS column sets over one decoded super-block ---------------------------------------------------
// sb_q45m / sb_q6m: the weights of the super-block are decoded once and every set s runs its MMAs,
// group-scale sums, d-scaling and minimum term on its own operands bq[s] (mq[s]); each set's integer
// and fp32 operations do not depend on NS, so out[s] and mn[s] are bitwise what NS = 1 leaves.
template <int QT, int NS>
__device__ __forceinline__ void sb_q45m(const uint8_t* __restrict__ r0, const uint8_t* __restrict__ r1,
                                        const uint8_t* const (&bq)[NS], const uint8_t* const (&mq)[NS], int t,
                                        float (&out)[NS][4], float (&mn)[NS][2]) {
    constexpr int QS = QT == T_Q4_K ? 16 : 48;
    const uint4 H0 = *reinterpret_cast<const uint4*>(r0), H1 = *reinterpret_cast<const uint4*>(r1);
    const uint32_t sA0 = H0.y & 0x3f3f3f3fu, sB0 = (H0.w & 0x0f0f0f0fu) | ((H0.y >> 2) & 0x30303030u);
    const uint32_t sA1 = H1.y & 0x3f3f3f3fu, sB1 = (H1.w & 0x0f0f0f0fu) | ((H1.y >> 2) & 0x30303030u);
    constexpr int LSH = QT == T_Q4_K ? 4 : 0;
    const uint32_t le0[2] = {(sA0 & 0x00ff00ffu) << LSH, (sB0 & 0x00ff00ffu) << LSH};
    const uint32_t le1[2] = {(sA1 & 0x00ff00ffu) << LSH, (sB1 & 0x00ff00ffu) << LSH};
    const uint32_t ho0[2] = {(sA0 >> 8) & 0x00ff00ffu, (sB0 >> 8) & 0x00ff00ffu};
    const uint32_t ho1[2] = {(sA1 >> 8) & 0x00ff00ffu, (sB1 >> 8) & 0x00ff00ffu};
    uint2 qh0{0u, 0u}, qh1{0u, 0u};
    if constexpr (QT == T_Q5_K) {
        qh0 = *reinterpret_cast<const uint2*>(r0 + 16 + 8 * t);
        qh1 = *reinterpret_cast<const uint2*>(r1 + 16 + 8 * t);
    }
    const uint8_t* q0 = r0 + QS + 8 * t;
    const uint8_t* q1 = r1 + QS + 8 * t;
    int acc[NS][4];
#pragma unroll
    for (int s = 0; s < NS; s++) acc[s][0] = acc[s][1] = acc[s][2] = acc[s][3] = 0;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint2 w0 = *reinterpret_cast<const uint2*>(q0 + 32 * c), w1 = *reinterpret_cast<const uint2*>(q1 + 32 * c);
        uint2 bl[NS], bh[NS];
#pragma unroll
        for (int s = 0; s < NS; s++) {
            bl[s] = *reinterpret_cast<const uint2*>(bq[s] + 96 * (2 * c));
            bh[s] = *reinterpret_cast<const uint2*>(bq[s] + 96 * (2 * c + 1));
        }
        uint32_t lo[4], hi[4];
        if constexpr (QT == T_Q4_K) {
            lo[0] = w0.x & 0x0f0f0f0fu;
            lo[1] = w1.x & 0x0f0f0f0fu;
            lo[2] = w0.y & 0x0f0f0f0fu;
            lo[3] = w1.y & 0x0f0f0f0fu;
            hi[0] = w0.x & 0xf0f0f0f0u;
            hi[1] = w1.x & 0xf0f0f0f0u;
            hi[2] = w0.y & 0xf0f0f0f0u;
            hi[3] = w1.y & 0xf0f0f0f0u;
        } else {
            lo[0] = (w0.x & 0x0f0f0f0fu) | (((qh0.x >> (2 * c)) & 0x01010101u) << 4);
            lo[1] = (w1.x & 0x0f0f0f0fu) | (((qh1.x >> (2 * c)) & 0x01010101u) << 4);
            lo[2] = (w0.y & 0x0f0f0f0fu) | (((qh0.y >> (2 * c)) & 0x01010101u) << 4);
            lo[3] = (w1.y & 0x0f0f0f0fu) | (((qh1.y >> (2 * c)) & 0x01010101u) << 4);
            hi[0] = ((w0.x >> 4) & 0x0f0f0f0fu) | (((qh0.x >> (2 * c + 1)) & 0x01010101u) << 4);
            hi[1] = ((w1.x >> 4) & 0x0f0f0f0fu) | (((qh1.x >> (2 * c + 1)) & 0x01010101u) << 4);
            hi[2] = ((w0.y >> 4) & 0x0f0f0f0fu) | (((qh0.y >> (2 * c + 1)) & 0x01010101u) << 4);
            hi[3] = ((w1.y >> 4) & 0x0f0f0f0fu) | (((qh1.y >> (2 * c + 1)) & 0x01010101u) << 4);
        }
        const int f = c & 1, wd = c >> 1;
        const int sl0 = f ? (int)(le0[wd] >> 16) : (int)(le0[wd] & 0xffffu);
        const int sl1 = f ? (int)(le1[wd] >> 16) : (int)(le1[wd] & 0xffffu);
        const int sh0 = f ? (int)(ho0[wd] >> 16) : (int)(ho0[wd] & 0xffffu);
        const int sh1 = f ? (int)(ho1[wd] >> 16) : (int)(ho1[wd] & 0xffffu);
#pragma unroll
        for (int s = 0; s < NS; s++) {
            scale_acc(acc[s], imma32(lo[0], lo[1], lo[2], lo[3], bl[s].x, bl[s].y), sl0, sl1);
            scale_acc(acc[s], imma32(hi[0], hi[1], hi[2], hi[3], bh[s].x, bh[s].y), sh0, sh1);
        }
    }
    constexpr float DS = QT == T_Q4_K ? 0.0625f : 1.0f;
    const float d0 = f16_to_f32(H0.x & 0xffffu) * DS, d1 = f16_to_f32(H1.x & 0xffffu) * DS;
#pragma unroll
    for (int s = 0; s < NS; s++) {
        out[s][0] = fmaf(d0, (float)acc[s][0], out[s][0]);
        out[s][1] = fmaf(d0, (float)acc[s][1], out[s][1]);
        out[s][2] = fmaf(d1, (float)acc[s][2], out[s][2]);
        out[s][3] = fmaf(d1, (float)acc[s][3], out[s][3]);
    }
    const uint32_t mA0 = H0.z & 0x3f3f3f3fu, mB0 = ((H0.w >> 4) & 0x0f0f0f0fu) | ((H0.z >> 2) & 0x30303030u);
    const uint32_t mA1 = H1.z & 0x3f3f3f3fu, mB1 = ((H1.w >> 4) & 0x0f0f0f0fu) | ((H1.z >> 2) & 0x30303030u);
    const uint32_t sel = (t & 1) ? 0x4342u : 0x4140u;
    const uint32_t ma0 = u8pair_f16(t < 2 ? mA0 : mB0, sel), ma1 = u8pair_f16(t < 2 ? mA1 : mB1, sel);
    const float dm0 = f16_to_f32(H0.x >> 16), dm1 = f16_to_f32(H1.x >> 16);
#pragma unroll
    for (int s = 0; s < NS; s++) {
        float cm[4];
        hmma8(cm, ma0, ma1, *reinterpret_cast<const uint32_t*>(mq[s]));
        mn[s][0] = fmaf(dm0, cm[0] + cm[1], mn[s][0]);
        mn[s][1] = fmaf(dm1, cm[2] + cm[3], mn[s][1]);
    }
}

template <bool M0, bool M1, int NS>
__device__ __forceinline__ void sb_q6m(const uint8_t* __restrict__ r0, const uint8_t* __restrict__ r1,
                                       const uint8_t* const (&bq)[NS], int t, float (&out)[NS][4]) {
    const uint8_t* p0 = r0 + 4 * t;
    const uint8_t* p1 = r1 + 4 * t;
    int acc[NS][4];
#pragma unroll
    for (int s = 0; s < NS; s++) acc[s][0] = acc[s][1] = acc[s][2] = acc[s][3] = 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint32_t sc0[2] = {ld32m<M0>(r0 + 192 + 8 * h), ld32m<M0>(r0 + 196 + 8 * h)};
        const uint32_t sc1[2] = {ld32m<M1>(r1 + 192 + 8 * h), ld32m<M1>(r1 + 196 + 8 * h)};
#pragma unroll
        for (int ib = 0; ib < 2; ib++) {
            const int o = 64 * h + 16 * ib;
            const uint32_t qa0 = ld32m<M0>(p0 + o), qb0 = ld32m<M0>(p0 + o + 32), qh0 = ld32m<M0>(p0 + 128 + 32 * h + 16 * ib);
            const uint32_t qa1 = ld32m<M1>(p1 + o), qb1 = ld32m<M1>(p1 + o + 32), qh1 = ld32m<M1>(p1 + 128 + 32 * h + 16 * ib);
            const uint32_t v0[4] = {lop_sel(qa0, qh0 << 4, 0x0f0f0f0fu), lop_sel(qb0, qh0 << 2, 0x0f0f0f0fu),
                                    lop_sel(qa0 >> 4, qh0, 0x0f0f0f0fu), lop_sel(qb0 >> 4, qh0 >> 2, 0x0f0f0f0fu)};
            const uint32_t v1[4] = {lop_sel(qa1, qh1 << 4, 0x0f0f0f0fu), lop_sel(qb1, qh1 << 2, 0x0f0f0f0fu),
                                    lop_sel(qa1 >> 4, qh1, 0x0f0f0f0fu), lop_sel(qb1 >> 4, qh1 >> 2, 0x0f0f0f0fu)};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint32_t a0 = ((v0[q] & 0x3f3f3f3fu) + 0x60606060u) ^ 0x80808080u;
                const uint32_t a1 = ((v1[q] & 0x3f3f3f3fu) + 0x60606060u) ^ 0x80808080u;
                const int gl = 2 * q + ib;
                const int sa = sbyte(sc0[gl >> 2], gl & 3), sbb = sbyte(sc1[gl >> 2], gl & 3);
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    const uint32_t b = *reinterpret_cast<const uint32_t*>(bq[s] + 96 * (4 * h + q) + 16 * ib);
                    scale_acc(acc[s], imma16s(a0, a1, b), sa, sbb);
                }
            }
        }
    }
    const float d0 = f16_to_f32(*reinterpret_cast<const uint16_t*>(r0 + 208));
    const float d1 = f16_to_f32(*reinterpret_cast<const uint16_t*>(r1 + 208));
#pragma unroll
    for (int s = 0; s < NS; s++) {
        out[s][0] = fmaf(d0, (float)acc[s][0], out[s][0]);
        out[s][1] = fmaf(d0, (float)acc[s][1], out[s][1]);
        out[s][2] = fmaf(d1, (float)acc[s][2], out[s][2]);
        out[s][3] = fmaf(d1, (float)acc[s][3], out[s][3]);
    }
}

// One column set (the decode kernels and groups of up to two slots): out / mn of that set.
// Q4_K / Q5_K super-block. Int32 bound per row: eight groups of 32 x 15 (x16 for in-place high
// nibbles, 31 for Q5_K) x 127 x 63 (x16 for Q4_K low-nibble scales) < 5e8.
template <int QT>
__device__ __forceinline__ void sb_q45(const uint8_t* __restrict__ r0, const uint8_t* __restrict__ r1,
                                       const uint8_t* __restrict__ bq, const uint8_t* __restrict__ mq, int t,
                                       float (&out)[4], float (&mn)[2]) {
    const uint8_t* const b[1] = {bq};
    const uint8_t* const m[1] = {mq};
    sb_q45m<QT, 1>(r0, r1, b, m, t, reinterpret_cast<float(&)[1][4]>(out), reinterpret_cast<float(&)[1][2]>(mn));
}
// Q6_K super-block (ql 128 | qh 64 | 16 int8 scales | f16 d; qwen3moe.cpp:180-202). M0/M1: row g /
// g+8 of this super-block starts 2 bytes past a 4-byte boundary. Int32 bound per row: sixteen groups
// of 16 x 32 x 127 x 128 < 1.4e8.
template <bool M0, bool M1>
__device__ __forceinline__ void sb_q6(const uint8_t* __restrict__ r0, const uint8_t* __restrict__ r1,
                                      const uint8_t* __restrict__ bq, int t, float (&out)[4]) {
    const uint8_t* const b[1] = {bq};
    sb_q6m<M0, M1, 1>(r0, r1, b, t, reinterpret_cast<float(&)[1][4]>(out));
}

}  // namespace eb
