// kq.cuh -- K-quant GEMV core on the tensor cores (integer mma.sync: u8 weights x s8 activations -> s32).
//
// Block formats are the ones the reference decodes on the CPU (qwen3moe.cpp:133-202):
//   Q4_K (144 B): f16 d | f16 dmin | 12 bytes of packed 6-bit scales/mins | 128 bytes of nibbles
//   Q5_K (176 B): as Q4_K, plus 32 bytes of high bits (qh) before the nibbles
//   Q6_K (210 B): 128 bytes low nibbles (ql) | 64 bytes of 2-bit highs (qh) | 16 int8 scales | f16 d
//
// Operand A (16 weight rows x k) is the quantized integers themselves: one 32-bit op unpacks four
// weights into four u8 lanes ((w & 0x0F0F0F0F) for low nibbles); Q6_K values enter as the signed
// q - 32 (s8), so its offset needs no separate term. Operand B holds each token's
// activations as three int8 digits of base 254 (x = s * (a + b/254 + c/254^2), s = max|x|/127,
// reconstruction error below 2^-23 of max|x|), one digit per MMA column, so a column set carries two
// tokens. Each MMA covers one quantization group (k32 for Q4_K/Q5_K, k16 for Q6_K); its exact int32
// sums are multiplied by the group's integer scale and accumulated in int32 per super-block half,
// then scaled by the super-block's fp16 d in fp32. Q4_K/Q5_K group minimums are applied through
// per-16 activation sums. Every task decodes the scales of its own rows from the staged block headers.
//
// Fragment ownership (PTX ISA, integer mma, lane = 4*g + t): A rows g and g+8, k 4t..4t+3 (and
// 16+4t.. for k32) -- exactly the t-th 32-bit word of a row's 16-byte run; B column g, same k;
// C rows g and g+8, columns 2t and 2t+1.
#pragma once
#include "common.cuh"

namespace eb {

// ---- constants ------------------------------------------------------------------------------------
constexpr int QT_GROUPS_Q6 = 16, QT_GROUPS_Q45 = 8;
constexpr float DIGIT = 254.0f;  // base of the activation digits
constexpr int TOK_PER_SET = 2;   // tokens per MMA column set (three digit columns each)

__host__ __device__ constexpr int groups_of(int qt) { return qt == T_Q6_K ? QT_GROUPS_Q6 : QT_GROUPS_Q45; }

// ---- warp-level MMA ---------------------------------------------------------------------------------
struct IFrag {
    int c[4];
};
// C = A (16x32 u8) x B (32x8 s8), fresh accumulator
__device__ __forceinline__ IFrag imma32(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    IFrag d;
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d.c[0]), "=r"(d.c[1]), "=r"(d.c[2]), "=r"(d.c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
    return d;
}
// C = A (16x16 u8) x B (16x8 s8), fresh accumulator
__device__ __forceinline__ IFrag imma16(uint32_t a0, uint32_t a1, uint32_t b0) {
    IFrag d;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
        : "=r"(d.c[0]), "=r"(d.c[1]), "=r"(d.c[2]), "=r"(d.c[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
    return d;
}
// C = A (16x16 s8) x B (16x8 s8), fresh accumulator
__device__ __forceinline__ IFrag imma16s(uint32_t a0, uint32_t a1, uint32_t b0) {
    IFrag d;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
        : "=r"(d.c[0]), "=r"(d.c[1]), "=r"(d.c[2]), "=r"(d.c[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
    return d;
}
// acc (rows g / g+8, this lane's two columns) += group scale * C
__device__ __forceinline__ void scale_acc(int (&acc)[4], const IFrag& C, int s0, int s1) {
    acc[0] += s0 * C.c[0];
    acc[1] += s0 * C.c[1];
    acc[2] += s1 * C.c[2];
    acc[3] += s1 * C.c[3];
}

// 32-bit word at any even byte offset of shared memory (Q6_K rows are 2-byte aligned)
__device__ __forceinline__ uint32_t ld_u32_any(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* b = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3) * 8;
    return sh ? __funnelshift_r(b[0], b[1], sh) : b[0];
}

__device__ __forceinline__ uint32_t lop_sel(uint32_t a, uint32_t b, uint32_t mask) {  // (a & mask) | (b & ~mask)
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(r) : "r"(a), "r"(b), "r"(mask));
    return r;
}

// Per-lane B-fragment pointers of up to NSET column sets over a staged copy of the tokens' fragment
// rows (frag: m rows of nblk * 12 uint2). Set st carries tokens 2st, 2st+1; column g holds digit g % 3
// of token 2st + g / 3 (columns 6, 7 are zero).
template <int NSET>
struct BPtr {
    const uint2* p[NSET];
    __device__ __forceinline__ BPtr(const uint2* frag, int nblk, int m) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int st = 0; st < NSET; st++) {
            const int i = TOK_PER_SET * st + g / 3;
            p[st] = (g < 6 && i < m) ? frag + ((size_t)i * nblk * 3 + g % 3) * 4 + t : nullptr;
        }
    }
    // (b0, b1) of the 32-k block j
    __device__ __forceinline__ uint2 blk(int st, int j) const { return p[st] ? p[st][j * 12] : make_uint2(0u, 0u); }
    // b0 of the 16-k segment s
    __device__ __forceinline__ uint32_t seg(int st, int s) const {
        return p[st] ? reinterpret_cast<const uint32_t*>(p[st] + (s >> 1) * 12)[s & 1] : 0u;
    }
};
__device__ __forceinline__ int sbyte(uint32_t w, int k) { return ((int32_t)(w << (24 - 8 * k))) >> 24; }

// ---- one task: 16 rows x 128 weights (half h of super-block sb) ------------------------------------
// base + r*stride: row r of the staged tile. out[set][4] receives d * (int32 sums) for rows g, g+8 and
// this lane's two digit columns; mn[2] the group-minimum term of rows g, g+8 for token t (Q4_K/Q5_K;
// sums: staged per-16 activation sums, m tokens x nseg).
template <int QT, int NSET>
__device__ __forceinline__ void mma_task(const uint8_t* __restrict__ base, int stride, int sb, int h,
                                         const BPtr<NSET>& bf, const float* __restrict__ sums, int nseg, int m,
                                         float (&out)[NSET][4], float (&mn)[2]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    constexpr int BB = block_bytes(QT);
    const uint8_t* r0 = base + (size_t)g * stride + (size_t)sb * BB;
    const uint8_t* r1 = r0 + (size_t)8 * stride;
    int acc[NSET][4];
#pragma unroll
    for (int st = 0; st < NSET; st++) acc[st][0] = acc[st][1] = acc[st][2] = acc[st][3] = 0;
    float d0, d1;
    if constexpr (QT == T_Q4_K || QT == T_Q5_K) {
        constexpr int QS = QT == T_Q4_K ? 16 : 48;
        const uint4 H0 = *reinterpret_cast<const uint4*>(r0), H1 = *reinterpret_cast<const uint4*>(r1);
        d0 = f16_to_f32(H0.x & 0xffffu);
        d1 = f16_to_f32(H1.x & 0xffffu);
        // 6-bit scales / mins of groups 4h..4h+3, word-parallel restatement of scale_min_k4
        // (qwen3moe.cpp:133-141): bytes 0..3 of the selected word
        const uint32_t s0 = h ? ((H0.w & 0x0f0f0f0fu) | ((H0.y >> 2) & 0x30303030u)) : (H0.y & 0x3f3f3f3fu);
        const uint32_t s1 = h ? ((H1.w & 0x0f0f0f0fu) | ((H1.y >> 2) & 0x30303030u)) : (H1.y & 0x3f3f3f3fu);
        if (t < m) {  // group minimums for token t: dmin * m_g * sum(x of the group)
            const uint32_t m0 = h ? (((H0.w >> 4) & 0x0f0f0f0fu) | ((H0.z >> 2) & 0x30303030u)) : (H0.z & 0x3f3f3f3fu);
            const uint32_t m1 = h ? (((H1.w >> 4) & 0x0f0f0f0fu) | ((H1.z >> 2) & 0x30303030u)) : (H1.z & 0x3f3f3f3fu);
            const float4 sa = *reinterpret_cast<const float4*>(sums + (size_t)t * nseg + sb * 16 + 8 * h);
            const float4 sbv = *reinterpret_cast<const float4*>(sums + (size_t)t * nseg + sb * 16 + 8 * h + 4);
            const float gs[4] = {sa.x + sa.y, sa.z + sa.w, sbv.x + sbv.y, sbv.z + sbv.w};
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                a0 = fmaf((float)((m0 >> (8 * k)) & 63u), gs[k], a0);
                a1 = fmaf((float)((m1 >> (8 * k)) & 63u), gs[k], a1);
            }
            mn[0] = f16_to_f32(H0.x >> 16) * a0;
            mn[1] = f16_to_f32(H1.x >> 16) * a1;
        } else {
            mn[0] = mn[1] = 0.f;
        }
        uint32_t qh0a = 0, qh0b = 0, qh1a = 0, qh1b = 0;
        if constexpr (QT == T_Q5_K) {
            qh0a = *reinterpret_cast<const uint32_t*>(r0 + 16 + 4 * t);
            qh0b = *reinterpret_cast<const uint32_t*>(r0 + 32 + 4 * t);
            qh1a = *reinterpret_cast<const uint32_t*>(r1 + 16 + 4 * t);
            qh1b = *reinterpret_cast<const uint32_t*>(r1 + 32 + 4 * t);
        }
#pragma unroll
        for (int cc = 0; cc < 2; cc++) {
            const int c = 2 * h + cc;
            const uint32_t w0a = *reinterpret_cast<const uint32_t*>(r0 + QS + 32 * c + 4 * t);       // row g, l 4t..
            const uint32_t w0b = *reinterpret_cast<const uint32_t*>(r0 + QS + 32 * c + 16 + 4 * t);  // row g, l 16+4t..
            const uint32_t w1a = *reinterpret_cast<const uint32_t*>(r1 + QS + 32 * c + 4 * t);
            const uint32_t w1b = *reinterpret_cast<const uint32_t*>(r1 + QS + 32 * c + 16 + 4 * t);
            uint32_t lo[4], hi[4];
            if constexpr (QT == T_Q4_K) {
                lo[0] = w0a & 0x0f0f0f0fu;
                lo[1] = w1a & 0x0f0f0f0fu;
                lo[2] = w0b & 0x0f0f0f0fu;
                lo[3] = w1b & 0x0f0f0f0fu;
                hi[0] = (w0a >> 4) & 0x0f0f0f0fu;
                hi[1] = (w1a >> 4) & 0x0f0f0f0fu;
                hi[2] = (w0b >> 4) & 0x0f0f0f0fu;
                hi[3] = (w1b >> 4) & 0x0f0f0f0fu;
            } else {  // fifth bit from qh: bit 2c for the low nibbles, 2c+1 for the high ones
                lo[0] = (w0a & 0x0f0f0f0fu) | (((qh0a >> (2 * c)) & 0x01010101u) << 4);
                lo[1] = (w1a & 0x0f0f0f0fu) | (((qh1a >> (2 * c)) & 0x01010101u) << 4);
                lo[2] = (w0b & 0x0f0f0f0fu) | (((qh0b >> (2 * c)) & 0x01010101u) << 4);
                lo[3] = (w1b & 0x0f0f0f0fu) | (((qh1b >> (2 * c)) & 0x01010101u) << 4);
                hi[0] = ((w0a >> 4) & 0x0f0f0f0fu) | (((qh0a >> (2 * c + 1)) & 0x01010101u) << 4);
                hi[1] = ((w1a >> 4) & 0x0f0f0f0fu) | (((qh1a >> (2 * c + 1)) & 0x01010101u) << 4);
                hi[2] = ((w0b >> 4) & 0x0f0f0f0fu) | (((qh0b >> (2 * c + 1)) & 0x01010101u) << 4);
                hi[3] = ((w1b >> 4) & 0x0f0f0f0fu) | (((qh1b >> (2 * c + 1)) & 0x01010101u) << 4);
            }
            const int sl0 = (s0 >> (16 * cc)) & 63, sh0 = (s0 >> (16 * cc + 8)) & 63;
            const int sl1 = (s1 >> (16 * cc)) & 63, sh1 = (s1 >> (16 * cc + 8)) & 63;
            const int jl = sb * 8 + 2 * c;  // 32-k blocks: low nibbles of chunk c, then its high nibbles
#pragma unroll
            for (int st = 0; st < NSET; st++) {
                const uint2 bl = bf.blk(st, jl), bh = bf.blk(st, jl + 1);
                scale_acc(acc[st], imma32(lo[0], lo[1], lo[2], lo[3], bl.x, bl.y), sl0, sl1);
                scale_acc(acc[st], imma32(hi[0], hi[1], hi[2], hi[3], bh.x, bh.y), sh0, sh1);
            }
        }
    } else {  // Q6_K: half h = 128 weights; ib selects l in [16ib, 16ib+16)
        d0 = f16_to_f32(*reinterpret_cast<const uint16_t*>(r0 + 208));
        d1 = f16_to_f32(*reinterpret_cast<const uint16_t*>(r1 + 208));
        const uint32_t sc0[2] = {ld_u32_any(r0 + 192 + 8 * h), ld_u32_any(r0 + 196 + 8 * h)};
        const uint32_t sc1[2] = {ld_u32_any(r1 + 192 + 8 * h), ld_u32_any(r1 + 196 + 8 * h)};
        mn[0] = mn[1] = 0.f;
        const bool al4 = ((reinterpret_cast<uintptr_t>(r0) | reinterpret_cast<uintptr_t>(r1)) & 3) == 0;
#pragma unroll
        for (int ib = 0; ib < 2; ib++) {
            const int o = 16 * ib + 4 * t;
            uint32_t qa0, qb0, qh0, qa1, qb1, qh1;
            if (al4) {
                qa0 = *reinterpret_cast<const uint32_t*>(r0 + 64 * h + o);
                qb0 = *reinterpret_cast<const uint32_t*>(r0 + 64 * h + 32 + o);
                qh0 = *reinterpret_cast<const uint32_t*>(r0 + 128 + 32 * h + o);
                qa1 = *reinterpret_cast<const uint32_t*>(r1 + 64 * h + o);
                qb1 = *reinterpret_cast<const uint32_t*>(r1 + 64 * h + 32 + o);
                qh1 = *reinterpret_cast<const uint32_t*>(r1 + 128 + 32 * h + o);
            } else {
                qa0 = ld_u32_any(r0 + 64 * h + o);
                qb0 = ld_u32_any(r0 + 64 * h + 32 + o);
                qh0 = ld_u32_any(r0 + 128 + 32 * h + o);
                qa1 = ld_u32_any(r1 + 64 * h + o);
                qb1 = ld_u32_any(r1 + 64 * h + 32 + o);
                qh1 = ld_u32_any(r1 + 128 + 32 * h + o);
            }
            // 6-bit values per byte (low nibble from ql, bits 4-5 from qh; qwen3moe.cpp:187-195),
            // then q - 32 as s8: ((q & 63) + 0x60) ^ 0x80 per byte, carry-free
            const uint32_t v0[4] = {lop_sel(qa0, qh0 << 4, 0x0f0f0f0fu), lop_sel(qb0, qh0 << 2, 0x0f0f0f0fu),
                                    lop_sel(qa0 >> 4, qh0, 0x0f0f0f0fu), lop_sel(qb0 >> 4, qh0 >> 2, 0x0f0f0f0fu)};
            const uint32_t v1[4] = {lop_sel(qa1, qh1 << 4, 0x0f0f0f0fu), lop_sel(qb1, qh1 << 2, 0x0f0f0f0fu),
                                    lop_sel(qa1 >> 4, qh1, 0x0f0f0f0fu), lop_sel(qb1 >> 4, qh1 >> 2, 0x0f0f0f0fu)};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint32_t a0 = ((v0[q] & 0x3f3f3f3fu) + 0x60606060u) ^ 0x80808080u;
                const uint32_t a1 = ((v1[q] & 0x3f3f3f3fu) + 0x60606060u) ^ 0x80808080u;
                const int gl = 2 * q + ib;  // scale index within the half; segment 8h + gl of the super-block
                const int sa = sbyte(sc0[gl >> 2], gl & 3), sbb = sbyte(sc1[gl >> 2], gl & 3);
#pragma unroll
                for (int st = 0; st < NSET; st++)
                    scale_acc(acc[st], imma16s(a0, a1, bf.seg(st, sb * 16 + 8 * h + gl)), sa, sbb);
            }
        }
    }
#pragma unroll
    for (int st = 0; st < NSET; st++) {
        out[st][0] = d0 * (float)acc[st][0];
        out[st][1] = d0 * (float)acc[st][1];
        out[st][2] = d1 * (float)acc[st][2];
        out[st][3] = d1 * (float)acc[st][3];
    }
}

}  // namespace eb
