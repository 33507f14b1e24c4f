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
// Fragment ownership (PTX ISA, integer mma, lane = 4*g + t): A rows g and g+8, B column g, C rows g
// and g+8 with columns 2t and 2t+1. The k order inside a 32-k MMA is free as long as A and B agree:
// here lane t's two A/B registers hold elements 8t..8t+3 and 8t+4..8t+7 of the group, so a lane
// loads 8 contiguous weight bytes of a row with one 64-bit shared load.
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
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d.c[0]), "=r"(d.c[1]), "=r"(d.c[2]), "=r"(d.c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
    return d;
}
// C = A (16x16 u8) x B (16x8 s8), fresh accumulator
__device__ __forceinline__ IFrag imma16(uint32_t a0, uint32_t a1, uint32_t b0) {
    IFrag d;
    asm(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
        : "=r"(d.c[0]), "=r"(d.c[1]), "=r"(d.c[2]), "=r"(d.c[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
    return d;
}
// C = A (16x16 s8) x B (16x8 s8), fresh accumulator
__device__ __forceinline__ IFrag imma16s(uint32_t a0, uint32_t a1, uint32_t b0) {
    IFrag d;
    asm(
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

// ---- activations in fragment form (XF) ----------------------------------------------------------
// A token row x (K floats) is stored as three int8 digits of base 254 of x / s, s = max|x| / 127, so
// x = s * (a + b/254 + c/254^2) to within s / (2 * 254^2). Layout of one row (nblk = K/32 blocks of 32
// elements): 96 bytes per block = 3 digit planes p x 4 lanes t x 8 bytes, where the 8 bytes of (p, t)
// are digit p of elements 32j + 8t .. 32j + 8t + 7. A 32-k MMA then takes the lane's uint2 directly
// as its B fragment (b0 = elements 8t..8t+3, b1 = 8t+4..8t+7: the k order the A side uses as well);
// a 16-k MMA over segment s of the block takes the u32 at byte 16 (s & 1) + 4t. Per-16-element sums
// of x followed by the scale s (and three zeros) complete the row.
constexpr int PREP_NT = 256;
// Digits by float arithmetic only: adding 1.5 * 2^23 rounds a float of magnitude below 2^22 to an integer
// (round to nearest even, as rintf) and leaves that integer's two's-complement low byte in the low
// mantissa bits. __fadd_rn keeps the compiler from folding the add/subtract pair.
constexpr float RNE_MAGIC = 12582912.0f;
__device__ __forceinline__ float digit_f(float v) {  // rintf(v) clamped to [-127, 127]
    return fminf(127.f, fmaxf(-127.f, __fadd_rn(__fadd_rn(v, RNE_MAGIC), -RNE_MAGIC)));
}
__device__ __forceinline__ uint32_t digit_byte(float d) { return __float_as_uint(__fadd_rn(d, RNE_MAGIC)) & 0xffu; }
// The three digit planes of 8 consecutive elements x[k] * inv: plane p packs digit p of elements 0..3 in
// .x and 4..7 in .y (byte k = element k), a = rint(v), b = rint((v - a) * 254), c = rint((... - b) * 254).
__device__ __forceinline__ void digits8(const float (&xv)[8], float inv, uint2 (&pl)[3]) {
    uint32_t w[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float v = __fmul_rn(xv[k], inv);  // explicit roundings: no contraction into FMAs
        const float a0 = digit_f(v);
        const float r1 = __fmul_rn(__fsub_rn(v, a0), DIGIT);
        const float a1 = digit_f(r1);
        const float a2 = digit_f(__fmul_rn(__fsub_rn(r1, a1), DIGIT));
        w[0][k >> 2] |= digit_byte(a0) << (8 * (k & 3));
        w[1][k >> 2] |= digit_byte(a1) << (8 * (k & 3));
        w[2][k >> 2] |= digit_byte(a2) << (8 * (k & 3));
    }
#pragma unroll
    for (int p = 0; p < 3; p++) pl[p] = make_uint2(w[p][0], w[p][1]);
}
// Group sum S of 32 elements (already divided by the row scale) -> f16 high part and residue at
// gs + 16 + sb * 32 + 2g and + 16 (see XF).
__device__ __forceinline__ void put_group_sum(uint8_t* gs, int j, float S) {
    const __half hi = __float2half_rn(S);
    const __half lo = __float2half_rn(S - __half2float(hi));
    __half* p = reinterpret_cast<__half*>(gs + 16 + (j >> 3) * 32) + (j & 7);
    p[0] = hi;
    p[8] = lo;
}
// One row x (K floats, K % 256 == 0, 16-byte aligned) by the whole block (blockDim.x a multiple of 32,
// <= 1024): writes frag (K * 3 bytes), sum (K / 16 segment sums, then s, 0, 0, 0) and gs (XF). red: 33
// floats of shared scratch.
__device__ __forceinline__ void prep_row(const float* __restrict__ x, int K, uint2* __restrict__ frag,
                                         float* __restrict__ sum, uint8_t* __restrict__ gs, float* red) {
    const int tid = threadIdx.x, lane = tid & 31, nthr = blockDim.x, nblk = K >> 5;
    float mx = 0.f;
    for (int i = tid; i < (K >> 2); i += nthr) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[tid >> 5] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = 0.f;
        for (int w = 0; w < (nthr >> 5); w++) m = fmaxf(m, red[w]);
        if (!(m > 0.f) || m == INFINITY) m = 127.f;  // all-zero (or non-finite) rows: any scale works
        *reinterpret_cast<float4*>(sum + (K >> 4)) = make_float4(m / 127.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(gs) = make_float4(m / 127.f, 0.f, 0.f, 0.f);
        red[32] = 127.f / m;
    }
    __syncthreads();
    const float inv = red[32];
    for (int i = tid; i < nblk * 4; i += nthr) {  // item (block j, lane t): elements 32j + 8t .. + 7
        const int j = i >> 2, t = i & 3;
        const float4 u = *reinterpret_cast<const float4*>(x + 32 * j + 8 * t);
        const float4 w = *reinterpret_cast<const float4*>(x + 32 * j + 8 * t + 4);
        const float xv[8] = {u.x, u.y, u.z, u.w, w.x, w.y, w.z, w.w};
        uint2 pl[3];
        digits8(xv, inv, pl);
        uint2* o = frag + (size_t)j * 12 + t;
#pragma unroll
        for (int p = 0; p < 3; p++) o[p * 4] = pl[p];
        // segment sums: lanes t = 0,1 hold segment 2j, t = 2,3 segment 2j + 1 (items i, i^1 are
        // adjacent lanes of the same warp: nthr is a multiple of 32 and items advance by nthr)
        float s8 = ((u.x + u.y) + (u.z + u.w)) + ((w.x + w.y) + (w.z + w.w));
        s8 += __shfl_xor_sync(0xffffffffu, s8, 1);
        if ((t & 1) == 0) sum[2 * j + (t >> 1)] = s8;
        const float s32 = s8 + __shfl_xor_sync(0xffffffffu, s8, 2);  // lanes i, i^2: the same warp
        if (t == 0) put_group_sum(gs, j, s32 * inv);
    }
}

// The RMSNorm input of one token: its residual row x (n floats, global) plus its pending MoE combine
// sum_k w_k y[slot_k] (K slots in ascending expert order; K = 0: none; slots null: slot k is k, the map
// of a single-token MoE call, so no load waits for the map), into row[] (shared memory),
// then normalised in place: row = (row * (1 / sqrtf(mean(row^2) + eps))) * w. Every element is formed
// the same way whatever the block size (blockDim.x >= 128, a multiple of 32; all threads call it), the
// sum of squares in row_sumsq128's order. Each thread handles CN_PAIRS element pairs per pass, their
// loads issued together. xw: the combined residual written back (one block per row only), xn: the
// normalised row stored, when not null. w may be in shared memory. sl, sw: K words of shared scratch;
// red: 33 floats.
constexpr int CN_PAIRS = 4;
__device__ __forceinline__ void combine_norm_row(const float* __restrict__ x, const float* __restrict__ y,
                                                 const int* __restrict__ slots, const float* __restrict__ slot_w,
                                                 int K, const float* w, float eps, int n, float* row, float* xw,
                                                 float* xn, int* sl, float* sw, float* red) {
    const int tid = threadIdx.x, nt = blockDim.x;
    if (y && !slots) {  // identity slot map: the weights and rows load together, one round trip
        for (int i0 = 2 * tid; i0 < n; i0 += 2 * nt * CN_PAIRS) {
            float2 acc[CN_PAIRS], xv[CN_PAIRS];
#pragma unroll
            for (int p = 0; p < CN_PAIRS; p++) {
                const int i = i0 + 2 * nt * p;
                acc[p] = make_float2(0.f, 0.f);
                xv[p] = i < n ? *reinterpret_cast<const float2*>(x + i) : make_float2(0.f, 0.f);
            }
#pragma unroll 8
            for (int k = 0; k < K; k++) {
                const float wk = __ldg(slot_w + k);
                const float* yk = y + (size_t)k * n;
                float2 v[CN_PAIRS];
#pragma unroll
                for (int p = 0; p < CN_PAIRS; p++) {
                    const int i = i0 + 2 * nt * p;
                    v[p] = i < n ? *reinterpret_cast<const float2*>(yk + i) : make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int p = 0; p < CN_PAIRS; p++) {
                    acc[p].x = fmaf(wk, v[p].x, acc[p].x);
                    acc[p].y = fmaf(wk, v[p].y, acc[p].y);
                }
            }
#pragma unroll
            for (int p = 0; p < CN_PAIRS; p++) {
                const int i = i0 + 2 * nt * p;
                if (i < n) {
                    xv[p].x += acc[p].x;
                    xv[p].y += acc[p].y;
                    if (xw) *reinterpret_cast<float2*>(xw + i) = xv[p];
                    row[i] = xv[p].x;
                    row[i + 1] = xv[p].y;
                }
            }
        }
    } else if (y) {
        if (tid < K) {
            const int s = slots[tid];
            sl[tid] = s;
            sw[tid] = slot_w[s];
        }
        __syncthreads();
        for (int i0 = 2 * tid; i0 < n; i0 += 2 * nt * CN_PAIRS) {  // pairs i0 + 2 nt p
            float2 acc[CN_PAIRS], xv[CN_PAIRS];
#pragma unroll
            for (int p = 0; p < CN_PAIRS; p++) {
                const int i = i0 + 2 * nt * p;
                acc[p] = make_float2(0.f, 0.f);
                xv[p] = i < n ? *reinterpret_cast<const float2*>(x + i) : make_float2(0.f, 0.f);
            }
#pragma unroll 4
            for (int k = 0; k < K; k++) {
                const float* yk = y + (size_t)sl[k] * n;
                float2 v[CN_PAIRS];
#pragma unroll
                for (int p = 0; p < CN_PAIRS; p++) {
                    const int i = i0 + 2 * nt * p;
                    v[p] = i < n ? *reinterpret_cast<const float2*>(yk + i) : make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int p = 0; p < CN_PAIRS; p++) {
                    acc[p].x = fmaf(sw[k], v[p].x, acc[p].x);
                    acc[p].y = fmaf(sw[k], v[p].y, acc[p].y);
                }
            }
#pragma unroll
            for (int p = 0; p < CN_PAIRS; p++) {
                const int i = i0 + 2 * nt * p;
                if (i < n) {
                    xv[p].x += acc[p].x;
                    xv[p].y += acc[p].y;
                    if (xw) *reinterpret_cast<float2*>(xw + i) = xv[p];
                    row[i] = xv[p].x;
                    row[i + 1] = xv[p].y;
                }
            }
        }
    } else {
        for (int i = tid; i < n; i += nt) row[i] = x[i];
    }
    __syncthreads();
    const float sc = 1.0f / sqrtf(row_sumsq128(row, n, red) / (float)n + eps);
    for (int i = tid; i < n; i += nt) {
        const float v = __fmul_rn(__fmul_rn(row[i], sc), w[i]);
        row[i] = v;
        if (xn) xn[i] = v;
    }
    __syncthreads();
}

// Per-lane B-fragment pointers of up to NSET column sets over staged XF rows (m tokens, nblk blocks
// per row). Set st carries tokens 2st, 2st+1; column g holds digit g % 3 of token 2st + g / 3.
// Columns 6, 7 and tokens >= m read token 0: MMA columns are independent, and the results of those
// columns are never used.
template <int NSET>
struct BPtr {
    const uint8_t* p[NSET];
    int t;
    __device__ __forceinline__ BPtr(const uint8_t* frag, int nblk, int m) {
        const int lane = threadIdx.x & 31, g = lane >> 2;
        t = lane & 3;
#pragma unroll
        for (int st = 0; st < NSET; st++) {
            int i = TOK_PER_SET * st + g / 3, pg = g % 3;
            if (g >= 6 || i >= m) i = pg = 0;
            p[st] = frag + ((size_t)i * nblk * 3 + pg) * 32;
        }
    }
    // (b0, b1) of the 32-k block j
    __device__ __forceinline__ uint2 blk(int st, int j) const {
        return *reinterpret_cast<const uint2*>(p[st] + 96 * j + 8 * t);
    }
    // b0 of the 16-k segment s
    __device__ __forceinline__ uint32_t seg(int st, int s) const {
        return *reinterpret_cast<const uint32_t*>(p[st] + 96 * (s >> 1) + 16 * (s & 1) + 4 * t);
    }
};
__device__ __forceinline__ int sbyte(uint32_t w, int k) { return ((int32_t)(w << (24 - 8 * k))) >> 24; }
__device__ __forceinline__ int ubyte(uint32_t w, int k) { return (int)((w >> (8 * k)) & 0xffu); }

// ---- row accessors: where the task's two rows (MMA rows g and g+8) live in shared memory ------------
// off: byte offset inside the row. ld128/ld64 need 16/8-byte alignment of the address they compute.
struct RowsAny {  // any 2-byte aligned rows (dense GEMV tiles): 32-bit loads go through ld_u32_any
    const uint8_t* r[2];
    __device__ __forceinline__ uint4 ld128(int i, int off) const { return *reinterpret_cast<const uint4*>(r[i] + off); }
    __device__ __forceinline__ uint2 ld64(int i, int off) const { return *reinterpret_cast<const uint2*>(r[i] + off); }
    __device__ __forceinline__ uint32_t ld32(int i, int off) const { return ld_u32_any(r[i] + off); }
    __device__ __forceinline__ uint32_t ld16(int i, int off) const { return *reinterpret_cast<const uint16_t*>(r[i] + off); }
};
struct RowsQ6 {  // row 0 4-byte aligned, row 1 two bytes past a 4-byte boundary (Q6_K rows of 630 B)
    const uint8_t* r[2];
    __device__ __forceinline__ uint4 ld128(int i, int off) const { return *reinterpret_cast<const uint4*>(r[i] + off); }
    __device__ __forceinline__ uint2 ld64(int i, int off) const { return *reinterpret_cast<const uint2*>(r[i] + off); }
    __device__ __forceinline__ uint32_t ld32(int i, int off) const {
        if (i == 0) return *reinterpret_cast<const uint32_t*>(r[0] + off);
        const uint32_t* w = reinterpret_cast<const uint32_t*>(r[1] + off - 2);
        return __funnelshift_r(w[0], w[1], 16);
    }
    __device__ __forceinline__ uint32_t ld16(int i, int off) const { return *reinterpret_cast<const uint16_t*>(r[i] + off); }
};
// ---- one task: 16 rows x 128 weights (half h of super-block sb) ------------------------------------
// The task's activation operands (B fragments of every column set, and for Q4_K/Q5_K the lane token's
// per-16 sums of the half), loaded apart from the arithmetic so that a caller can fetch the next task's
// while this one computes.
template <int QT, int NSET>
struct KqB {
    uint2 l[2][NSET], h[2][NSET];  // Q4_K/Q5_K: 32-k blocks of the low / high nibbles of chunk cc
    float4 sa, sb;                 // Q4_K/Q5_K: per-16 sums 8h .. 8h + 7 of the lane's token (if any)
};
template <int NSET>
struct KqB<T_Q6_K, NSET> {
    uint32_t s[2][4][NSET];  // 16-k segments
};
// tsum: the lane token's per-16 sums at super-block sb (nullptr when the lane has no token)
template <int QT, int NSET, class BP>
__device__ __forceinline__ void kq_load_b(const BP& bf, int sb, int h, const float* __restrict__ tsum, KqB<QT, NSET>& B) {
    if constexpr (QT == T_Q4_K || QT == T_Q5_K) {
#pragma unroll
        for (int cc = 0; cc < 2; cc++) {
            const int c = 2 * h + cc;
#pragma unroll
            for (int st = 0; st < NSET; st++) {
                B.l[cc][st] = bf.blk(st, sb * 8 + 2 * c);      // 32-k blocks: low nibbles of chunk c,
                B.h[cc][st] = bf.blk(st, sb * 8 + 2 * c + 1);  // then its high nibbles
            }
        }
        if (tsum) {
            B.sa = *reinterpret_cast<const float4*>(tsum + 8 * h);
            B.sb = *reinterpret_cast<const float4*>(tsum + 8 * h + 4);
        }
    } else {
#pragma unroll
        for (int ib = 0; ib < 2; ib++)
#pragma unroll
            for (int q = 0; q < 4; q++)
#pragma unroll
                for (int st = 0; st < NSET; st++) B.s[ib][q][st] = bf.seg(st, sb * 16 + 8 * h + 2 * q + ib);
    }
}
// Operand sources of kq_compute_src: the B fragments (and, for Q4_K/Q5_K, the lane token's per-16 sums)
// of one task, either held in registers (KqB, loaded ahead by the caller) or read where they are used.
template <int QT, int NSET>
struct KqBRegs {
    const KqB<QT, NSET>& B;
    __device__ __forceinline__ uint2 l(int cc, int st) const { return B.l[cc][st]; }
    __device__ __forceinline__ uint2 h(int cc, int st) const { return B.h[cc][st]; }
    __device__ __forceinline__ uint32_t s(int ib, int q, int st) const { return B.s[ib][q][st]; }
    __device__ __forceinline__ float4 sa() const { return B.sa; }
    __device__ __forceinline__ float4 sb() const { return B.sb; }
};
template <int NSET>
struct KqBLazy {  // the same values as kq_load_b's, loaded at their use
    const BPtr<NSET>& bf;
    int sbk, hh;
    const float* __restrict__ tsum;
    __device__ __forceinline__ uint2 l(int cc, int st) const { return bf.blk(st, sbk * 8 + 2 * (2 * hh + cc)); }
    __device__ __forceinline__ uint2 h(int cc, int st) const { return bf.blk(st, sbk * 8 + 2 * (2 * hh + cc) + 1); }
    __device__ __forceinline__ uint32_t s(int ib, int q, int st) const { return bf.seg(st, sbk * 16 + 8 * hh + 2 * q + ib); }
    __device__ __forceinline__ float4 sa() const { return *reinterpret_cast<const float4*>(tsum + 8 * hh); }
    __device__ __forceinline__ float4 sb() const { return *reinterpret_cast<const float4*>(tsum + 8 * hh + 4); }
};
// R: the task's two rows; offsets are relative to the rows' starts (super-block sb at sb * block bytes).
// Accumulates into out[set][4] the d-scaled int32 sums of rows g, g+8 for this lane's two digit
// columns, and into mn[2] the group-minimum term of rows g, g+8 for token t (Q4_K/Q5_K, when has_sum:
// B holds the token's sums). Each 32-k chunk's weight words and B fragments are read right before its
// MMAs.
template <int QT, int NSET, class R, class BS>
__device__ __forceinline__ void kq_compute_src(const R& rows, int sb, int h, int t, const BS& B, bool has_sum,
                                               float (&out)[NSET][4], float (&mn)[2]) {
    constexpr int BB = block_bytes(QT);
    const int o = sb * BB;
    int acc[NSET][4];
#pragma unroll
    for (int st = 0; st < NSET; st++) acc[st][0] = acc[st][1] = acc[st][2] = acc[st][3] = 0;
    float d0, d1;
    if constexpr (QT == T_Q4_K || QT == T_Q5_K) {
        constexpr int QS = QT == T_Q4_K ? 16 : 48;
        const uint4 H0 = rows.ld128(0, o), H1 = rows.ld128(1, o);
        // Q4_K: high nibbles enter the MMA in place (16 x their value), so low-nibble groups take
        // 16 x their scale and d is divided by 16 (exact)
        constexpr float DS = QT == T_Q4_K ? 0.0625f : 1.0f;
        d0 = f16_to_f32(H0.x & 0xffffu) * DS;
        d1 = f16_to_f32(H1.x & 0xffffu) * DS;
        // 6-bit scales / mins of groups 4h..4h+3, word-parallel restatement of scale_min_k4
        // (qwen3moe.cpp:133-141): bytes 0..3 of the selected word
        const uint32_t s0 = h ? ((H0.w & 0x0f0f0f0fu) | ((H0.y >> 2) & 0x30303030u)) : (H0.y & 0x3f3f3f3fu);
        const uint32_t s1 = h ? ((H1.w & 0x0f0f0f0fu) | ((H1.y >> 2) & 0x30303030u)) : (H1.y & 0x3f3f3f3fu);
        if (has_sum) {  // group minimums for token t: dmin * m_g * sum(x of the group)
            const uint32_t m0 = h ? (((H0.w >> 4) & 0x0f0f0f0fu) | ((H0.z >> 2) & 0x30303030u)) : (H0.z & 0x3f3f3f3fu);
            const uint32_t m1 = h ? (((H1.w >> 4) & 0x0f0f0f0fu) | ((H1.z >> 2) & 0x30303030u)) : (H1.z & 0x3f3f3f3fu);
            const float4 sa = B.sa(), sbv = B.sb();
            const float gs[4] = {sa.x + sa.y, sa.z + sa.w, sbv.x + sbv.y, sbv.z + sbv.w};
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                a0 = fmaf((float)ubyte(m0, k), gs[k], a0);
                a1 = fmaf((float)ubyte(m1, k), gs[k], a1);
            }
            mn[0] = fmaf(f16_to_f32(H0.x >> 16), a0, mn[0]);
            mn[1] = fmaf(f16_to_f32(H1.x >> 16), a1, mn[1]);
        }
        uint2 qh0{0u, 0u}, qh1{0u, 0u};
        if constexpr (QT == T_Q5_K) {
            qh0 = rows.ld64(0, o + 16 + 8 * t);
            qh1 = rows.ld64(1, o + 16 + 8 * t);
        }
#pragma unroll
        for (int cc = 0; cc < 2; cc++) {
            const int c = 2 * h + cc;
            // bytes 8t..8t+7 of chunk c: low nibbles = weights 64c + 8t.., high = 64c + 32 + 8t..
            const uint2 w0 = rows.ld64(0, o + QS + 32 * c + 8 * t), w1 = rows.ld64(1, o + QS + 32 * c + 8 * t);
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
            } else {  // fifth bit from qh: bit 2c for the low nibbles, 2c+1 for the high ones
                lo[0] = (w0.x & 0x0f0f0f0fu) | (((qh0.x >> (2 * c)) & 0x01010101u) << 4);
                lo[1] = (w1.x & 0x0f0f0f0fu) | (((qh1.x >> (2 * c)) & 0x01010101u) << 4);
                lo[2] = (w0.y & 0x0f0f0f0fu) | (((qh0.y >> (2 * c)) & 0x01010101u) << 4);
                lo[3] = (w1.y & 0x0f0f0f0fu) | (((qh1.y >> (2 * c)) & 0x01010101u) << 4);
                hi[0] = ((w0.x >> 4) & 0x0f0f0f0fu) | (((qh0.x >> (2 * c + 1)) & 0x01010101u) << 4);
                hi[1] = ((w1.x >> 4) & 0x0f0f0f0fu) | (((qh1.x >> (2 * c + 1)) & 0x01010101u) << 4);
                hi[2] = ((w0.y >> 4) & 0x0f0f0f0fu) | (((qh0.y >> (2 * c + 1)) & 0x01010101u) << 4);
                hi[3] = ((w1.y >> 4) & 0x0f0f0f0fu) | (((qh1.y >> (2 * c + 1)) & 0x01010101u) << 4);
            }
            constexpr int LS = QT == T_Q4_K ? 16 : 1;
            const int sl0 = LS * ubyte(s0, 2 * cc), sh0 = ubyte(s0, 2 * cc + 1);
            const int sl1 = LS * ubyte(s1, 2 * cc), sh1 = ubyte(s1, 2 * cc + 1);
#pragma unroll
            for (int st = 0; st < NSET; st++) {
                const uint2 bl = B.l(cc, st), bh = B.h(cc, st);
                scale_acc(acc[st], imma32(lo[0], lo[1], lo[2], lo[3], bl.x, bl.y), sl0, sl1);
                scale_acc(acc[st], imma32(hi[0], hi[1], hi[2], hi[3], bh.x, bh.y), sh0, sh1);
            }
        }
    } else {  // Q6_K: half h = 128 weights; ib selects l in [16ib, 16ib+16)
        d0 = f16_to_f32(rows.ld16(0, o + 208));
        d1 = f16_to_f32(rows.ld16(1, o + 208));
        const uint32_t sc0[2] = {rows.ld32(0, o + 192 + 8 * h), rows.ld32(0, o + 196 + 8 * h)};
        const uint32_t sc1[2] = {rows.ld32(1, o + 192 + 8 * h), rows.ld32(1, o + 196 + 8 * h)};
#pragma unroll
        for (int ib = 0; ib < 2; ib++) {
            const int q0 = o + 16 * ib + 4 * t;
            uint32_t qa[2], qb[2], qh[2];  // [row]
#pragma unroll
            for (int r = 0; r < 2; r++) {
                qa[r] = rows.ld32(r, q0 + 64 * h);
                qb[r] = rows.ld32(r, q0 + 64 * h + 32);
                qh[r] = rows.ld32(r, q0 + 128 + 32 * h);
            }
            // 6-bit values per byte (low nibble from ql, bits 4-5 from qh; qwen3moe.cpp:187-195),
            // then q - 32 as s8: ((q & 63) + 0x60) ^ 0x80 per byte, carry-free
            const uint32_t v0[4] = {lop_sel(qa[0], qh[0] << 4, 0x0f0f0f0fu), lop_sel(qb[0], qh[0] << 2, 0x0f0f0f0fu),
                                    lop_sel(qa[0] >> 4, qh[0], 0x0f0f0f0fu), lop_sel(qb[0] >> 4, qh[0] >> 2, 0x0f0f0f0fu)};
            const uint32_t v1[4] = {lop_sel(qa[1], qh[1] << 4, 0x0f0f0f0fu), lop_sel(qb[1], qh[1] << 2, 0x0f0f0f0fu),
                                    lop_sel(qa[1] >> 4, qh[1], 0x0f0f0f0fu), lop_sel(qb[1] >> 4, qh[1] >> 2, 0x0f0f0f0fu)};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint32_t a0 = ((v0[q] & 0x3f3f3f3fu) + 0x60606060u) ^ 0x80808080u;
                const uint32_t a1 = ((v1[q] & 0x3f3f3f3fu) + 0x60606060u) ^ 0x80808080u;
                const int gl = 2 * q + ib;  // scale index within the half; segment 8h + gl of the super-block
                const int sa = sbyte(sc0[gl >> 2], gl & 3), sbb = sbyte(sc1[gl >> 2], gl & 3);
#pragma unroll
                for (int st = 0; st < NSET; st++) scale_acc(acc[st], imma16s(a0, a1, B.s(ib, q, st)), sa, sbb);
            }
        }
    }
#pragma unroll
    for (int st = 0; st < NSET; st++) {
        out[st][0] = fmaf(d0, (float)acc[st][0], out[st][0]);
        out[st][1] = fmaf(d0, (float)acc[st][1], out[st][1]);
        out[st][2] = fmaf(d1, (float)acc[st][2], out[st][2]);
        out[st][3] = fmaf(d1, (float)acc[st][3], out[st][3]);
    }
}
template <int QT, int NSET, class R>
__device__ __forceinline__ void kq_compute(const R& rows, int sb, int h, int t, const KqB<QT, NSET>& B, bool has_sum,
                                           float (&out)[NSET][4], float (&mn)[2]) {
    kq_compute_src<QT, NSET>(rows, sb, h, t, KqBRegs<QT, NSET>{B}, has_sum, out, mn);
}
// Both steps of one task (tsum: as kq_load_b).
template <int QT, int NSET, class R>
__device__ __forceinline__ void kq_task(const R& rows, int sb, int h, const BPtr<NSET>& bf,
                                        const float* __restrict__ tsum, float (&out)[NSET][4], float (&mn)[2]) {
    kq_compute_src<QT, NSET>(rows, sb, h, bf.t, KqBLazy<NSET>{bf, sb, h, tsum}, tsum != nullptr, out, mn);
}

}  // namespace eb
