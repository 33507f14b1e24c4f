// kq.cuh -- K-quant GEMV core on the tensor cores (mma.sync m16n8k16, f16 x f16 -> f32).
//
// Block formats are the ones the reference decodes on the CPU (qwen3moe.cpp:133-202):
//   Q4_K (144 B): f16 d | f16 dmin | 12 bytes of packed 6-bit scales/mins | 128 bytes of nibbles
//   Q5_K (176 B): as Q4_K, plus 32 bytes of high bits (qh) before the nibbles
//   Q6_K (210 B): 128 bytes low nibbles (ql) | 64 bytes of 2-bit highs (qh) | 16 int8 scales | f16 d
//
// Operand A (16 weight rows x 16 k) is built in registers straight from the quantized bytes: masking
// a field in place, (w & 0x000F000F), leaves the bit pattern q of an f16 subnormal whose value is
// q * 2^-24 exactly (every f16 pattern below 2^11 is linear in its bits), two weights per 32-bit op.
// Operand B (16 k x 8 columns) holds the activations of up to four tokens, each split into an f16
// high part and an f16 low part (x = hi + lo to ~2^-22 relative), so the products accumulate in fp32
// with fp32-level accuracy. Each MMA covers one quantization group, whose scale is applied to the
// fp32 accumulator afterwards; group minimums / the Q6_K offset of 32 are applied per super-block
// through per-group activation sums.
//
// Fragment ownership (PTX ISA, mma.m16n8k16 .f16): lane = 4*g + t; A: rows g and g+8, k in
// {2t, 2t+1, 2t+8, 2t+9}; B: column g, same k; C: rows g and g+8, columns 2t and 2t+1.
// Logical k {2t, 2t+1, 2t+8, 2t+9} of a 16-weight segment is mapped to the physical weights
// {4t, 4t+2, 4t+1, 4t+3}, i.e. bytes 0/2 and 1/3 of the segment's t-th 32-bit word; the staged
// activation fragments use the same mapping. Column 2j is token j's high part, 2j+1 its low part.
#pragma once
#include "common.cuh"

namespace eb {

// ---- constants ------------------------------------------------------------------------------------
constexpr float P2_24 = 16777216.0f;  // subnormal f16 field at bit 0: value q * 2^-24
constexpr float P2_20 = 1048576.0f;   // field at bit 4 (Q4_K high nibbles): q * 2^-20
constexpr int QT_GROUPS_Q6 = 16, QT_GROUPS_Q45 = 8;

__host__ __device__ constexpr int groups_of(int qt) { return qt == T_Q6_K ? QT_GROUPS_Q6 : QT_GROUPS_Q45; }

// ---- warp-level MMA ---------------------------------------------------------------------------------
struct Frag4 {
    float c[4];
};
__device__ __forceinline__ void mma16816(Frag4& d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d.c[0]), "+f"(d.c[1]), "+f"(d.c[2]), "+f"(d.c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// acc (rows g / g+8, this lane's token, hi and lo columns) += s_row * C
__device__ __forceinline__ void scale_acc(float (&acc)[4], const Frag4& C, float s0, float s1) {
    acc[0] = fmaf(s0, C.c[0], acc[0]);
    acc[1] = fmaf(s0, C.c[1], acc[1]);
    acc[2] = fmaf(s1, C.c[2], acc[2]);
    acc[3] = fmaf(s1, C.c[3], acc[3]);
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

// Per-lane fragment pointers of up to NSET column sets: tok[i] is the xf row of token i (< m).
template <int NSET>
struct BPtr {
    const uint2* p[NSET];
    __device__ __forceinline__ BPtr(const XF& xf, const int* tok, int m) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int st = 0; st < NSET; st++) {
            const int i = 4 * st + (g >> 1);
            p[st] = i < m ? xf.frag + (size_t)tok[i] * xf.nseg * 8 + (g & 1) * 4 + t : nullptr;
        }
    }
    __device__ __forceinline__ uint2 get(int st, int seg) const {
        if (!p[st]) return make_uint2(0u, 0u);
        return __ldg(p[st] + (size_t)seg * 8);
    }
};

// ---- one task: 16 rows x 128 weights (half a super-block) ----------------------------------------
// rows: row r of the tile at base + r*stride; scl: this row group's decoded scales, laid out
// [sb][group][16] with rows r and r+8 adjacent (index 2*(r&7) + (r>>3)); acc[set][4].
template <int QT, int NSET>
__device__ __forceinline__ void mma_task(const uint8_t* __restrict__ base, int stride, int sb, int h,
                                         const BPtr<NSET>& bf, const float* __restrict__ scl, float (&acc)[NSET][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    constexpr int BB = block_bytes(QT);
    constexpr int G = groups_of(QT);
    const uint8_t* r0 = base + (size_t)g * stride + (size_t)sb * BB;
    const uint8_t* r1 = r0 + (size_t)8 * stride;
    const float* sc = scl + (size_t)sb * G * 16 + 2 * g;
    const int seg0 = sb * 16;  // first 16-k segment of the super-block
    if constexpr (QT == T_Q4_K || QT == T_Q5_K) {
        constexpr int QS = QT == T_Q4_K ? 16 : 48;
        uint32_t hA[2] = {0, 0}, hB[2] = {0, 0};
        if constexpr (QT == T_Q5_K) {
#pragma unroll
            for (int s = 0; s < 2; s++) {
                hA[s] = *reinterpret_cast<const uint32_t*>(r0 + 16 + 16 * s + 4 * t);
                hB[s] = *reinterpret_cast<const uint32_t*>(r1 + 16 + 16 * s + 4 * t);
            }
        }
#pragma unroll
        for (int cc = 0; cc < 2; cc++) {
            const int c = 2 * h + cc;
            uint32_t lo[2][4], hi[2][4];  // [segment][a0..a3]
#pragma unroll
            for (int s = 0; s < 2; s++) {
                const uint32_t w0 = *reinterpret_cast<const uint32_t*>(r0 + QS + 32 * c + 16 * s + 4 * t);
                const uint32_t w1 = *reinterpret_cast<const uint32_t*>(r1 + QS + 32 * c + 16 * s + 4 * t);
                if constexpr (QT == T_Q4_K) {
                    const uint32_t u0 = w0 >> 8, u1 = w1 >> 8;
                    lo[s][0] = w0 & 0x000f000fu;
                    lo[s][1] = w1 & 0x000f000fu;
                    lo[s][2] = u0 & 0x000f000fu;
                    lo[s][3] = u1 & 0x000f000fu;
                    hi[s][0] = w0 & 0x00f000f0u;  // field at bit 4: q * 2^-20
                    hi[s][1] = w1 & 0x00f000f0u;
                    hi[s][2] = u0 & 0x00f000f0u;
                    hi[s][3] = u1 & 0x00f000f0u;
                } else {
                    const uint32_t l0 = (w0 & 0x0f0f0f0fu) | (((hA[s] >> (2 * c)) & 0x01010101u) << 4);
                    const uint32_t l1 = (w1 & 0x0f0f0f0fu) | (((hB[s] >> (2 * c)) & 0x01010101u) << 4);
                    const uint32_t k0 = ((w0 >> 4) & 0x0f0f0f0fu) | (((hA[s] >> (2 * c + 1)) & 0x01010101u) << 4);
                    const uint32_t k1 = ((w1 >> 4) & 0x0f0f0f0fu) | (((hB[s] >> (2 * c + 1)) & 0x01010101u) << 4);
                    lo[s][0] = l0 & 0x001f001fu;
                    lo[s][1] = l1 & 0x001f001fu;
                    lo[s][2] = (l0 >> 8) & 0x001f001fu;
                    lo[s][3] = (l1 >> 8) & 0x001f001fu;
                    hi[s][0] = k0 & 0x001f001fu;
                    hi[s][1] = k1 & 0x001f001fu;
                    hi[s][2] = (k0 >> 8) & 0x001f001fu;
                    hi[s][3] = (k1 >> 8) & 0x001f001fu;
                }
            }
            const float2 slo = *reinterpret_cast<const float2*>(sc + (2 * c) * 16);
            const float2 shi = *reinterpret_cast<const float2*>(sc + (2 * c + 1) * 16);
            const int jl = seg0 + 4 * c, jh = jl + 2;  // low nibbles: k 64c..64c+31, high: 64c+32..
#pragma unroll
            for (int st = 0; st < NSET; st++) {
                Frag4 Cl{{0.f, 0.f, 0.f, 0.f}}, Ch{{0.f, 0.f, 0.f, 0.f}};
                uint2 b = bf.get(st, jl);
                mma16816(Cl, lo[0][0], lo[0][1], lo[0][2], lo[0][3], b.x, b.y);
                b = bf.get(st, jl + 1);
                mma16816(Cl, lo[1][0], lo[1][1], lo[1][2], lo[1][3], b.x, b.y);
                b = bf.get(st, jh);
                mma16816(Ch, hi[0][0], hi[0][1], hi[0][2], hi[0][3], b.x, b.y);
                b = bf.get(st, jh + 1);
                mma16816(Ch, hi[1][0], hi[1][1], hi[1][2], hi[1][3], b.x, b.y);
                scale_acc(acc[st], Cl, slo.x, slo.y);
                scale_acc(acc[st], Ch, shi.x, shi.y);
            }
        }
    } else {  // Q6_K: half h = 128 weights; ib selects l in [16ib, 16ib+16)
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
            // 6-bit values per byte (bits 6-7 are dropped by the pair masks below)
            const uint32_t v0[4] = {lop_sel(qa0, qh0 << 4, 0x0f0f0f0fu), lop_sel(qb0, qh0 << 2, 0x0f0f0f0fu),
                                    lop_sel(qa0 >> 4, qh0, 0x0f0f0f0fu), lop_sel(qb0 >> 4, qh0 >> 2, 0x0f0f0f0fu)};
            const uint32_t v1[4] = {lop_sel(qa1, qh1 << 4, 0x0f0f0f0fu), lop_sel(qb1, qh1 << 2, 0x0f0f0f0fu),
                                    lop_sel(qa1 >> 4, qh1, 0x0f0f0f0fu), lop_sel(qb1 >> 4, qh1 >> 2, 0x0f0f0f0fu)};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint32_t a0 = v0[q] & 0x003f003fu, a1 = v1[q] & 0x003f003fu;
                const uint32_t a2 = (v0[q] >> 8) & 0x003f003fu, a3 = (v1[q] >> 8) & 0x003f003fu;
                const int grp = 8 * h + 2 * q + ib;  // scale index; its 16 weights are k = 16*grp ..
                const float2 s = *reinterpret_cast<const float2*>(sc + grp * 16);
                const int j = seg0 + grp;
#pragma unroll
                for (int st = 0; st < NSET; st++) {
                    const uint2 b = bf.get(st, j);
                    Frag4 C{{0.f, 0.f, 0.f, 0.f}};
                    mma16816(C, a0, a1, a2, a3, b.x, b.y);
                    scale_acc(acc[st], C, s.x, s.y);
                }
            }
        }
    }
}

// ---- per-tile scale decode ----------------------------------------------------------------------
// For row r (of a row group) and super-block sb: the per-group multipliers of the MMA sums (the
// subnormal 2^24 / 2^20 factors folded in) into scl, and for each token the constant term
// (group minimums for Q4_K/Q5_K, the offset of 32 for Q6_K) into mins[tok].
template <int QT, typename Sx>
__device__ __forceinline__ void decode_scales(const uint8_t* __restrict__ blk, float* __restrict__ scl_rs, int ip, Sx sx16,
                                              int sb, int m, float* __restrict__ mins, int mstride) {
    if constexpr (QT == T_Q4_K || QT == T_Q5_K) {
        const uint32_t h0 = *reinterpret_cast<const uint32_t*>(blk);
        const uint32_t y = *reinterpret_cast<const uint32_t*>(blk + 4), z = *reinterpret_cast<const uint32_t*>(blk + 8),
                       w = *reinterpret_cast<const uint32_t*>(blk + 12);
        const float d = f16_to_f32(h0 & 0xffffu), dmin = f16_to_f32(h0 >> 16);
        // 6-bit scales/mins, word-parallel restatement of scale_min_k4 (qwen3moe.cpp:133-141)
        const uint32_t sA = y & 0x3f3f3f3fu, mA = z & 0x3f3f3f3fu;
        const uint32_t sB = (w & 0x0f0f0f0fu) | ((y >> 2) & 0x30303030u);
        const uint32_t mB = ((w >> 4) & 0x0f0f0f0fu) | ((z >> 2) & 0x30303030u);
        float mg[8];
#pragma unroll
        for (int gi = 0; gi < 8; gi++) {
            const uint32_t sw = gi < 4 ? sA : sB, mw = gi < 4 ? mA : mB;
            const int sh = 8 * (gi & 3);
            const float s = (float)((sw >> sh) & 63u), mn = (float)((mw >> sh) & 63u);
            const float f = (QT == T_Q4_K && (gi & 1)) ? P2_20 : P2_24;
            scl_rs[gi * 16 + ip] = d * s * f;
            mg[gi] = dmin * mn;
        }
        for (int tk = 0; tk < m; tk++) {
            const float* sx = sx16(tk) + sb * 16;
            float a = 0.f;
#pragma unroll
            for (int gi = 0; gi < 8; gi++) a = fmaf(mg[gi], __ldg(sx + 2 * gi) + __ldg(sx + 2 * gi + 1), a);
            mins[(size_t)tk * mstride] = a;
        }
    } else {
        const float d = f16_to_f32(*reinterpret_cast<const uint16_t*>(blk + 208));
        uint32_t sw[4];
#pragma unroll
        for (int i = 0; i < 4; i++) sw[i] = ld_u32_any(blk + 192 + 4 * i);
        float dsg[16];
#pragma unroll
        for (int gi = 0; gi < 16; gi++) {
            dsg[gi] = d * (float)(int8_t)(sw[gi >> 2] >> (8 * (gi & 3)));
            scl_rs[gi * 16 + ip] = dsg[gi] * P2_24;
        }
        for (int tk = 0; tk < m; tk++) {
            const float* sx = sx16(tk) + sb * 16;
            float a = 0.f;
#pragma unroll
            for (int gi = 0; gi < 16; gi++) a = fmaf(32.0f * dsg[gi], __ldg(sx + gi), a);
            mins[(size_t)tk * mstride] = a;
        }
    }
}

}  // namespace eb
