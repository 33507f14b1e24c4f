// gemm.cu -- the grouped tensor-core path of the MoE block for ragged batches (many tokens per expert):
// the per-expert projections as dense contractions on the 5th-generation tensor cores (tcgen05).
//
//   1. k_dequant_f16: every active expert's gate/up/down rows dequantized once (the reference decoders,
//      qwen3moe.cpp:142-202, exact fp32) and stored as f16 scaled by a per-row power of two (from a bound
//      read off the super-block headers), so that the f16 rounding (2^-12 relative) is the only loss.
//   2. k_token_scale + k_pack_groups / k_pack_slots: the activation rows of the slots (for gate/up each
//      token's xn, scaled and rounded to f16 once per token and copied per slot; for down each slot's h)
//      as a power-of-two scale and f16 values of x/s (2^-12 relative rounding, like the weights).
//   Both are written tile-major in the tensor cores' K-major core-matrix order (8 rows x 16 bytes), so
//   that one 64-element K stage of a 128-row tile is one contiguous 16 KB block: a single bulk copy.
//   3. k_gemm_tc<GATEUP>: persistent, warp-specialised. Tiles are (expert, 128 slots, 128 FF rows): the
//      slot tile is the MMA's A operand (M 128) and two 128-row weight blocks, each 64 gate rows + the
//      same 64 up rows, are B (N 256). A producer lane streams (slots, weight block, weight block) stage
//      blocks into a 4-deep shared-memory ring (1-D bulk copies, mbarrier complete_tx); one lane issues
//      tcgen05.mma (M 128, N 256, K 16, f16 in, fp32 accumulate in tensor memory) and commits each stage
//      back to the producer; two accumulators (all 512 tensor-memory columns) let four epilogue warps
//      read tile i (tcgen05.ld) while tile i+1 accumulates. An accumulator row is one slot holding its
//      gate and up values: each thread forms h = SiLU(g) * u (qwen3moe.cpp:1056-1059) for its own slot
//      and the warp writes the rows out as whole lines through a shared-memory transpose.
//   4. k_gemm_tc<DOWN>: tiles of (expert, 128 slots, 256 rows of D) over h, the same way, writing y per
//      slot; the weighted combine in expert order is k_moe_combine (moe.cu).
#include <cuda_fp16.h>

#include <algorithm>

#include "kernels.cuh"
#include "tc.cuh"

namespace eb {

namespace {
__device__ __forceinline__ float h16(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}
__device__ __forceinline__ void sm_k4(int j, const uint8_t* q, int& sc, int& mn) {
    if (j < 4) {
        sc = q[j] & 63;
        mn = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}
// Elements i .. i+7 (i a multiple of 8) of a quantized row, as the reference's decoders compute them.
__device__ void dq8(const uint8_t* row, int type, int i, float (&y)[8]) {
    if (type == T_Q4_K || type == T_Q5_K) {
        const bool q5 = type == T_Q5_K;
        const uint8_t* b = row + (i >> 8) * (q5 ? 176 : 144);
        const int e = i & 255, c = e >> 6, hi = (e >> 5) & 1, l0 = e & 31;
        int sc, mn;
        sm_k4(2 * c + hi, b + 4, sc, mn);
        const float d = h16(b) * (float)sc, o = h16(b + 2) * (float)mn;
        const uint8_t* qs = b + (q5 ? 48 : 16) + 32 * c + l0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int q = hi ? (qs[j] >> 4) : (qs[j] & 0x0f);
            if (q5) q += ((b[16 + l0 + j] >> (2 * c + hi)) & 1) << 4;
            y[j] = d * (float)q - o;
        }
    } else if (type == T_Q6_K) {
        const uint8_t* b = row + (i >> 8) * 210;
        const int e = i & 255, h = e >> 7, r = e & 127, quad = r >> 5, l0 = r & 31;
        const uint8_t* ql = b + 64 * h + ((quad & 1) ? 32 : 0) + l0;
        const uint8_t* qh = b + 128 + 32 * h + l0;
        const float d = h16(b + 208);
        const float s = (float)reinterpret_cast<const int8_t*>(b + 192)[8 * h + l0 / 16 + 2 * quad];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int q = (int)(((quad & 2) ? (ql[j] >> 4) : (ql[j] & 0x0f)) | (((qh[j] >> (2 * quad)) & 3) << 4)) - 32;
            y[j] = d * s * (float)q;
        }
    } else if (type == T_Q8_0) {
        const uint8_t* b = row + (i >> 5) * 34;
        const float d = h16(b);
#pragma unroll
        for (int j = 0; j < 8; j++) y[j] = d * (float)(int8_t)b[2 + (i & 31) + j];
    } else if (type == T_F16) {
#pragma unroll
        for (int j = 0; j < 8; j++) y[j] = h16(row + 2 * (i + j));
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) y[j] = reinterpret_cast<const float*>(row)[i + j];
    }
}
// power-of-two scale that brings max|x| into [2^13, 2^14) (1 for an all-zero row)
__device__ __forceinline__ float pow2_scale(float m) {
    if (!(m > 0.f) || !isfinite(m)) return 1.f;
    int e;
    frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1)
    return ldexpf(1.f, e - 14);
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
}  // namespace

// Tile-major core-matrix offset (elements) of element (r, k) of a 128-row tile whose K stages are
// consecutive 128 x 64 blocks: stage k / 64, then core matrix (r / 8, (k % 64) / 8), row r % 8.
__device__ __forceinline__ size_t tile_off(int r, int k) {
    return (size_t)(k >> 6) * (128 * 64) + (size_t)(((r >> 3) * 8 + ((k & 63) >> 3)) * 64 + (r & 7) * 8 + (k & 7));
}

// Byte k of w (0..255) as a float, exactly: the bit pattern 0x4B0000bb is 2^23 + bb.
template <int k>
__device__ __forceinline__ float byte_f(uint32_t w) {
    return __int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7650u | k)) - 8388608.f;
}
// little-endian 32-bit word at a 2-byte-aligned address
__device__ __forceinline__ uint32_t ld32_a2(const uint8_t* p) {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
    return (uint32_t)q[0] | ((uint32_t)q[1] << 16);
}
// One lane's share of a Q4_K / Q5_K super-block at b (16-byte aligned): elements 64 c + kq .. +15 of
// each of its four 64-element chunks c (kq a multiple of 16), times the power of two inv, as f16 pairs
// stored to dst + c * 8192 and dst + c * 8192 + 64 (the chunk's two core-matrix columns of this row in
// the tile). Same values as dq8: d q is exact in fp32 (an 11-bit f16 times a 6-bit scale times a 5-bit
// quant), so fma(d inv, q, -o inv) rounds (d q - o) once and scales it exactly. The header and the Q5_K
// high bits are read once per super-block; four quants per word: nibble masks, then byte permutes into
// 2^23 + q.
__device__ __forceinline__ void dq_sb_k45(const uint8_t* b, bool q5, int kq, float inv, __half* dst) {
    const int hi = kq >> 5, l0 = kq & 31;
    const uint4 hd = *reinterpret_cast<const uint4*>(b);  // d, dmin, 12 scale / min bytes
    const float dh = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xffff)));
    const float mh = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
    const uint4 hw = q5 ? *reinterpret_cast<const uint4*>(b + 16 + l0) : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t ha[4] = {hw.x, hw.y, hw.z, hw.w};
#pragma unroll
    for (int c = 0; c < 4; c++) {
        // scale / min of sub-block j = 2 c + hi: bytes j and j + 4 of the 12 (c < 2), or the low / high
        // nibbles of byte j + 4 with the top two bits of bytes j - 4 / j (c >= 2)
        const int j = 2 * c + hi, sh = 16 * (c & 1) + 8 * hi;
        int sc, mn;
        if (c < 2) {
            sc = (int)((hd.y >> sh) & 63);
            mn = (int)((hd.z >> sh) & 63);
        } else {
            const uint32_t bw = (hd.w >> sh) & 0xff, by = (hd.y >> sh) & 0xff, bz = (hd.z >> sh) & 0xff;
            sc = (int)((bw & 0x0f) | ((by >> 6) << 4));
            mn = (int)((bw >> 4) | ((bz >> 6) << 4));
        }
        const float d = dh * (float)sc * inv, mo = -(mh * (float)mn * inv);
        const uint4 qw = *reinterpret_cast<const uint4*>(b + (q5 ? 48 : 16) + 32 * c + l0);
        const uint32_t qa[4] = {qw.x, qw.y, qw.z, qw.w};
        __align__(16) __half2 o[8];
#pragma unroll
        for (int w = 0; w < 4; w++) {
            uint32_t nib = (qa[w] >> (4 * hi)) & 0x0f0f0f0fu;
            if (q5) nib |= ((ha[w] >> j) & 0x01010101u) << 4;
            o[2 * w] = __floats2half2_rn(fmaf(d, byte_f<0>(nib), mo), fmaf(d, byte_f<1>(nib), mo));
            o[2 * w + 1] = __floats2half2_rn(fmaf(d, byte_f<2>(nib), mo), fmaf(d, byte_f<3>(nib), mo));
        }
        *reinterpret_cast<uint4*>(dst + c * 8192) = *reinterpret_cast<const uint4*>(o);
        *reinterpret_cast<uint4*>(dst + c * 8192 + 64) = *reinterpret_cast<const uint4*>(o + 4);
    }
}
// The same for a Q6_K super-block at b (2-byte aligned): y = (d s inv) (q - 32), the reference's products
// in its order (d s, then times q - 32) scaled exactly. Chunks 2 h and 2 h + 1 take the low and high
// nibbles of the same 16 low-bit bytes and the 16 high-bit bytes at other shifts: each half reads them once.
__device__ __forceinline__ void dq_sb_q6k(const uint8_t* b, int kq, float inv, __half* dst) {
    const int hi = kq >> 5, l0 = kq & 31;
    const float dd = h16(b + 208);
    const int8_t* scl = reinterpret_cast<const int8_t*>(b + 192);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        uint32_t lw[4], hw[4];
#pragma unroll
        for (int w = 0; w < 4; w++) {
            lw[w] = ld32_a2(b + 64 * h + kq + 4 * w);  // = 64 h + 32 (quad & 1) + l0
            hw[w] = ld32_a2(b + 128 + 32 * h + l0 + 4 * w);
        }
#pragma unroll
        for (int cl = 0; cl < 2; cl++) {
            const int c = 2 * h + cl, quad = 2 * cl + hi, shift = 2 * quad;
            const float ds = dd * (float)scl[8 * h + (l0 >> 4) + 2 * quad] * inv;
            __align__(16) __half2 o[8];
#pragma unroll
            for (int w = 0; w < 4; w++) {
                const uint32_t v = (cl ? (lw[w] >> 4) & 0x0f0f0f0fu : lw[w] & 0x0f0f0f0fu) |
                                   (((hw[w] >> shift) & 0x03030303u) << 4);
                o[2 * w] = __floats2half2_rn(ds * (byte_f<0>(v) - 32.f), ds * (byte_f<1>(v) - 32.f));
                o[2 * w + 1] = __floats2half2_rn(ds * (byte_f<2>(v) - 32.f), ds * (byte_f<3>(v) - 32.f));
            }
            *reinterpret_cast<uint4*>(dst + c * 8192) = *reinterpret_cast<const uint4*>(o);
            *reinterpret_cast<uint4*>(dst + c * 8192 + 64) = *reinterpret_cast<const uint4*>(o + 4);
        }
    }
}

// SiLU(g) * u with the fast exponential and division (a few ulp): this path's operands already carry
// the f16 rounding, 2^-12 relative, so the IEEE forms of the single-token kernels buy nothing here.
__device__ __forceinline__ float silu_mul_fast(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

// Upper bound of |y| over super-block sb of a K-quant row, from its header alone: Q4_K / Q5_K
// y = d sc q - dmin m with q in [0, 15] / [0, 31]; Q6_K y = d sc (q - 32) with q - 32 in [-32, 31].
__device__ float kq_bound(const uint8_t* row, int type, int sb) {
    if (type == T_Q6_K) {
        const uint8_t* b = row + (size_t)sb * 210;
        int ms = 0;
#pragma unroll
        for (int j = 0; j < 16; j++) ms = max(ms, abs((int)reinterpret_cast<const int8_t*>(b + 192)[j]));
        return fabsf(h16(b + 208)) * (float)ms * 32.f;
    }
    const bool q5 = type == T_Q5_K;
    const uint8_t* b = row + (size_t)sb * (q5 ? 176 : 144);
    const float d = fabsf(h16(b)), dm = fabsf(h16(b + 2)), qmax = q5 ? 31.f : 15.f;
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        int sc, mn;
        sm_k4(j, b + 4, sc, mn);
        m = fmaxf(m, d * (float)sc * qmax + dm * (float)mn);
    }
    return m;
}

// ---- 1. expert weights -> scaled f16, tile-major; one warp per 8-row group of an active expert
// Per expert: gate/up blocks (FF/64 of them; rows 0..63 = gate rows 64 blk.., 64..127 = the same up rows;
// D/64 stages), then down blocks (D/128 of 128 rows, FF/64 stages). Each row's scale is the power of two of an upper
// bound of its max|y|; the bound only has to keep the f16 values below 2^14, and since the scale is a
// power of two the f16 rounding of y / s is the same whatever binade it lands in. K-quant rows take the
// bound from their super-block headers (one decode pass), other types decode twice. Eight rows of one
// core-matrix row group per warp: every 64-element K chunk of the group is one contiguous 1 KB block
// of the tile, written by the warp as 32 x 2 full-line 16-byte stores.
// The group's 8 rows are one contiguous span of 8 x row-bytes; when it is 16-byte aligned the warp first
// copies it into its shared-memory slot (`stage` bytes per warp) with every 16-byte load in flight at
// once, and decodes from there.
constexpr int DQ_WARPS = 4;
__global__ void __launch_bounds__(32 * DQ_WARPS) k_dequant_f16(GroupedArgs g, int stage) {
    extern __shared__ __align__(16) uint8_t dq_raw[];
    pdl_wait();
    pdl_trigger();
    const int rows_e = 2 * g.FF + g.D;  // gate, up, down rows of one expert
    const int groups_e = rows_e / 8;
    const long long gw = ((long long)blockIdx.x * (32 * DQ_WARPS) + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int e = (int)(gw / groups_e), r0 = 8 * (int)(gw - (long long)e * groups_e);
    if (e >= g.E) return;
    if (g.offsets[e + 1] == g.offsets[e]) return;  // expert not routed in this call
    const int c = r0 < g.FF ? 0 : r0 < 2 * g.FF ? 1 : 2;
    const int row0 = c == 2 ? r0 - 2 * g.FF : r0 - c * g.FF;
    const int K = c == 2 ? g.FF : g.D;
    const size_t rb = g.rb[c];
    const int type = g.type[c];
    const uint8_t* src0 = g.w[c][e] + (size_t)row0 * rb;
    const size_t span = 8 * rb;
    if (stage && span <= (size_t)stage && span % 16 == 0 && (reinterpret_cast<uintptr_t>(src0) & 15) == 0) {
        uint4* dst = reinterpret_cast<uint4*>(dq_raw + (size_t)(threadIdx.x >> 5) * stage);
        const uint4* gsrc = reinterpret_cast<const uint4*>(src0);
        const int n16 = (int)(span / 16);
#pragma unroll 8
        for (int i = lane; i < n16; i += 32) dst[i] = __ldg(gsrc + i);
        __syncwarp();
        src0 = reinterpret_cast<const uint8_t*>(dst);
    }
    float m_own = 0.f;  // lane r < 8: the bound of row r of the group
    for (int r = 0; r < 8; r++) {
        float m = 0.f;
        if (is_kquant(type)) {
            for (int sb = lane; sb < K / 256; sb += 32) m = fmaxf(m, kq_bound(src0 + (size_t)r * rb, type, sb));
        } else {
            for (int i = 8 * lane; i < K; i += 256) {
                float y[8];
                dq8(src0 + (size_t)r * rb, type, i, y);
#pragma unroll
                for (int j = 0; j < 8; j++) m = fmaxf(m, fabsf(y[j]));
            }
        }
        m = warp_max(m);
        if (lane == r) m_own = m;
    }
    const float s_own = pow2_scale(m_own);
    // this lane: row r of the group, elements 16 (lane % 4) .. +15 of every 64-element chunk
    const int r = lane >> 2, kq = 16 * (lane & 3), row = row0 + r;
    const float inv = 1.f / __shfl_sync(0xffffffffu, s_own, r);  // exact: powers of two
    const uint8_t* src = src0 + (size_t)r * rb;
    const bool fast45 = (type == T_Q4_K || type == T_Q5_K) && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
    const bool fast6 = type == T_Q6_K && (reinterpret_cast<uintptr_t>(src) & 1) == 0;
    const int bsz = type == T_Q5_K ? 176 : type == T_Q6_K ? 210 : 144;
    __half* base = g.wf + (size_t)e * g.w_expert;
    int ar;  // row within its 128-row tile
    if (c < 2) {
        base += (size_t)(row >> 6) * 128 * K;
        ar = (c == 0 ? 0 : 64) + (row & 63);
    } else {
        base += (size_t)2 * g.FF * g.D + (size_t)(row >> 7) * 128 * K;
        ar = row & 127;
    }
    if (fast45 || fast6) {
        // super-block sb of the row: chunks 4 sb .. 4 sb + 3, each a 128 x 64 block (8192 elements) of
        // the tile; this lane's two 8-element words of a chunk are at tile_off(ar, 64 c + kq) and + 8
        __half* dst = base + tile_off(ar, kq);
        for (int sb = 0; sb < K / 256; sb++, dst += 4 * 8192) {
            if (fast45) dq_sb_k45(src + (size_t)sb * bsz, type == T_Q5_K, kq, inv, dst);
            else dq_sb_q6k(src + (size_t)sb * bsz, kq, inv, dst);
        }
    } else {
        for (int k0 = 0; k0 < K; k0 += 64) {
            const int i = k0 + kq;
            __align__(16) __half2 o[8];
            float y[8], z[8];
            dq8(src, type, i, y);
            dq8(src, type, i + 8, z);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                o[j] = __floats2half2_rn(y[2 * j] * inv, y[2 * j + 1] * inv);
                o[4 + j] = __floats2half2_rn(z[2 * j] * inv, z[2 * j + 1] * inv);
            }
            *reinterpret_cast<uint4*>(base + tile_off(ar, i)) = *reinterpret_cast<const uint4*>(o);
            *reinterpret_cast<uint4*>(base + tile_off(ar, i + 8)) = *reinterpret_cast<const uint4*>(o + 4);
        }
    }
    if (lane < 8) g.rs[(size_t)e * rows_e + r0 + lane] = s_own;
}

// ---- 2a. gate/up activations. k_token_scale: one warp per token, the power-of-two scale of its xn row
// and the row as f16 of x / s (g.xh, half the bytes of the fp32 row, so that the rows stay in L2 while
// every slot of the token copies them). k_pack_groups: one warp per 8 consecutive slots of one expert's
// slot tile (a core-matrix row group): each 64-element K chunk of the group is one contiguous 1 KB block
// of the tile, copied from the tokens' f16 rows and written as whole lines (evict-first, so the stream
// of tile lines does not push the f16 rows out of L2); rows past the expert's slots are written as zeros.
__global__ void __launch_bounds__(256) k_token_scale(GroupedArgs g) {
    pdl_wait();
    pdl_trigger();
    const int t = (blockIdx.x * 256 + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (t >= g.T) return;
    const float* xr = g.xn + (size_t)t * g.D;
    float m = 0.f;
    for (int i = 4 * lane; i < g.D; i += 128) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    m = warp_max(m);
    const float sc = pow2_scale(m), inv = 1.f / sc;
    __half* xo = g.xh + (size_t)t * g.D;
    for (int i = 4 * lane; i < g.D; i += 128) {  // the row again (L1 / L2), as f16 of x / s
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        __align__(8) __half2 hv[2];
        hv[0] = __floats2half2_rn(v.x * inv, v.y * inv);
        hv[1] = __floats2half2_rn(v.z * inv, v.w * inv);
        *reinterpret_cast<uint2*>(xo + i) = *reinterpret_cast<const uint2*>(hv);
    }
    if (lane == 0) g.tscale[t] = sc;
}

__global__ void __launch_bounds__(256) k_pack_groups(GroupedArgs g) {
    pdl_wait();
    pdl_trigger();
    const long long gw = ((long long)blockIdx.x * 256 + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31, RT = g.FF / GU_TILE_ROWS;
    const int bt = (int)(gw >> 4), grp = (int)(gw & 15);  // slot tile, row group within it
    if ((long long)bt * RT >= g.tiles_gu[g.E]) return;
    int lo_ = 0, hi_ = g.E;  // expert of the slot tile: largest e with tiles_gu[e] <= bt RT
    while (hi_ - lo_ > 1) {
        const int mid = (lo_ + hi_) >> 1;
        if (g.tiles_gu[mid] <= bt * RT) lo_ = mid;
        else hi_ = mid;
    }
    const int e = lo_, cnt = g.offsets[e + 1] - g.offsets[e];
    const int j0 = 128 * (bt - g.tiles_gu[e] / RT) + 8 * grp;
    if (j0 >= cnt) return;
    const int r = lane >> 2, kq = 16 * (lane & 3), jr = 8 * grp + r, K = g.D;
    const bool valid = j0 + r < cnt;
    const int slot = g.offsets[e] + j0 + r;
    const int tok = valid ? g.slot_token[slot] : 0;
    // this lane's 16 elements of every 64-element chunk: two 16-byte words of the token's f16 row
    const uint4* xr = reinterpret_cast<const uint4*>(g.xh + (size_t)tok * K + kq);
    __half* bh = g.bhi + (size_t)bt * 128 * K;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    for (int k0 = 0; k0 < K; k0 += 256) {  // four 64-element chunks: all loads first, then the stores
        uint4 v[4][2];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const bool in = valid && k0 + 64 * u < K;
            v[u][0] = in ? __ldg(xr + (k0 + 64 * u) / 8) : zero;
            v[u][1] = in ? __ldg(xr + (k0 + 64 * u) / 8 + 1) : zero;
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (k0 + 64 * u >= K) break;
            const int i = k0 + 64 * u + kq;
            __stcs(reinterpret_cast<uint4*>(bh + tile_off(jr, i)), v[u][0]);
            __stcs(reinterpret_cast<uint4*>(bh + tile_off(jr, i + 8)), v[u][1]);
        }
    }
    if (valid && (lane & 3) == 0) g.bscale[slot] = g.tscale[tok];
}

// ---- 2b. down activations: each slot's h row -> power-of-two scale + f16, tile-major by (expert, slot
// tile). One warp per 8 consecutive slots of one expert's slot tile (a core-matrix row group), four lanes
// per slot: the row's max in a first pass over it, then every 64-element K chunk of the group written as
// one contiguous 1 KB block of whole lines (rows past the expert's slots as zeros).
__global__ void __launch_bounds__(256) k_pack_slots(GroupedArgs g) {
    pdl_wait();
    pdl_trigger();
    const long long gw = ((long long)blockIdx.x * 256 + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31, RT = g.FF / GU_TILE_ROWS;
    const int bt = (int)(gw >> 4), grp = (int)(gw & 15);  // slot tile, row group within it
    if ((long long)bt * RT >= g.tiles_gu[g.E]) return;
    int lo_ = 0, hi_ = g.E;  // expert of the slot tile: largest e with tiles_gu[e] <= bt RT
    while (hi_ - lo_ > 1) {
        const int mid = (lo_ + hi_) >> 1;
        if (g.tiles_gu[mid] <= bt * RT) lo_ = mid;
        else hi_ = mid;
    }
    const int e = lo_, cnt = g.offsets[e + 1] - g.offsets[e];
    const int j0 = 128 * (bt - g.tiles_gu[e] / RT) + 8 * grp;
    if (j0 >= cnt) return;
    const int r = lane >> 2, kq = 16 * (lane & 3), jr = 8 * grp + r, K = g.FF;
    const bool valid = j0 + r < cnt;
    const int slot = g.offsets[e] + j0 + r;
    const float* xr = g.h + (size_t)(valid ? slot : g.offsets[e] + j0) * K + kq;
    float m = 0.f;
    for (int k0 = 0; k0 < K; k0 += 64) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 v = *reinterpret_cast<const float4*>(xr + k0 + 4 * q);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));  // the row's four lanes
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const float sc = valid ? pow2_scale(m) : 1.f, inv = valid ? 1.f / sc : 0.f;
    __half* bh = g.bhi + (size_t)bt * 128 * K;
    for (int k0 = 0; k0 < K; k0 += 256) {  // four 64-element chunks: all loads first, then the stores
        float4 v[4][4];
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
            for (int q = 0; q < 4; q++)
                v[u][q] = k0 + 64 * u < K ? *reinterpret_cast<const float4*>(xr + k0 + 64 * u + 4 * q)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (k0 + 64 * u >= K) break;
            __align__(16) __half2 hv[8];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                hv[2 * q] = __floats2half2_rn(v[u][q].x * inv, v[u][q].y * inv);
                hv[2 * q + 1] = __floats2half2_rn(v[u][q].z * inv, v[u][q].w * inv);
            }
            const int i = k0 + 64 * u + kq;
            *reinterpret_cast<uint4*>(bh + tile_off(jr, i)) = *reinterpret_cast<const uint4*>(hv);
            *reinterpret_cast<uint4*>(bh + tile_off(jr, i + 8)) = *reinterpret_cast<const uint4*>(hv + 4);
        }
    }
    if (valid && (lane & 3) == 0) g.bscale[slot] = sc;
}

// ---- 3/4. the grouped GEMM
constexpr int TC_KT = 64;                     // K elements per stage
constexpr int TC_BLOCK = 128 * TC_KT * 2;     // one 128-row f16 stage block: 16 KB
constexpr int TC_STAGES = 4;
constexpr int TC_STAGE_BYTES = 3 * TC_BLOCK;  // the slot tile (A), two 128-row weight blocks (B)
constexpr int TC_XP = 36;                     // row stride (floats) of an epilogue transpose tile
constexpr int TC_U_BYTES = 4 * 32 * TC_XP * 4;  // one 32 x 32 transpose tile per epilogue warp
constexpr int TC_SMEM = TC_STAGES * TC_STAGE_BYTES + TC_U_BYTES + 256;
constexpr int TC_NT = 192;  // warp 0 producer, warp 1 MMA + tensor-memory owner, warps 2..5 epilogue
constexpr int TC_N = 256;   // accumulator columns of a tile: two weight blocks

struct TcTile {
    int e, rt, m0, mc, btile;
};
// tile b of the GEMM (tiles of one expert: row tile fastest, then slot tile)
template <int MODE>
__device__ __forceinline__ bool tc_tile(const GroupedArgs& g, int b, TcTile& t) {
    const int* off = MODE == 0 ? g.tiles_gu : g.tiles_dn;
    if (b >= off[g.E]) return false;
    int lo_ = 0, hi_ = g.E;
    while (hi_ - lo_ > 1) {
        const int mid = (lo_ + hi_) >> 1;
        if (off[mid] <= b) lo_ = mid;
        else hi_ = mid;
    }
    const int RT = MODE == 0 ? g.FF / GU_TILE_ROWS : g.D / DN_TILE_ROWS;
    const int local = b - off[lo_], st = local / RT;
    t.e = lo_;
    t.rt = local - st * RT;
    t.m0 = g.offsets[lo_] + 128 * st;
    t.mc = min(128, g.offsets[lo_ + 1] - t.m0);
    t.btile = g.tiles_gu[lo_] / (g.FF / GU_TILE_ROWS) + st;
    return true;
}

// D[128 slots x 256] = A[slot tile] * B[two weight blocks]^T over K. Gate/up: weight blocks 2 rt and 2 rt + 1
// (each 64 gate rows + the same 64 up rows), so accumulator columns 0..63 / 64..127 pair the gate and up
// values of FF rows 128 rt + 0..63 and columns 128..255 those of rows + 64..127. Down: blocks 2 rt, 2 rt + 1
// are D rows 256 rt + 0..255 = the columns. An accumulator row is one slot: each epilogue thread finishes
// its own slot's row and the warp writes 32 rows x 32 columns at a time through its transpose tile.
template <int MODE>
__global__ void __launch_bounds__(TC_NT, 1) k_gemm_tc(GroupedArgs g) {
    extern __shared__ __align__(1024) uint8_t smt[];
    float* U = reinterpret_cast<float*>(smt + TC_STAGES * TC_STAGE_BYTES);  // [4 warps][32][TC_XP]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smt + TC_STAGES * TC_STAGE_BYTES + TC_U_BYTES);
    uint64_t* full = bars;                    // [TC_STAGES] stage landed
    uint64_t* empty = bars + TC_STAGES;       // [TC_STAGES] stage consumed by the MMAs
    uint64_t* acc_full = bars + 2 * TC_STAGES;       // [2] accumulator complete
    uint64_t* acc_empty = bars + 2 * TC_STAGES + 2;  // [2] accumulator read out (4 epilogue warps)
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = MODE == 0 ? g.D : g.FF, nk = K / TC_KT;
    if (warp == 1) tc_alloc(&s_tmem, 2 * TC_N);
    if (tid == 0) {
        for (int i = 0; i < TC_STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);
        }
        s_abort = 0;
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_wait();  // routing, packed activations and weights come from the previous grids
    pdl_trigger();
    const uint32_t tmem = s_tmem;
    auto fail = [&]() {
        if (g.status) atomicOr(g.status, ST_WAIT_TIMEOUT);
        atomicExch(&s_abort, 1);
    };
    if (warp == 0) {  // ---------------- producer
        if (lane == 0) {
            int it = 0;  // stage fills issued
            TcTile t;
            for (int b = blockIdx.x; tc_tile<MODE>(g, b, t) && !*(volatile int*)&s_abort; b += gridDim.x) {
                const __half* W = g.wf + (size_t)t.e * g.w_expert + (MODE == 0 ? 0 : (size_t)2 * g.FF * g.D) +
                                  (size_t)(2 * t.rt) * 128 * K;
                const __half* X = g.bhi + (size_t)t.btile * 128 * K;
                for (int kt = 0; kt < nk; kt++, it++) {
                    const int s = it % TC_STAGES;
                    if (it >= TC_STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)(it / TC_STAGES - 1) & 1u)) {
                        fail();
                        break;
                    }
                    uint8_t* dst = smt + s * TC_STAGE_BYTES;
                    mbar_expect_tx(&full[s], 3 * TC_BLOCK);
                    tma_load_1d(dst, X + (size_t)kt * 128 * TC_KT, TC_BLOCK, &full[s]);
                    tma_load_1d(dst + TC_BLOCK, W + (size_t)kt * 128 * TC_KT, TC_BLOCK, &full[s]);
                    tma_load_1d(dst + 2 * TC_BLOCK, W + (size_t)128 * K + (size_t)kt * 128 * TC_KT, TC_BLOCK, &full[s]);
                }
            }
            // no copy may still be landing when the CTA exits: wait for the last fill of every stage
            for (int k = (it > TC_STAGES ? it - TC_STAGES : 0); k < it; k++)
                if (!mbar_wait_bounded(&full[k % TC_STAGES], (uint32_t)(k / TC_STAGES) & 1u)) break;
        }
    } else if (warp == 1) {  // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc_f16(128, TC_N);
            int it = 0, ti = 0;
            TcTile t;
            for (int b = blockIdx.x; tc_tile<MODE>(g, b, t); b += gridDim.x, ti++) {
                const int a = ti & 1;
                if (ti >= 2 && !mbar_wait_bounded(&acc_empty[a], (uint32_t)(ti / 2 - 1) & 1u)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(TC_N * a);
                bool ok = true;
                for (int kt = 0; kt < nk; kt++, it++) {
                    const int s = it % TC_STAGES;
                    if (!mbar_wait_bounded(&full[s], (uint32_t)(it / TC_STAGES) & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t abase = smem_u32(smt + s * TC_STAGE_BYTES), bbase = abase + TC_BLOCK;
#pragma unroll
                    for (int j = 0; j < TC_KT / 16; j++) {
                        // K-major core matrices: 128 B between the two K chunks of a step, 1 KB between row
                        // groups (the second weight block's row groups continue the first's)
                        const uint64_t da = tc_desc(abase + 256 * j, 128, (TC_KT / 8) * 128);
                        const uint64_t db = tc_desc(bbase + 256 * j, 128, (TC_KT / 8) * 128);
                        tc_mma_f16(acc, da, db, idesc, (kt > 0 || j > 0) ? 1u : 0u);
                    }
                    tc_commit(&empty[s]);  // the stage is free once these MMAs completed
                }
                if (!ok) {
                    fail();
                    break;
                }
                tc_commit(&acc_full[a]);
            }
        }
    } else {  // ---------------- epilogue: warps 2..5, tensor-memory lane quadrant warp % 4
        const int q = warp & 3;
        float* xp = U + (warp - 2) * (32 * TC_XP);  // this warp's 32 x 32 transpose tile
        const int sl = 32 * q + lane;                 // this thread's slot within the tile
        int ti = 0;
        TcTile t;
        for (int b = blockIdx.x; tc_tile<MODE>(g, b, t); b += gridDim.x, ti++) {
            const int a = ti & 1;
            // the tile's row scales (this lane's one per 32-column pass) and its slot's scale, loaded
            // before the accumulator wait so that no pass waits on them
            const float* rs = g.rs + (size_t)t.e * (2 * g.FF + g.D);
            const float bs = sl < t.mc ? g.bscale[t.m0 + sl] : 0.f;
            float rsc[8];
#pragma unroll
            for (int k = 0; k < 8; k++)
                rsc[k] = MODE == 0 ? rs[(k & 1) * g.FF + 128 * t.rt + 32 * (k >> 1) + lane]  // gate / up, pass k / 2
                                   : rs[2 * g.FF + 256 * t.rt + 32 * k + lane];              // down, pass k
            bool ok = mbar_wait_bounded(&acc_full[a], (uint32_t)(ti / 2) & 1u);
            ok = __all_sync(0xffffffffu, ok);  // the tensor-memory loads below are warp-collective
            if (!ok && lane == 0) fail();
            tc_fence_after();
            const uint32_t acc = tmem + (uint32_t)(TC_N * a) + ((uint32_t)(32 * q) << 16);
            // one pass: 32 output columns of this thread's row, scaled, through the transpose tile to
            // out + row * ld + col0 (rows of the tile's slots only)
            auto emit = [&](float (&v)[32], float* out, int ld, int col0) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(xp + lane * TC_XP + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                __syncwarp();
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int r = 4 * i + (lane >> 3), c = 4 * (lane & 7), sr = 32 * q + r;
                    if (sr < t.mc)
                        *reinterpret_cast<float4*>(out + (size_t)(t.m0 + sr) * ld + col0 + c) =
                            *reinterpret_cast<const float4*>(xp + r * TC_XP + c);
                }
                __syncwarp();
            };
            if (MODE == 0 && ok) {
#pragma unroll
                for (int qq = 0; qq < 4; qq++) {  // FF rows 128 rt + 32 qq + 0..31
                    const int fr = 128 * t.rt + 32 * qq, gcol = (qq >> 1) * 128 + (qq & 1) * 32;
                    const float sg = rsc[2 * qq], su = rsc[2 * qq + 1];
                    float hv[32];
#pragma unroll
                    for (int c0 = 0; c0 < 32; c0 += 16) {
                        float gv[16], uv[16];
                        tc_ld16x2(acc + (uint32_t)(gcol + c0), acc + (uint32_t)(gcol + 64 + c0), gv, uv);
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const float gs = __shfl_sync(0xffffffffu, sg, c0 + j), us = __shfl_sync(0xffffffffu, su, c0 + j);
                            hv[c0 + j] = silu_mul_fast(gv[j] * gs * bs, uv[j] * us * bs);
                        }
                    }
                    emit(hv, g.h, g.FF, fr);
                }
            } else if (ok) {
#pragma unroll
                for (int p = 0; p < 8; p++) {  // D rows 256 rt + 32 p + 0..31
                    const int dr = 256 * t.rt + 32 * p;
                    const float sd = rsc[p];
                    float yv[32], v[16], w[16];
                    tc_ld16x2(acc + (uint32_t)(32 * p), acc + (uint32_t)(32 * p + 16), v, w);
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        yv[j] = v[j] * __shfl_sync(0xffffffffu, sd, j) * bs;
                        yv[16 + j] = w[j] * __shfl_sync(0xffffffffu, sd, 16 + j) * bs;
                    }
                    emit(yv, g.y, g.D, dr);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
            if (!ok) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tc_dealloc(tmem, 2 * TC_N);
}

// ---- launchers ----------------------------------------------------------------------------------
cudaError_t launch_grouped_dequant(const GroupedArgs& g, cudaStream_t st) {
    if (g.FF % 8 || g.D % 8) return cudaErrorInvalidValue;
    const long long warps = (long long)g.E * ((2 * g.FF + g.D) / 8);
    size_t span = 0;
    for (int c = 0; c < 3; c++) span = std::max(span, 8 * g.rb[c]);
    int stage = (int)((span + 15) / 16 * 16);
    if ((size_t)stage * DQ_WARPS > 200 * 1024) stage = 0;  // rows too long to stage: decode from global memory
    const int smem = stage * DQ_WARPS;
    static int attr = 0;
    if (smem > 48 * 1024 && smem > attr) {
        if (cudaFuncSetAttribute(k_dequant_f16, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return cudaErrorInvalidValue;
        attr = smem;
    }
    return launch_pdl(k_dequant_f16, dim3((unsigned)((warps + DQ_WARPS - 1) / DQ_WARPS)), dim3(32 * DQ_WARPS), smem, st,
                      g, stage);
}
cudaError_t launch_pack_tokens(const GroupedArgs& g, int slot_tiles, cudaStream_t st) {
    if (g.T < 1 || slot_tiles < 1) return cudaSuccess;
    if (g.D % 64) return cudaErrorInvalidValue;
    cudaError_t err = launch_pdl(k_token_scale, dim3((g.T + 7) / 8), dim3(256), 0, st, g);
    if (err != cudaSuccess) return err;
    return launch_pdl(k_pack_groups, dim3((unsigned)(((long long)slot_tiles * 16 + 7) / 8)), dim3(256), 0, st, g);
}
cudaError_t launch_pack_slots(const GroupedArgs& g, int slot_tiles, cudaStream_t st) {
    if (slot_tiles < 1) return cudaSuccess;
    if (g.FF % 64) return cudaErrorInvalidValue;
    return launch_pdl(k_pack_slots, dim3((unsigned)(((long long)slot_tiles * 16 + 7) / 8)), dim3(256), 0, st, g);
}
cudaError_t launch_grouped_gemm(const GroupedArgs& g, int mode, int max_tiles, cudaStream_t st) {
    if (g.D % DN_TILE_ROWS || g.FF % GU_TILE_ROWS || g.D % TC_KT || g.FF % TC_KT) return cudaErrorInvalidValue;
    if (max_tiles < 1) return cudaSuccess;
    const int grid = std::min(max_tiles, sm_count());
    if (mode == 0) {
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(k_gemm_tc<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
            attr = true;
        }
        return launch_pdl(k_gemm_tc<0>, dim3(grid), dim3(TC_NT), TC_SMEM, st, g);
    }
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_gemm_tc<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
        attr = true;
    }
    return launch_pdl(k_gemm_tc<1>, dim3(grid), dim3(TC_NT), TC_SMEM, st, g);
}

}  // namespace eb
