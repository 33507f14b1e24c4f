// gemm.cu -- the grouped tensor-core path of the MoE block for ragged batches (many tokens per expert):
// the per-expert projections as dense contractions on the 5th-generation tensor cores (tcgen05).
//
//   1. k_dequant_f16: every active expert's gate/up/down rows dequantized once (the reference decoders,
//      qwen3moe.cpp:142-202, exact fp32) and stored as f16 scaled by a per-row power of two, so that
//      the f16 rounding (2^-12 relative) is the only loss.
//   2. k_pack_f16: activation rows (tokens for gate/up, slots for down) as a per-row power-of-two
//      scale and an f16 hi/lo pair, x/s = hi + lo to ~2^-22.
//   3. k_gemm_tc<GATEUP>: tiles of (expert, 64 gate rows + the same 64 up rows, 128 slots); the K loop
//      stages W and both activation halves in shared memory (cp.async, two stages) as K-major core
//      matrices; one thread issues tcgen05.mma (M 128, N 128, K 16, f16 in, fp32 accumulate in tensor
//      memory) for hi and lo into the same accumulator and commits to an mbarrier; the epilogue reads
//      the accumulator with tcgen05.ld, pairs gate and up rows through shared memory and writes
//      h = SiLU(g) * u (qwen3moe.cpp:1056-1059) per slot.
//   4. k_gemm_tc<DOWN>: tiles of (expert, 128 rows of D, 128 slots) over h, writing y per slot; the
//      weighted combine in expert order is k_moe_combine (moe.cu).
#include <cuda_fp16.h>

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

// ---- 1. expert weights -> scaled f16, one warp per row of an active expert
__global__ void __launch_bounds__(256) k_dequant_f16(GroupedArgs g) {
    pdl_trigger();
    pdl_wait();
    const int rows_e = 2 * g.FF + g.D;  // gate, up, down rows of one expert
    const long long gw = ((long long)blockIdx.x * 256 + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int e = (int)(gw / rows_e), r = (int)(gw - (long long)e * rows_e);
    if (e >= g.E) return;
    if (g.offsets[e + 1] == g.offsets[e]) return;  // expert not routed in this call
    const int c = r < g.FF ? 0 : r < 2 * g.FF ? 1 : 2;
    const int row = c == 2 ? r - 2 * g.FF : r - c * g.FF;
    const int K = c == 2 ? g.FF : g.D;
    const uint8_t* src = g.w[c][e] + (size_t)row * g.rb[c];
    const int type = g.type[c];
    float m = 0.f;
    for (int i = 8 * lane; i < K; i += 256) {
        float y[8];
        dq8(src, type, i, y);
#pragma unroll
        for (int j = 0; j < 8; j++) m = fmaxf(m, fabsf(y[j]));
    }
    const float s = pow2_scale(warp_max(m)), inv = 1.f / s;  // exact: powers of two
    __half* dst = g.wf + (size_t)e * g.w_expert + g.w_off[c] + (size_t)row * K;
    for (int i = 8 * lane; i < K; i += 256) {
        float y[8];
        dq8(src, type, i, y);
        __align__(16) __half o[8];
#pragma unroll
        for (int j = 0; j < 8; j++) o[j] = __float2half_rn(y[j] * inv);
        *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(o);
    }
    if (lane == 0) g.rs[(size_t)e * rows_e + r] = s;
}

// ---- 2. fp32 rows -> scale + f16 hi/lo, one warp per row
__global__ void __launch_bounds__(256) k_pack_f16(const float* __restrict__ x, int n, int K, __half* __restrict__ hi,
                                                   __half* __restrict__ lo, float* __restrict__ scale) {
    pdl_trigger();
    pdl_wait();
    const int row = (blockIdx.x * 256 + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= n) return;
    const float* xr = x + (size_t)row * K;
    float m = 0.f;
    for (int i = 4 * lane; i < K; i += 128) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    const float s = pow2_scale(warp_max(m)), inv = 1.f / s;
    for (int i = 4 * lane; i < K; i += 128) {
        const float4 v = *reinterpret_cast<const float4*>(xr + i);
        const float a[4] = {v.x * inv, v.y * inv, v.z * inv, v.w * inv};
        __align__(8) __half h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            h[j] = __float2half_rn(a[j]);
            l[j] = __float2half_rn(a[j] - __half2float(h[j]));
        }
        *reinterpret_cast<uint2*>(hi + (size_t)row * K + i) = *reinterpret_cast<const uint2*>(h);
        *reinterpret_cast<uint2*>(lo + (size_t)row * K + i) = *reinterpret_cast<const uint2*>(l);
    }
    if (lane == 0) scale[row] = s;
}

// ---- 3/4. the grouped GEMM
constexpr int TC_KT = 64;                                 // K elements per stage
constexpr int TC_TILE_BYTES = 128 * TC_KT * 2;            // one 128-row f16 operand tile of a stage
constexpr int TC_STAGE_BYTES = 3 * TC_TILE_BYTES;         // W, activations hi, activations lo
constexpr int TC_SMEM = 2 * TC_STAGE_BYTES + 1024 + 512;  // two stages, slot scales/rows, barriers

template <int MODE>
__global__ void __launch_bounds__(128) k_gemm_tc(GroupedArgs g) {
    extern __shared__ __align__(1024) uint8_t smt[];
    uint8_t* stage0 = smt;
    float* s_bscale = reinterpret_cast<float*>(smt + 2 * TC_STAGE_BYTES);  // [128]
    int* s_brow = reinterpret_cast<int*>(smt + 2 * TC_STAGE_BYTES + 512);   // [128]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smt + 2 * TC_STAGE_BYTES + 1024);  // [2]
    __shared__ uint32_t s_tmem;
    __shared__ int s_info[4];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_trigger();
    pdl_wait();
    const int* tile_off = MODE == 0 ? g.tiles_gu : g.tiles_dn;
    if (tid == 0) {  // which (expert, slot tile, row tile)
        const int b = blockIdx.x, total = tile_off[g.E];
        int e = -1;
        if (b < total) {
            int lo_ = 0, hi_ = g.E;  // largest e with tile_off[e] <= b
            while (hi_ - lo_ > 1) {
                const int mid = (lo_ + hi_) >> 1;
                if (tile_off[mid] <= b) lo_ = mid;
                else hi_ = mid;
            }
            e = lo_;
        }
        s_info[0] = e;
        if (e >= 0) {
            const int RT = MODE == 0 ? g.FF / 64 : g.D / 128;
            const int local = b - tile_off[e];
            s_info[1] = local % RT;                           // row tile
            s_info[2] = g.offsets[e] + 128 * (local / RT);    // first slot
            s_info[3] = min(128, g.offsets[e + 1] - s_info[2]);  // slots in the tile
        }
    }
    __syncthreads();
    const int e = s_info[0];
    if (e < 0) return;
    const int rt = s_info[1], m0 = s_info[2], mc = s_info[3];
    const int K = MODE == 0 ? g.D : g.FF;
    // activation row of each slot of the tile, and its scale
    {
        const int j = tid;
        int br = 0;
        float bs = 0.f;
        if (j < mc) {
            br = MODE == 0 ? g.slot_token[m0 + j] : m0 + j;
            bs = (MODE == 0 ? g.xscale : g.hscale)[br];
        }
        s_brow[j] = br;
        s_bscale[j] = bs;
    }
    if (warp == 0) tc_alloc(&s_tmem, 128);
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const __half* We = g.wf + (size_t)e * g.w_expert;
    const __half* Bh = MODE == 0 ? g.xhi : g.hhi;
    const __half* Bl = MODE == 0 ? g.xlo : g.hlo;
    // source row of A row i (the tile's 128 rows)
    auto a_row = [&](int i) -> const __half* {
        if (MODE == 0)
            return We + (i < 64 ? g.w_off[0] : g.w_off[1]) + (size_t)(64 * rt + (i & 63)) * K;
        return We + g.w_off[2] + (size_t)(128 * rt + i) * K;
    };
    auto load_stage = [&](int s, int k0) {
        uint8_t* st = stage0 + s * TC_STAGE_BYTES;
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const int i = tid + 128 * q, r = i >> 3, c = i & 7;  // row r, 16-byte chunk c
            const uint32_t off = (uint32_t)(((r >> 3) * (TC_KT / 8) + c) * 128 + (r & 7) * 16);
            cp_async16_zfill(st + off, a_row(r) + k0 + 8 * c, 16);
            const bool ok = r < mc;
            const size_t boff = (size_t)s_brow[r] * K + k0 + 8 * c;
            cp_async16_zfill(st + TC_TILE_BYTES + off, Bh + boff, ok ? 16u : 0u);
            cp_async16_zfill(st + 2 * TC_TILE_BYTES + off, Bl + boff, ok ? 16u : 0u);
        }
    };
    constexpr uint32_t idesc = tc_idesc_f16(128, 128);
    const int nk = K / TC_KT;
    bool ok = true;
    for (int kt = 0; kt <= nk && ok; kt++) {
        if (kt < nk) {
            const int s = kt & 1;
            if (kt >= 2) ok = mbar_wait_bounded(&bars[s], (uint32_t)((kt - 2) >> 1) & 1u);
            load_stage(s, kt * TC_KT);
            cp_async_commit();
        }
        if (kt >= 1) {
            if (kt < nk) cp_async_wait<1>();
            else cp_async_wait<0>();
            fence_async_smem();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const int s = (kt - 1) & 1;
                const uint32_t base = smem_u32(stage0 + s * TC_STAGE_BYTES);
#pragma unroll
                for (int j = 0; j < TC_KT / 16; j++) {
                    const uint64_t da = tc_desc(base + 256 * j, 128, (TC_KT / 8) * 128);
                    const uint64_t dh = tc_desc(base + TC_TILE_BYTES + 256 * j, 128, (TC_KT / 8) * 128);
                    const uint64_t dl = tc_desc(base + 2 * TC_TILE_BYTES + 256 * j, 128, (TC_KT / 8) * 128);
                    tc_mma_f16(tmem, da, dh, idesc, (kt > 1 || j > 0) ? 1u : 0u);
                    tc_mma_f16(tmem, da, dl, idesc, 1u);
                }
                tc_commit(&bars[s]);
            }
        }
        ok = __syncthreads_and(ok);
    }
    if (ok) ok = mbar_wait_bounded(&bars[(nk - 1) & 1], (uint32_t)((nk - 1) >> 1) & 1u);
    ok = __syncthreads_and(ok);
    if (!ok) {
        cp_async_wait<0>();
        if (tid == 0 && g.status) atomicOr(g.status, ST_WAIT_TIMEOUT);
    } else {
        tc_fence_after();
        const int row = 32 * warp + lane;  // accumulator lane = A row
        const float* rs = g.rs + (size_t)e * (2 * g.FF + g.D);
        if (MODE == 0) {
            float* U = reinterpret_cast<float*>(stage0);  // [128 slots][64 rows] up values (stages are idle now)
            if (warp >= 2) {
                const float su = rs[g.FF + 64 * rt + row - 64];
                for (int c0 = 0; c0 < 128; c0 += 16) {
                    float v[16];
                    tc_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
#pragma unroll
                    for (int j = 0; j < 16; j++) U[(c0 + j) * 64 + row - 64] = v[j] * su;
                }
            }
            __syncthreads();
            if (warp < 2) {
                const float sg = rs[64 * rt + row];
                for (int c0 = 0; c0 < 128; c0 += 16) {
                    float v[16];
                    tc_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int col = c0 + j;
                        if (col < mc) {
                            const float bs = s_bscale[col];
                            const float gv = v[j] * sg * bs, uv = U[col * 64 + row] * bs;
                            g.h[(size_t)(m0 + col) * g.FF + 64 * rt + row] = silu_mul(gv, uv);
                        }
                    }
                }
            }
        } else {
            const float sd = rs[2 * g.FF + 128 * rt + row];
            for (int c0 = 0; c0 < 128; c0 += 16) {
                float v[16];
                tc_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int col = c0 + j;
                    if (col < mc) g.y[(size_t)(m0 + col) * g.D + 128 * rt + row] = v[j] * sd * s_bscale[col];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tc_dealloc(tmem, 128);
}

// ---- launchers ----------------------------------------------------------------------------------
cudaError_t launch_grouped_dequant(const GroupedArgs& g, cudaStream_t st) {
    const long long warps = (long long)g.E * (2 * g.FF + g.D);
    return launch_pdl(k_dequant_f16, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, st, g);
}
cudaError_t launch_pack_f16(const float* x, int n, int K, __half* hi, __half* lo, float* scale, cudaStream_t st) {
    if (n < 1 || K % 128) return cudaErrorInvalidValue;
    return launch_pdl(k_pack_f16, dim3((n + 7) / 8), dim3(256), 0, st, x, n, K, hi, lo, scale);
}
cudaError_t launch_grouped_gemm(const GroupedArgs& g, int mode, int max_tiles, cudaStream_t st) {
    if (g.D % 128 || g.FF % 64 || g.D % TC_KT || g.FF % TC_KT) return cudaErrorInvalidValue;
    if (max_tiles < 1) return cudaSuccess;
    if (mode == 0) {
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(k_gemm_tc<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
            attr = true;
        }
        return launch_pdl(k_gemm_tc<0>, dim3(max_tiles), dim3(128), TC_SMEM, st, g);
    }
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_gemm_tc<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
        attr = true;
    }
    return launch_pdl(k_gemm_tc<1>, dim3(max_tiles), dim3(128), TC_SMEM, st, g);
}

}  // namespace eb
