// kernels.cu -- sm_100a kernels of the MoE expert hot path.
//
//   k_prep_x            activations -> fragment form (f16 high/low split, per-16 sums, power-of-two
//                       scale), once per token row, read by every weight tile afterwards.
//   k_gemv<QT,N>        dense quantized GEMV (attention/output rows, the C ABI): 16-row tiles streamed
//                       HBM -> shared memory by 1-D TMA bulk copies (two-slot mbarrier ring per CTA,
//                       several small CTAs per SM) and decoded in registers straight into tensor-core
//                       operands (kq.cuh).
//   k_gemv_generic      one warp per row for F32/F16/Q8_0 and for buffers TMA cannot address.
//   k_route_permute     router softmax + top-k + renormalisation (warp per token, the CPU comparator of
//                       qwen3moe.cpp:1016) fused with the token->expert grouping (histogram, exclusive
//                       scan, stable scatter), one CTA, no host round trip.
//   k_moe_gateup<G,U>   gate and up projections of every routed (expert, token) pair with SiLU(g)*u in
//                       the epilogue; work = (active expert, 16-row group) units split evenly over the grid.
//   k_moe_down<QD>      down projection per (16-row group, active expert) unit, fused with the router-
//                       weighted combine and the residual add: the CTA completing a row group adds each
//                       token's expert outputs in ascending expert order (qwen3moe.cpp:1025-1069).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "kq.cuh"

namespace eb {

// ------------------------------------------------------------------------------------------------
// small helpers
// ------------------------------------------------------------------------------------------------
struct Span {
    const uint8_t* src;  // 16-byte aligned copy source
    uint32_t lead;       // bytes between src and the first row
    uint32_t bytes;      // copy size, multiple of 16
};
// Rows [r0, r1) of a matrix, widened to 16-byte boundaries for cp.async.bulk.
__device__ __forceinline__ Span row_span(const uint8_t* base, size_t rb, int r0, int r1) {
    const uintptr_t s = reinterpret_cast<uintptr_t>(base) + (size_t)r0 * rb;
    const uintptr_t e = reinterpret_cast<uintptr_t>(base) + (size_t)r1 * rb;
    const uintptr_t as = s & ~(uintptr_t)15, ae = (e + 15) & ~(uintptr_t)15;
    return {reinterpret_cast<const uint8_t*>(as), (uint32_t)(s - as), (uint32_t)(ae - as)};
}
__device__ __forceinline__ uint32_t align16(uint32_t x) { return (x + 15u) & ~15u; }

__device__ __forceinline__ void flag(int* status, int bits) {
    if (status) atomicOr(status, bits);
}

// After a timed-out wait: give every slot that may still have a copy in flight one more bounded wait,
// so the CTA does not retire with bulk copies still writing its shared memory.
__device__ void drain_ring(uint64_t* bar, int issued, int consumed, int depth) {
    for (int i = consumed; i < issued; i++) mbar_wait_bounded(&bar[i % depth], (uint32_t)(i / depth) & 1u);
}

// ------------------------------------------------------------------------------------------------
// generic per-element decode (F32, F16, Q8_0 and K-quants), one weight at a time
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ int kq_scale(const uint8_t* q, int j, int* mn) {
    if (j < 4) {
        *mn = q[j + 4] & 63;
        return q[j] & 63;
    }
    *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    return (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
}
__device__ __forceinline__ float rd_f16(const uint8_t* p) { return f16_to_f32((uint32_t)p[0] | ((uint32_t)p[1] << 8)); }

__device__ float weight_at(const uint8_t* row, int type, int k) {
    switch (type) {
        case T_F32: {
            float v;
            memcpy(&v, row + 4 * (size_t)k, 4);
            return v;
        }
        case T_F16: return rd_f16(row + 2 * (size_t)k);
        case T_Q8_0: {
            const uint8_t* b = row + (size_t)(k >> 5) * 34;
            return rd_f16(b) * (float)(int8_t)b[2 + (k & 31)];
        }
        case T_Q4_K:
        case T_Q5_K: {
            const int bb = type == T_Q4_K ? 144 : 176;
            const uint8_t* b = row + (size_t)(k >> 8) * bb;
            const int i = k & 255, c = i >> 6, l = i & 31, hi = (i >> 5) & 1;
            int mn;
            const int sc = kq_scale(b + 4, 2 * c + hi, &mn);
            const uint8_t* qs = b + (type == T_Q4_K ? 16 : 48);
            int q = hi ? (qs[32 * c + l] >> 4) : (qs[32 * c + l] & 15);
            if (type == T_Q5_K && ((b[16 + l] >> (2 * c + hi)) & 1)) q += 16;
            return rd_f16(b) * sc * q - rd_f16(b + 2) * mn;
        }
        case T_Q6_K: {
            const uint8_t* b = row + (size_t)(k >> 8) * 210;
            const int i = k & 255, h = i >> 7, j = i & 127, qq = j >> 5, l = j & 31;
            const uint8_t lb = b[64 * h + l + ((qq & 1) ? 32 : 0)];
            int q = (qq < 2) ? (lb & 15) : (lb >> 4);
            q |= ((b[128 + 32 * h + l] >> (2 * qq)) & 3) << 4;
            return rd_f16(b + 208) * (float)(int8_t)b[192 + 8 * h + (l >> 4) + 2 * qq] * (q - 32);
        }
        default: return 0.f;
    }
}

// One warp per row; lanes stride over K; up to MT tokens per launch.
__global__ void __launch_bounds__(256) k_gemv_generic(GemvArgs a) {
    const int warp = (blockIdx.x * 256 + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= a.W.rows) return;
    const uint8_t* row = a.W.w + (size_t)warp * a.W.row_bytes;
    float acc[MT];
#pragma unroll
    for (int t = 0; t < MT; t++) acc[t] = 0.f;
    for (int k = lane; k < a.W.K; k += 32) {
        const float w = weight_at(row, a.W.type, k);
#pragma unroll
        for (int t = 0; t < MT; t++)
            if (t < a.m) acc[t] = fmaf(w, a.X[(size_t)t * a.ldx + k], acc[t]);
    }
#pragma unroll
    for (int t = 0; t < MT; t++) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && t < a.m) {
            float* y = a.Y + (size_t)t * a.ldy + warp;
            *y = a.accumulate ? *y + v : v;
        }
    }
}


// ------------------------------------------------------------------------------------------------
// activations -> fragment form (XF); one CTA per token row
// ------------------------------------------------------------------------------------------------
constexpr int PREP_NT = 256;
// rows: X + row * ldx (row < nrows), K floats each (K % 16 == 0, rows 16-byte aligned).
__global__ void __launch_bounds__(PREP_NT) k_prep_x(const float* __restrict__ X, int ldx, int K, uint2* __restrict__ frag,
                                                     float* __restrict__ sum, float* __restrict__ tsc) {
    __shared__ float wmax[PREP_NT / 32];
    __shared__ int sh_e;
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, nseg = K >> 4;
    const float* x = X + (size_t)row * ldx;
    float mx = 0.f;
    for (int i = tid; i < (K >> 2); i += PREP_NT) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) wmax[tid >> 5] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = 0.f;
        for (int w = 0; w < PREP_NT / 32; w++) m = fmaxf(m, wmax[w]);
        int e = 0;
        if (m > 0.f && m < INFINITY) {
            int p;
            frexpf(m, &p);  // m < 2^p: scaled max lands in [2^13, 2^14)
            e = 14 - p;
            e = e > 100 ? 100 : (e < -100 ? -100 : e);
        }
        sh_e = e;
        tsc[row] = pow2f(-e);
    }
    __syncthreads();
    const float sc = pow2f(sh_e);
    for (int i = tid; i < nseg * 4; i += PREP_NT) {  // item = (segment, t): 4 consecutive lanes share a segment
        const int j = i >> 2, t = i & 3;
        const float4 v = *reinterpret_cast<const float4*>(x + 16 * j + 4 * t);
        const float xs[4] = {v.x * sc, v.z * sc, v.y * sc, v.w * sc};  // physical order 0, 2, 1, 3
        uint32_t h16[4], l16[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const __half hh = __float2half_rn(xs[k]);
            h16[k] = __half_as_ushort(hh);
            l16[k] = __half_as_ushort(__float2half_rn(xs[k] - __half2float(hh)));
        }
        uint2* o = frag + ((size_t)row * nseg + j) * 8;
        o[t] = make_uint2(h16[0] | (h16[1] << 16), h16[2] | (h16[3] << 16));
        o[4 + t] = make_uint2(l16[0] | (l16[1] << 16), l16[2] | (l16[3] << 16));
        float s = (v.x + v.y) + (v.z + v.w);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if (t == 0) sum[(size_t)row * nseg + j] = s;
    }
}

// ------------------------------------------------------------------------------------------------
// tile engine: small persistent CTAs (4 warps), one 16-row tile per step, two-slot TMA ring
// ------------------------------------------------------------------------------------------------
constexpr int NTS = 128;
constexpr int NWS = NTS / 32;
constexpr int RING = 2;
constexpr int SETS = 2;  // 4-token column sets per pass (8 tokens)

__host__ __device__ inline size_t al128(size_t x) { return (x + 127) & ~(size_t)127; }

// Row placement of a staged tile. Rows whose byte stride is a multiple of 32 words would put the same
// word of eight consecutive rows in one bank; they are copied one bulk copy per row into a 16-byte
// padded stride. Other strides are copied as one contiguous span (rows start at `lead`).
struct RowLayout {
    int per_row;
    int stride;
};
__host__ __device__ inline RowLayout row_layout(size_t rb, bool base16) {
    if (base16 && rb % 16 == 0 && (rb % 128) % 32 == 0) return {1, (int)rb + 16};
    return {0, (int)rb};
}
__host__ __device__ inline size_t slot_bytes(const RowLayout& L, int nrows) { return al128((size_t)nrows * L.stride + 64); }
__device__ __forceinline__ RowLayout layout_of(const uint8_t* base, size_t rb) {
    return row_layout(rb, (reinterpret_cast<uintptr_t>(base) & 15) == 0);
}

// Copies rows [r0, r1) of a matrix into dst, completion on bar; returns the bytes in flight.
__device__ __forceinline__ uint32_t issue_rows(const RowLayout& L, const uint8_t* base, size_t rb, int r0, int r1,
                                               uint8_t* dst, uint64_t* bar) {
    if (L.per_row) {
        for (int r = r0; r < r1; r++) tma_load_1d(dst + (size_t)(r - r0) * L.stride, base + (size_t)r * rb, (uint32_t)rb, bar);
        return (uint32_t)((r1 - r0) * rb);
    }
    const Span sp = row_span(base, rb, r0, r1);
    tma_load_1d(dst, sp.src, sp.bytes, bar);
    return sp.bytes;
}
__device__ __forceinline__ uint32_t rows_bytes(const RowLayout& L, const uint8_t* base, size_t rb, int r0, int r1) {
    return L.per_row ? (uint32_t)((r1 - r0) * rb) : row_span(base, rb, r0, r1).bytes;
}
__device__ __forceinline__ uint32_t rows_lead(const RowLayout& L, const uint8_t* base, size_t rb, int r0) {
    return L.per_row ? 0u : (uint32_t)((reinterpret_cast<uintptr_t>(base) + (size_t)r0 * rb) & 15);
}

// Scale decode of one 16-row tile: scl [sb][group][16] (rows r and r+8 adjacent), mins [tok][row][sb].
template <int QT>
__device__ __forceinline__ void tile_scales(const uint8_t* rows, int stride, int nsb, const XF& xf, const int* tok,
                                            int m, float* scl, float* mins) {
    constexpr int G = groups_of(QT);
    for (int i = threadIdx.x; i < 16 * nsb; i += blockDim.x) {
        const int r = i / nsb, sb = i - r * nsb;
        decode_scales<QT>(rows + (size_t)r * stride + (size_t)sb * block_bytes(QT), scl + (size_t)sb * G * 16,
                          2 * (r & 7) + (r >> 3), [&](int tk) { return xf.sum + (size_t)tok[tk] * xf.nseg; }, sb, m,
                          mins + (size_t)r * nsb + sb, 16 * nsb);
    }
}

// All MMA tasks (super-block, half) of a staged 16-row tile, part[(task0 + task) * NSET + st][row][tok].
template <int QT, int NSET>
__device__ __forceinline__ void tile_tasks(const uint8_t* rows, int stride, int nsb, const XF& xf, const int* tok, int m,
                                           const float* scl, float* part, int task0) {
    constexpr int G = groups_of(QT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const BPtr<NSET> bp(xf, tok, m);
    for (int k = warp; k < nsb * 2; k += (int)(blockDim.x >> 5)) {
        const int sb = k >> 1, h = k & 1;
        float acc[NSET][4];
#pragma unroll
        for (int st = 0; st < NSET; st++) acc[st][0] = acc[st][1] = acc[st][2] = acc[st][3] = 0.f;
        mma_task<QT, NSET>(rows, stride, sb, h, bp, scl, acc);
#pragma unroll
        for (int st = 0; st < NSET; st++) {
            float* p = part + ((size_t)(task0 + k) * NSET + st) * 64;
            p[g * 4 + t] = acc[st][0] + acc[st][1];
            p[(g + 8) * 4 + t] = acc[st][2] + acc[st][3];
        }
    }
}

// Row r (0..15) of the tile times token tk: MMA partials in super-block order, scaled back by the
// token's power of two, minus the constant terms.
template <int NSET>
__device__ __forceinline__ float tile_value(const float* part, int task0, int r, int nsb, int tk, float tscale,
                                            const float* mins) {
    const int st = tk >> 2, c = tk & 3;
    float s = 0.f, mn = 0.f;
    for (int sb = 0; sb < nsb; sb++) {
        const int task = task0 + 2 * sb;
        s += part[((size_t)task * NSET + st) * 64 + r * 4 + c];
        s += part[((size_t)(task + 1) * NSET + st) * 64 + r * 4 + c];
        mn += mins[((size_t)tk * 16 + r) * nsb + sb];
    }
    return fmaf(s, tscale, -mn);
}

// ------------------------------------------------------------------------------------------------
// dense K-quant GEMV: row groups of 16 strided over the grid
// ------------------------------------------------------------------------------------------------
struct GPlan {
    size_t scl_off, mins_off, part_off, ring_off, slot, total;
};
__host__ __device__ inline GPlan gemv_plan(int qt, int K, size_t rb, int nset) {
    GPlan p;
    const int nsb = K / 256;
    p.scl_off = 128;
    p.mins_off = al128(p.scl_off + (size_t)16 * nsb * groups_of(qt) * 4);
    p.part_off = al128(p.mins_off + (size_t)4 * SETS * 16 * nsb * 4);
    p.ring_off = al128(p.part_off + (size_t)nsb * 2 * nset * 256);
    p.slot = slot_bytes(row_layout(rb, true), 16);
    p.total = p.ring_off + RING * p.slot;
    return p;
}

template <int QT, int NSET>
__global__ void __launch_bounds__(NTS) k_gemv(GemvXArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int K = a.W.K, nsb = K >> 8, m = a.m, tid = threadIdx.x;
    const size_t rb = a.W.row_bytes;
    const GPlan pl = gemv_plan(QT, K, rb, NSET);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    int* tok = reinterpret_cast<int*>(sm + 64);
    float* scl = reinterpret_cast<float*>(sm + pl.scl_off);
    float* mins = reinterpret_cast<float*>(sm + pl.mins_off);
    float* part = reinterpret_cast<float*>(sm + pl.part_off);
    uint8_t* ring = sm + pl.ring_off;
    const RowLayout L = layout_of(a.W.w, rb);
    const int NRG = (a.W.rows + 15) >> 4;
    const int G = gridDim.x;
    if ((int)blockIdx.x >= NRG) return;
    const int nunits = (NRG - 1 - (int)blockIdx.x) / G + 1;
    if (tid == 0) {
        for (int s = 0; s < RING; s++) mbar_init(&bar[s], 1);
        mbar_fence_init();
    }
    if (tid < 8) tok[tid] = tid;
    __syncthreads();
    auto rows_of = [&](int i, int& r0, int& r1) {
        r0 = 16 * ((int)blockIdx.x + i * G);
        r1 = min(a.W.rows, r0 + 16);
    };
    int issued = 0;
    auto issue = [&]() {
        int r0, r1;
        rows_of(issued, r0, r1);
        uint64_t* b = &bar[issued % RING];
        mbar_expect_tx(b, rows_bytes(L, a.W.w, rb, r0, r1));
        issue_rows(L, a.W.w, rb, r0, r1, ring + (size_t)(issued % RING) * pl.slot, b);
        issued++;
    };
    if (tid == 0)
        while (issued < min(RING, nunits)) issue();
    for (int i = 0; i < nunits; i++) {
        int r0, r1;
        rows_of(i, r0, r1);
        const bool ok = mbar_wait_bounded(&bar[i % RING], (uint32_t)(i / RING) & 1u);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                flag(a.status, ST_WAIT_TIMEOUT);
                drain_ring(bar, issued, i, RING);
            }
            return;
        }
        const uint8_t* rows = ring + (size_t)(i % RING) * pl.slot + rows_lead(L, a.W.w, rb, r0);
        tile_scales<QT>(rows, L.stride, nsb, a.xf, tok, m, scl, mins);
        __syncthreads();
        tile_tasks<QT, NSET>(rows, L.stride, nsb, a.xf, tok, m, scl, part, 0);
        __syncthreads();
        for (int j = tid; j < (r1 - r0) * m; j += NTS) {
            const int r = j / m, tk = j - r * m;
            const float v = tile_value<NSET>(part, 0, r, nsb, tk, __ldg(a.xf.tsc + tk), mins);
            float* y = a.Y + (size_t)tk * a.ldy + r0 + r;
            *y = a.accumulate ? *y + v : v;
        }
        __syncthreads();
        if (tid == 0 && issued < nunits) issue();
    }
}
// ------------------------------------------------------------------------------------------------
// routing + permutation (single CTA of 1024 threads)
// ------------------------------------------------------------------------------------------------
struct Cand {
    float r;
    int e;
};
__device__ __forceinline__ bool better(const Cand& a, const Cand& b) {
    return a.r > b.r || (a.r == b.r && a.e < b.e);  // the partial_sort comparator, qwen3moe.cpp:1016
}

__global__ void __launch_bounds__(1024) k_route_permute(MoeArgs a) {
    __shared__ int cnt[MAX_EXPERTS];
    __shared__ int off[MAX_EXPERTS + 1];
    __shared__ unsigned long long mask[MAX_EXPERTS * (ROUTE_TMAX / 64)];
    const int T = a.T, E = a.n_expert, K = a.n_used, tid = threadIdx.x;
    const int W = (T + 63) >> 6;
    for (int i = tid; i < E; i += blockDim.x) cnt[i] = 0;
    for (int i = tid; i < (a.D >> 4); i += blockDim.x) a.rw.group_done[i] = 0;
    for (int i = tid; i < E * W; i += blockDim.x) mask[i] = 0ull;
    __syncthreads();

    // ---- softmax numerators, top-k, renormalisation: one warp per token (qwen3moe.cpp:1012-1022)
    const int warp = tid >> 5, lane = tid & 31, nwarp = blockDim.x >> 5;
    constexpr int PER = MAX_EXPERTS / 32;
    for (int t = warp; t < T; t += nwarp) {
        const float* lg = a.logits + (size_t)t * E;
        float l[PER];
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int e = lane + 32 * i;
            l[i] = e < E ? lg[e] : -INFINITY;
            mx = fmaxf(mx, l[i]);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // r = exp(l - max): the difference in fp32 as on the CPU, the exponential correctly rounded
        float r[PER];
#pragma unroll
        for (int i = 0; i < PER; i++) r[i] = (lane + 32 * i) < E ? (float)exp((double)(l[i] - mx)) : -1.0f;
        unsigned used = 0;
        float tot = 0.f;
        int my_e = -1;
        float my_r = 0.f;
        for (int k = 0; k < K; k++) {
            Cand best{-2.0f, 0x7fffffff};
#pragma unroll
            for (int i = 0; i < PER; i++) {
                const Cand c{r[i], lane + 32 * i};
                if (!((used >> i) & 1u) && (lane + 32 * i) < E && better(c, best)) best = c;
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                Cand other{__shfl_xor_sync(0xffffffffu, best.r, o), __shfl_xor_sync(0xffffffffu, best.e, o)};
                if (better(other, best)) best = other;
            }
            if ((best.e & 31) == lane) used |= 1u << (best.e >> 5);
            tot += best.r;  // rank-order sum, identical on every lane
            if (lane == k) {
                my_e = best.e;
                my_r = best.r;
            }
        }
        if (lane < K) {
            const float w = __fdiv_rn(my_r, tot);
            if (my_e < 0 || my_e >= E) {  // only reachable with NaN logits
                flag(a.status, ST_BAD_INDEX);
                my_e = 0;
            }
            a.rw.ids[(size_t)t * K + lane] = my_e;
            a.rw.wts[(size_t)t * K + lane] = w;
            atomicAdd(&cnt[my_e], 1);
            atomicOr(&mask[my_e * W + (t >> 6)], 1ull << (t & 63));
        }
    }
    __syncthreads();
    // ---- exclusive scan of the counts and the ascending active-expert list
    if (warp == 0) {
        int run = 0, nact = 0;
        for (int base = 0; base < E; base += 32) {
            const int e = base + lane;
            const int c = e < E ? cnt[e] : 0;
            int inc = c, act = c > 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, inc, o), u = __shfl_up_sync(0xffffffffu, act, o);
                if (lane >= o) {
                    inc += v;
                    act += u;
                }
            }
            if (e < E) {
                off[e] = run + inc - c;
                a.rw.offsets[e] = run + inc - c;
                if (c > 0) a.rw.active[1 + nact + act - 1] = e;
            }
            run += __shfl_sync(0xffffffffu, inc, 31);
            nact += __shfl_sync(0xffffffffu, act, 31);
        }
        if (lane == 0) {
            off[E] = run;
            a.rw.offsets[E] = run;
            a.rw.active[0] = nact;
        }
    }
    __syncthreads();
    // ---- stable scatter: slot = offset[e] + number of earlier tokens routed to e
    for (int t = tid; t < T; t += blockDim.x) {
        int slots[32];
        for (int k = 0; k < K; k++) {
            const int e = a.rw.ids[(size_t)t * K + k];
            int rank = __popcll(mask[e * W + (t >> 6)] & ((1ull << (t & 63)) - 1ull));
            for (int w = 0; w < (t >> 6); w++) rank += __popcll(mask[e * W + w]);
            const int s = off[e] + rank;
            a.rw.slot_token[s] = t;
            a.rw.slot_w[s] = a.rw.wts[(size_t)t * K + k];
            int j = k;  // insertion: token_slots ascending == expert ascending
            while (j > 0 && slots[j - 1] > s) {
                slots[j] = slots[j - 1];
                j--;
            }
            slots[j] = s;
        }
        for (int k = 0; k < K; k++) a.rw.token_slots[(size_t)t * K + k] = slots[k];
    }
}


// ------------------------------------------------------------------------------------------------
// gate + up + SiLU*mul: units = (active expert, 16-row group), contiguous unit ranges per CTA
// ------------------------------------------------------------------------------------------------
struct UPlan {
    size_t sclg_off, sclu_off, minsg_off, minsu_off, part_off, ring_off, up_at, slot, total;
};
__host__ __device__ inline UPlan gateup_plan(int qg, int qu, int D, size_t rbg, size_t rbu) {
    UPlan p;
    const int nsb = D / 256;
    p.sclg_off = 256;
    p.sclu_off = al128(p.sclg_off + (size_t)16 * nsb * groups_of(qg) * 4);
    p.minsg_off = al128(p.sclu_off + (size_t)16 * nsb * groups_of(qu) * 4);
    p.minsu_off = al128(p.minsg_off + (size_t)4 * SETS * 16 * nsb * 4);
    p.part_off = al128(p.minsu_off + (size_t)4 * SETS * 16 * nsb * 4);
    p.ring_off = al128(p.part_off + (size_t)2 * nsb * 2 * SETS * 256);
    p.up_at = slot_bytes(row_layout(rbg, true), 16);
    p.slot = p.up_at + slot_bytes(row_layout(rbu, true), 16);
    p.total = p.ring_off + RING * p.slot;
    return p;
}

template <int QG, int QU, int NSET>
__device__ __forceinline__ void gateup_tasks(const uint8_t* grows, int gstride, const uint8_t* urows, int ustride,
                                             int nsb, const XF& xf, const int* tok, int m, const float* sclg,
                                             const float* sclu, float* part) {
    tile_tasks<QG, NSET>(grows, gstride, nsb, xf, tok, m, sclg, part, 0);
    tile_tasks<QU, NSET>(urows, ustride, nsb, xf, tok, m, sclu, part, 2 * nsb);
}

template <int QG, int QU>
__global__ void __launch_bounds__(NTS) k_moe_gateup(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int D = a.D, FF = a.FF, nsb = D >> 8, tid = threadIdx.x;
    const UPlan pl = gateup_plan(QG, QU, D, a.gate_rb, a.up_rb);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    int* tok = reinterpret_cast<int*>(sm + 64);
    float* sclg = reinterpret_cast<float*>(sm + pl.sclg_off);
    float* sclu = reinterpret_cast<float*>(sm + pl.sclu_off);
    float* minsg = reinterpret_cast<float*>(sm + pl.minsg_off);
    float* minsu = reinterpret_cast<float*>(sm + pl.minsu_off);
    float* part = reinterpret_cast<float*>(sm + pl.part_off);
    uint8_t* ring = sm + pl.ring_off;

    const int NRG = FF >> 4;
    const int nact = a.rw.active[0];
    const long long U = (long long)nact * NRG;
    const int u0 = (int)(U * blockIdx.x / gridDim.x), u1 = (int)(U * (blockIdx.x + 1) / gridDim.x);
    if (u0 >= u1) return;
    if (tid == 0) {
        for (int s = 0; s < RING; s++) mbar_init(&bar[s], 1);
        mbar_fence_init();
    }
    __syncthreads();
    int issued = 0;
    auto issue = [&]() {
        const int u = u0 + issued, ai = u / NRG, r0 = 16 * (u - ai * NRG);
        const int e = a.rw.active[1 + ai];
        const RowLayout Lg = layout_of(a.gate[e], a.gate_rb), Lu = layout_of(a.up[e], a.up_rb);
        uint8_t* dst = ring + (size_t)(issued % RING) * pl.slot;
        uint64_t* b = &bar[issued % RING];
        mbar_expect_tx(b, rows_bytes(Lg, a.gate[e], a.gate_rb, r0, r0 + 16) + rows_bytes(Lu, a.up[e], a.up_rb, r0, r0 + 16));
        issue_rows(Lg, a.gate[e], a.gate_rb, r0, r0 + 16, dst, b);
        issue_rows(Lu, a.up[e], a.up_rb, r0, r0 + 16, dst + pl.up_at, b);
        issued++;
    };
    if (tid == 0)
        while (issued < min(RING, u1 - u0)) issue();
    for (int i = 0; i < u1 - u0; i++) {
        const int u = u0 + i, ai = u / NRG, r0 = 16 * (u - ai * NRG);
        const int e = a.rw.active[1 + ai];
        const int s0 = a.rw.offsets[e], me = a.rw.offsets[e + 1] - s0;
        const RowLayout Lg = layout_of(a.gate[e], a.gate_rb), Lu = layout_of(a.up[e], a.up_rb);
        const uint8_t* slot = ring + (size_t)(i % RING) * pl.slot;
        const uint8_t* grows = slot + rows_lead(Lg, a.gate[e], a.gate_rb, r0);
        const uint8_t* urows = slot + pl.up_at + rows_lead(Lu, a.up[e], a.up_rb, r0);
        const bool ok = mbar_wait_bounded(&bar[i % RING], (uint32_t)(i / RING) & 1u);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                flag(a.status, ST_WAIT_TIMEOUT);
                drain_ring(bar, issued, i, RING);
            }
            return;
        }
        for (int c0 = 0; c0 < me; c0 += 4 * SETS) {
            const int mc = min(4 * SETS, me - c0);
            if (tid < mc) tok[tid] = a.rw.slot_token[s0 + c0 + tid];
            __syncthreads();
            tile_scales<QG>(grows, Lg.stride, nsb, a.xf, tok, mc, sclg, minsg);
            tile_scales<QU>(urows, Lu.stride, nsb, a.xf, tok, mc, sclu, minsu);
            __syncthreads();
            if (mc > 4) gateup_tasks<QG, QU, 2>(grows, Lg.stride, urows, Lu.stride, nsb, a.xf, tok, mc, sclg, sclu, part);
            else gateup_tasks<QG, QU, 1>(grows, Lg.stride, urows, Lu.stride, nsb, a.xf, tok, mc, sclg, sclu, part);
            __syncthreads();
            for (int j = tid; j < 16 * mc; j += NTS) {
                const int r = j / mc, tk = j - r * mc;
                const float ts = __ldg(a.xf.tsc + tok[tk]);
                float g, u;
                if (mc > 4) {
                    g = tile_value<2>(part, 0, r, nsb, tk, ts, minsg);
                    u = tile_value<2>(part, 2 * nsb, r, nsb, tk, ts, minsu);
                } else {
                    g = tile_value<1>(part, 0, r, nsb, tk, ts, minsg);
                    u = tile_value<1>(part, 2 * nsb, r, nsb, tk, ts, minsu);
                }
                a.h[(size_t)(s0 + c0 + tk) * FF + r0 + r] = silu_mul(g, u);
            }
            __syncthreads();
        }
        if (tid == 0 && issued < u1 - u0) issue();
    }
}

// ------------------------------------------------------------------------------------------------
// down projection: units = (16-row group of D, active expert), contiguous ranges per CTA, so a CTA
// mostly walks the experts of one row group. Expert outputs go to y[slot][D]; the CTA that completes a
// row group (a per-group counter reaches the number of active experts) adds each token's expert
// outputs in ascending expert order, weighted, to the residual (qwen3moe.cpp:1024-1069).
// ------------------------------------------------------------------------------------------------
struct DPlan {
    size_t scl_off, mins_off, part_off, ring_off, slot, total;
};
__host__ __device__ inline DPlan down_plan(int qd, int FF, size_t rb) {
    DPlan p;
    const int nsb = FF / 256;
    p.scl_off = 256;
    p.mins_off = al128(p.scl_off + (size_t)16 * nsb * groups_of(qd) * 4);
    p.part_off = al128(p.mins_off + (size_t)4 * SETS * 16 * nsb * 4);
    p.ring_off = al128(p.part_off + (size_t)nsb * 2 * SETS * 256);
    p.slot = slot_bytes(row_layout(rb, true), 16);
    p.total = p.ring_off + RING * p.slot;
    return p;
}

template <int QD>
__global__ void __launch_bounds__(NTS) k_moe_down(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ int s_last;
    const int D = a.D, FF = a.FF, nsb = FF >> 8, T = a.T, K = a.n_used, tid = threadIdx.x;
    const size_t rb = a.down_rb;
    const DPlan pl = down_plan(QD, FF, rb);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    int* tok = reinterpret_cast<int*>(sm + 64);
    float* scl = reinterpret_cast<float*>(sm + pl.scl_off);
    float* mins = reinterpret_cast<float*>(sm + pl.mins_off);
    float* part = reinterpret_cast<float*>(sm + pl.part_off);
    uint8_t* ring = sm + pl.ring_off;

    const int NRG = D >> 4;
    const int nact = a.rw.active[0];
    const int* act = a.rw.active + 1;
    const int* off = a.rw.offsets;
    const long long U = (long long)NRG * nact;
    const int u0 = (int)(U * blockIdx.x / gridDim.x), u1 = (int)(U * (blockIdx.x + 1) / gridDim.x);
    if (u0 >= u1) return;
    if (tid == 0) {
        for (int s = 0; s < RING; s++) mbar_init(&bar[s], 1);
        mbar_fence_init();
    }
    __syncthreads();
    int issued = 0;
    auto issue = [&]() {
        const int u = u0 + issued, rg = u / nact, ai = u - rg * nact;
        const uint8_t* w = a.down[act[ai]];
        const RowLayout L = layout_of(w, rb);
        uint64_t* b = &bar[issued % RING];
        mbar_expect_tx(b, rows_bytes(L, w, rb, 16 * rg, 16 * rg + 16));
        issue_rows(L, w, rb, 16 * rg, 16 * rg + 16, ring + (size_t)(issued % RING) * pl.slot, b);
        issued++;
    };
    if (tid == 0)
        while (issued < min(RING, u1 - u0)) issue();
    int done_in_group = 0;
    for (int i = 0; i < u1 - u0; i++) {
        const int u = u0 + i, rg = u / nact, ai = u - rg * nact, r0 = 16 * rg;
        const int e = act[ai];
        const int s0 = off[e], me = off[e + 1] - s0;
        const uint8_t* w = a.down[e];
        const RowLayout L = layout_of(w, rb);
        const uint8_t* rows = ring + (size_t)(i % RING) * pl.slot + rows_lead(L, w, rb, r0);
        const bool ok = mbar_wait_bounded(&bar[i % RING], (uint32_t)(i / RING) & 1u);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                flag(a.status, ST_WAIT_TIMEOUT);
                drain_ring(bar, issued, i, RING);
            }
            return;
        }
        for (int c0 = 0; c0 < me; c0 += 4 * SETS) {
            const int mc = min(4 * SETS, me - c0);
            if (tid < mc) tok[tid] = s0 + c0 + tid;  // xf rows of the down input are slots
            __syncthreads();
            tile_scales<QD>(rows, L.stride, nsb, a.hf, tok, mc, scl, mins);
            __syncthreads();
            if (mc > 4) tile_tasks<QD, 2>(rows, L.stride, nsb, a.hf, tok, mc, scl, part, 0);
            else tile_tasks<QD, 1>(rows, L.stride, nsb, a.hf, tok, mc, scl, part, 0);
            __syncthreads();
            for (int j = tid; j < 16 * mc; j += NTS) {
                const int r = j / mc, tk = j - r * mc;
                const float ts = __ldg(a.hf.tsc + tok[tk]);
                const float v = mc > 4 ? tile_value<2>(part, 0, r, nsb, tk, ts, mins) : tile_value<1>(part, 0, r, nsb, tk, ts, mins);
                a.y[(size_t)(s0 + c0 + tk) * D + r0 + r] = v;
            }
            __syncthreads();
        }
        if (tid == 0 && issued < u1 - u0) issue();
        done_in_group++;
        const bool group_end = (i + 1 == u1 - u0) || ((u + 1) / nact != rg);
        if (group_end) {
            // publish this CTA's expert outputs of the group; the CTA that completes it combines
            __threadfence();
            __syncthreads();
            if (tid == 0) s_last = (atomicAdd(&a.rw.group_done[rg], done_in_group) + done_in_group == nact);
            __syncthreads();
            done_in_group = 0;
            if (s_last) {
                __threadfence();
                for (int j = tid; j < T * 16; j += NTS) {
                    const int t = j >> 4, r = j & 15;
                    const int* ts = a.rw.token_slots + (size_t)t * K;
                    float acc = 0.f;
                    for (int k = 0; k < K; k++) {
                        const int s = ts[k];
                        acc = fmaf(a.rw.slot_w[s], __ldcg(a.y + (size_t)s * D + r0 + r), acc);
                    }
                    a.x[(size_t)t * D + r0 + r] += acc;
                }
                if (tid == 0) a.rw.group_done[rg] = 0;  // ready for the next call
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------
// launchers
// ------------------------------------------------------------------------------------------------
int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// Persistent grid of a kernel: SMs x resident CTAs at this shared-memory size.
template <typename Kern>
static int persistent_grid(Kern k, size_t smem) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int per = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k, NTS, smem) != cudaSuccess || per < 1) per = 1;
    return sm_count() * per;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
constexpr size_t SMEM_CAP = 227 * 1024;

bool gemv_mma_ok(const QMat& W) {
    return is_kquant(W.type) && W.K % 256 == 0 && W.row_bytes == (size_t)(W.K / 256) * block_bytes(W.type) &&
           gemv_plan(W.type, W.K, W.row_bytes, SETS).total <= SMEM_CAP;
}

size_t xf_bytes(int rows, int K) { return (size_t)rows * K * 4 + (size_t)rows * (K / 16) * 4 + (size_t)rows * 4 + 256; }
XF xf_carve(void* base, int rows, int K) {
    uint8_t* p = static_cast<uint8_t*>(base);
    XF x;
    x.frag = reinterpret_cast<const uint2*>(p);
    x.sum = reinterpret_cast<const float*>(p + (size_t)rows * K * 4);
    x.tsc = reinterpret_cast<const float*>(p + (size_t)rows * K * 4 + (size_t)rows * (K / 16) * 4);
    x.nseg = K / 16;
    return x;
}

cudaError_t launch_prep_x(const float* X, int ldx, int rows, int K, const XF& out, cudaStream_t st) {
    if (rows < 1 || K % 16 || ldx % 4 || !aligned16(X)) return cudaErrorInvalidValue;
    k_prep_x<<<rows, PREP_NT, 0, st>>>(X, ldx, K, const_cast<uint2*>(out.frag), const_cast<float*>(out.sum),
                                       const_cast<float*>(out.tsc));
    return cudaGetLastError();
}

template <int QT, int NSET>
static void gemv_go(const GemvXArgs& a, cudaStream_t st) {
    const GPlan pl = gemv_plan(QT, a.W.K, a.W.row_bytes, NSET);
    const int nrg = (a.W.rows + 15) / 16;
    static int grid = 0;
    static size_t grid_smem = 0;
    if (grid_smem != pl.total) {
        grid = persistent_grid(k_gemv<QT, NSET>, pl.total);
        grid_smem = pl.total;
    }
    k_gemv<QT, NSET><<<std::min(grid, nrg), NTS, pl.total, st>>>(a);
}

cudaError_t launch_gemv_xf(const GemvXArgs& a, cudaStream_t st) {
    if (a.m < 1 || a.m > 4 * SETS || !gemv_mma_ok(a.W)) return cudaErrorInvalidValue;
    const bool two = a.m > 4;
    switch (a.W.type) {
        case T_Q4_K: two ? gemv_go<T_Q4_K, 2>(a, st) : gemv_go<T_Q4_K, 1>(a, st); break;
        case T_Q5_K: two ? gemv_go<T_Q5_K, 2>(a, st) : gemv_go<T_Q5_K, 1>(a, st); break;
        default: two ? gemv_go<T_Q6_K, 2>(a, st) : gemv_go<T_Q6_K, 1>(a, st); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t st) {
    if (a.m < 1 || a.m > MT) return cudaErrorInvalidValue;
    k_gemv_generic<<<(a.W.rows * 32 + 255) / 256, 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_route_permute(const MoeArgs& a, cudaStream_t st) {
    if (a.T < 1 || a.T > ROUTE_TMAX || a.n_expert > MAX_EXPERTS || a.n_used > 32 || a.n_used > a.n_expert)
        return cudaErrorInvalidValue;
    k_route_permute<<<1, 1024, 0, st>>>(a);
    return cudaGetLastError();
}

template <int QG, int QU>
static cudaError_t gateup_as(const MoeArgs& a, cudaStream_t st) {
    const UPlan pl = gateup_plan(QG, QU, a.D, a.gate_rb, a.up_rb);
    if (pl.total > SMEM_CAP) return cudaErrorInvalidValue;
    static int grid = 0;
    static size_t grid_smem = 0;
    if (grid_smem != pl.total) {
        grid = persistent_grid(k_moe_gateup<QG, QU>, pl.total);
        grid_smem = pl.total;
    }
    k_moe_gateup<QG, QU><<<grid, NTS, pl.total, st>>>(a);
    return cudaGetLastError();
}
template <int QG>
static cudaError_t gateup_g(const MoeArgs& a, cudaStream_t st) {
    switch (a.up_type) {
        case T_Q4_K: return gateup_as<QG, T_Q4_K>(a, st);
        case T_Q5_K: return gateup_as<QG, T_Q5_K>(a, st);
        case T_Q6_K: return gateup_as<QG, T_Q6_K>(a, st);
        default: return cudaErrorInvalidValue;
    }
}
cudaError_t launch_moe_gateup(const MoeArgs& a, cudaStream_t st) {
    if (a.D % 256 || a.FF % 16) return cudaErrorInvalidValue;
    switch (a.gate_type) {
        case T_Q4_K: return gateup_g<T_Q4_K>(a, st);
        case T_Q5_K: return gateup_g<T_Q5_K>(a, st);
        case T_Q6_K: return gateup_g<T_Q6_K>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

template <int QD>
static cudaError_t down_as(const MoeArgs& a, cudaStream_t st) {
    const DPlan pl = down_plan(QD, a.FF, a.down_rb);
    if (pl.total > SMEM_CAP) return cudaErrorInvalidValue;
    static int grid = 0;
    static size_t grid_smem = 0;
    if (grid_smem != pl.total) {
        grid = persistent_grid(k_moe_down<QD>, pl.total);
        grid_smem = pl.total;
    }
    k_moe_down<QD><<<grid, NTS, pl.total, st>>>(a);
    return cudaGetLastError();
}
cudaError_t launch_moe_down(const MoeArgs& a, cudaStream_t st) {
    if (a.FF % 256 || a.D % 16 || a.T > DOWN_TMAX) return cudaErrorInvalidValue;
    switch (a.down_type) {
        case T_Q4_K: return down_as<T_Q4_K>(a, st);
        case T_Q5_K: return down_as<T_Q5_K>(a, st);
        case T_Q6_K: return down_as<T_Q6_K>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_f32_gemv(const float* W, int K, int rows, const float* X, int ldx, int m, float* Y, int ldy,
                            cudaStream_t st) {  // F32 rows take the per-row kernel, MT tokens per pass
    for (int t0 = 0; t0 < m; t0 += MT) {
        GemvArgs a{};
        a.W = QMat{reinterpret_cast<const uint8_t*>(W), T_F32, K, rows, (size_t)K * 4};
        a.X = X + (size_t)t0 * ldx;
        a.ldx = ldx;
        a.m = m - t0 < MT ? m - t0 : MT;
        a.Y = Y + (size_t)t0 * ldy;
        a.ldy = ldy;
        cudaError_t e = launch_gemv(a, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace eb
