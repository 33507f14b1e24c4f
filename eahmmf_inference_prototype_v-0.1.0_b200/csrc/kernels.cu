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
#include <mutex>
#include <unordered_map>

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
__device__ __forceinline__ int digit(float v) { return (int)fminf(127.f, fmaxf(-127.f, rintf(v))); }
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) | ((uint32_t)(d & 255) << 24);
}
// rows: X + row * ldx (row < nrows), K floats each (K % 32 == 0, rows 16-byte aligned). Writes each row
// as three int8 digits of base 254 of x / s, s = max|x| / 127, in MMA B-fragment order, plus the
// per-16 sums of x and s.
__global__ void __launch_bounds__(PREP_NT) k_prep_x(const float* __restrict__ X, int ldx, int K, uint2* __restrict__ frag,
                                                     float* __restrict__ sum, float* __restrict__ tsc) {
    __shared__ float wmax[PREP_NT / 32];
    __shared__ float sh_inv;
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, nblk = K >> 5;
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
        if (!(m > 0.f) || m == INFINITY) m = 127.f;  // all-zero (or non-finite) rows: any scale works
        tsc[row] = m / 127.f;
        sh_inv = 127.f / m;
    }
    __syncthreads();
    const float inv = sh_inv;
    for (int i = tid; i < nblk * 4; i += PREP_NT) {  // item = (32-k block j, t): 4 consecutive lanes share a block
        const int j = i >> 2, t = i & 3;
        const float4 u = *reinterpret_cast<const float4*>(x + 32 * j + 4 * t);
        const float4 w = *reinterpret_cast<const float4*>(x + 32 * j + 16 + 4 * t);
        const float xv[8] = {u.x, u.y, u.z, u.w, w.x, w.y, w.z, w.w};
        int dg[3][8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float v = xv[k] * inv;
            const int a0 = digit(v);
            const float r1 = (v - (float)a0) * DIGIT;
            const int a1 = digit(r1);
            const int a2 = digit((r1 - (float)a1) * DIGIT);
            dg[0][k] = a0;
            dg[1][k] = a1;
            dg[2][k] = a2;
        }
        uint2* o = frag + ((size_t)row * nblk + j) * 12 + t;
#pragma unroll
        for (int p = 0; p < 3; p++)
            o[p * 4] = make_uint2(pack4(dg[p][0], dg[p][1], dg[p][2], dg[p][3]), pack4(dg[p][4], dg[p][5], dg[p][6], dg[p][7]));
        float s0 = (u.x + u.y) + (u.z + u.w), s1 = (w.x + w.y) + (w.z + w.w);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
        if (t == 0) {
            sum[(size_t)row * (K >> 4) + 2 * j] = s0;
            sum[(size_t)row * (K >> 4) + 2 * j + 1] = s1;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// tile engine: small persistent CTAs (4 warps), one 16-row tile per step, two-slot TMA ring
// ------------------------------------------------------------------------------------------------
constexpr int SETS = 2;  // MMA column sets per pass of the dense GEMV (TOK_PER_SET tokens each)
constexpr int TPASS = SETS * TOK_PER_SET;  // tokens per pass of the dense GEMV
constexpr int MPASS = TOK_PER_SET;         // tokens per pass of the expert kernels (one column set)

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

// Bulk-copies the fragment rows and per-16 sums of m tokens into shared memory (sfrag: m x K*3 bytes,
// ssum: m x K/16 floats). rows(i) gives token i's xf row; consecutive rows are merged into one copy.
// Returns the bytes in flight on bar.
template <typename Rows>
__device__ __forceinline__ uint32_t issue_xf(const XF& xf, Rows rows, int m, int K, uint8_t* sfrag, float* ssum,
                                             uint64_t* bar) {
    const uint32_t fb = (uint32_t)K * 3, sbytes = (uint32_t)K / 4;
    uint32_t total = 0;
    for (int i = 0; i < m;) {
        int n = 1;
        while (i + n < m && rows(i + n) == rows(i) + n) n++;
        const size_t r = (size_t)rows(i);
        tma_load_1d(sfrag + (size_t)i * fb, reinterpret_cast<const uint8_t*>(xf.frag) + r * fb, n * fb, bar);
        tma_load_1d(ssum + (size_t)i * (K >> 4), xf.sum + r * (K >> 4), n * sbytes, bar);
        total += n * (fb + sbytes);
        i += n;
    }
    return total;
}
__device__ __forceinline__ uint32_t xf_bytes_of(int m, int K) { return (uint32_t)m * ((uint32_t)K * 3 + (uint32_t)K / 4); }

// All MMA tasks (super-block, half) of a staged 16-row tile:
//   part[((task0 + task) * NSET + st) * 128 + row * 8 + column] = d * (int32 digit sums)
//   mpart[(task0 + task) * 64 + row * 4 + token]                = group-minimum term
template <int QT, int NSET>
__device__ __forceinline__ void tile_tasks(const uint8_t* rows, int stride, int nsb, const uint2* sfrag,
                                           const float* ssum, int m, float* part, float* mpart, int task0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const BPtr<NSET> bp(sfrag, nsb * 8, m);
    for (int k = warp; k < nsb * 2; k += (int)(blockDim.x >> 5)) {
        float o[NSET][4], mn[2];
        mma_task<QT, NSET>(rows, stride, k >> 1, k & 1, bp, ssum, nsb * 16, m, o, mn);
#pragma unroll
        for (int st = 0; st < NSET; st++) {
            float* p = part + ((size_t)(task0 + k) * NSET + st) * 128;
            *reinterpret_cast<float2*>(p + g * 8 + 2 * t) = make_float2(o[st][0], o[st][1]);
            *reinterpret_cast<float2*>(p + (g + 8) * 8 + 2 * t) = make_float2(o[st][2], o[st][3]);
        }
        float* q = mpart + (size_t)(task0 + k) * 64;
        q[g * 4 + t] = mn[0];
        q[(g + 8) * 4 + t] = mn[1];
    }
}

// Row r (0..15) of the tile times token tk: the three digit columns summed over the tasks in
// super-block order and recombined, scaled by the token's s, minus the group-minimum terms.
template <int NSET>
__device__ __forceinline__ float tile_value(const float* part, const float* mpart, int task0, int r, int nsb, int tk,
                                            float tscale) {
    const int st = tk / TOK_PER_SET, c = 3 * (tk % TOK_PER_SET);
    float a = 0.f, b = 0.f, e = 0.f, mn = 0.f;
    for (int k = 0; k < 2 * nsb; k++) {
        const float* p = part + ((size_t)(task0 + k) * NSET + st) * 128 + r * 8 + c;
        a += p[0];
        b += p[1];
        e += p[2];
        mn += mpart[(size_t)(task0 + k) * 64 + r * 4 + tk];
    }
    return fmaf(fmaf(fmaf(e, 1.0f / DIGIT, b), 1.0f / DIGIT, a), tscale, -mn);
}

// ------------------------------------------------------------------------------------------------
// dense K-quant GEMV: row groups of 16 strided over the grid
// ------------------------------------------------------------------------------------------------
constexpr int NTU = 256;  // threads of the one-unit-per-CTA kernels (8 warps)
struct GPlan {
    size_t sfrag_off, ssum_off, part_off, mpart_off, slot_off, total;
};
// Shared memory of a one-tile unit with m staged tokens and ntask MMA tasks of nset column sets.
__host__ __device__ inline GPlan unit_plan(int K, int m, int ntask, int nset, size_t slot_bytes_total) {
    GPlan p;
    p.sfrag_off = 128;
    p.ssum_off = al128(p.sfrag_off + (size_t)m * K * 3);
    p.part_off = al128(p.ssum_off + (size_t)m * (K / 16) * 4);
    p.mpart_off = al128(p.part_off + (size_t)ntask * nset * 512);
    p.slot_off = al128(p.mpart_off + (size_t)ntask * 256);
    p.total = p.slot_off + slot_bytes_total;
    return p;
}
__host__ __device__ inline GPlan gemv_plan(int qt, int K, size_t rb, int nset, int m) {
    (void)qt;
    return unit_plan(K, m, 2 * (K / 256), nset, slot_bytes(row_layout(rb, true), 16));
}

template <int QT, int NSET>
__global__ void __launch_bounds__(NTU) k_gemv(GemvXArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int K = a.W.K, nsb = K >> 8, m = a.m, tid = threadIdx.x;
    const size_t rb = a.W.row_bytes;
    const GPlan pl = gemv_plan(QT, K, rb, NSET, m);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    uint8_t* sfrag = sm + pl.sfrag_off;
    float* ssum = reinterpret_cast<float*>(sm + pl.ssum_off);
    float* part = reinterpret_cast<float*>(sm + pl.part_off);
    float* mpart = reinterpret_cast<float*>(sm + pl.mpart_off);
    uint8_t* slot = sm + pl.slot_off;
    const RowLayout L = layout_of(a.W.w, rb);
    const int r0 = 16 * (int)blockIdx.x, r1 = min(a.W.rows, r0 + 16);
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_fence_init();
        mbar_expect_tx(&bar[0], rows_bytes(L, a.W.w, rb, r0, r1) + xf_bytes_of(m, K));
        issue_rows(L, a.W.w, rb, r0, r1, slot, &bar[0]);
        issue_xf(a.xf, [](int i) { return i; }, m, K, sfrag, ssum, &bar[0]);
    }
    __syncthreads();
    if (__syncthreads_or(!mbar_wait_bounded(&bar[0], 0u))) {
        if (tid == 0) {
            flag(a.status, ST_WAIT_TIMEOUT);
            drain_ring(bar, 1, 0, 1);
        }
        return;
    }
    const uint8_t* rows = slot + rows_lead(L, a.W.w, rb, r0);
    tile_tasks<QT, NSET>(rows, L.stride, nsb, reinterpret_cast<const uint2*>(sfrag), ssum, m, part, mpart, 0);
    __syncthreads();
    for (int j = tid; j < (r1 - r0) * m; j += blockDim.x) {
        const int r = j / m, tk = j - r * m;
        const float v = tile_value<NSET>(part, mpart, 0, r, nsb, tk, __ldg(a.xf.tsc + tk));
        float* y = a.Y + (size_t)tk * a.ldy + r0 + r;
        *y = a.accumulate ? *y + v : v;
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
    const int per = (E + 31) >> 5;  // entries per lane
    for (int t = warp; t < T; t += nwarp) {
        const float* lg = a.logits + (size_t)t * E;
        float l[PER];
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int e = lane + 32 * i;
            l[i] = (i < per && e < E) ? lg[e] : -INFINITY;
            mx = fmaxf(mx, l[i]);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // r = exp(l - max): the difference in fp32 as on the CPU, the exponential correctly rounded
        float r[PER];
#pragma unroll
        for (int i = 0; i < PER; i++)
            r[i] = (i < per && (lane + 32 * i) < E) ? (float)exp((double)(l[i] - mx)) : -1.0f;
        unsigned used = 0;
        float tot = 0.f;
        int my_e = -1;
        float my_r = 0.f;
        for (int k = 0; k < K; k++) {
            Cand best{-2.0f, 0x7fffffff};
#pragma unroll
            for (int i = 0; i < PER; i++) {
                if (i >= per) break;
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
    GPlan u;
    size_t up_at;
};
__host__ __device__ inline UPlan gateup_plan(int qg, int qu, int D, size_t rbg, size_t rbu) {
    (void)qg;
    (void)qu;
    UPlan p;
    p.up_at = slot_bytes(row_layout(rbg, true), 16);
    p.u = unit_plan(D, MPASS, 4 * (D / 256), 1, p.up_at + slot_bytes(row_layout(rbu, true), 16));
    return p;
}

template <int QG, int QU, int NSET>
__device__ __forceinline__ void gateup_tasks(const uint8_t* grows, int gstride, const uint8_t* urows, int ustride,
                                             int nsb, const uint2* sfrag, const float* ssum, int m, float* part,
                                             float* mpart) {
    tile_tasks<QG, NSET>(grows, gstride, nsb, sfrag, ssum, m, part, mpart, 0);
    tile_tasks<QU, NSET>(urows, ustride, nsb, sfrag, ssum, m, part, mpart, 2 * nsb);
}

template <int QG, int QU>
__global__ void __launch_bounds__(NTU) k_moe_gateup(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int D = a.D, FF = a.FF, nsb = D >> 8, tid = threadIdx.x;
    const UPlan pl = gateup_plan(QG, QU, D, a.gate_rb, a.up_rb);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    int* tok = reinterpret_cast<int*>(sm + 64);
    uint8_t* sfrag = sm + pl.u.sfrag_off;
    float* ssum = reinterpret_cast<float*>(sm + pl.u.ssum_off);
    float* part = reinterpret_cast<float*>(sm + pl.u.part_off);
    float* mpart = reinterpret_cast<float*>(sm + pl.u.mpart_off);
    uint8_t* slot = sm + pl.u.slot_off;

    const int NRG = FF >> 4;
    const int nact = a.rw.active[0];
    const int ai = (int)blockIdx.x / NRG, r0 = 16 * ((int)blockIdx.x - ai * NRG);
    if (ai >= nact) return;  // the grid covers the largest possible number of active experts
    const int e = a.rw.active[1 + ai];
    const int s0 = a.rw.offsets[e], me = a.rw.offsets[e + 1] - s0;
    const RowLayout Lg = layout_of(a.gate[e], a.gate_rb), Lu = layout_of(a.up[e], a.up_rb);
    const uint8_t* grows = slot + rows_lead(Lg, a.gate[e], a.gate_rb, r0);
    const uint8_t* urows = slot + pl.up_at + rows_lead(Lu, a.up[e], a.up_rb, r0);
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_fence_init();
    }
    for (int c0 = 0, pass = 0; c0 < me; c0 += MPASS, pass++) {
        const int mc = min(MPASS, me - c0);
        if (tid < mc) tok[tid] = a.rw.slot_token[s0 + c0 + tid];
        __syncthreads();  // tok visible; the previous pass is done with the staged activations
        if (tid == 0) {
            uint32_t bytes = xf_bytes_of(mc, D);
            if (pass == 0) bytes += rows_bytes(Lg, a.gate[e], a.gate_rb, r0, r0 + 16) + rows_bytes(Lu, a.up[e], a.up_rb, r0, r0 + 16);
            mbar_expect_tx(&bar[0], bytes);
            if (pass == 0) {
                issue_rows(Lg, a.gate[e], a.gate_rb, r0, r0 + 16, slot, &bar[0]);
                issue_rows(Lu, a.up[e], a.up_rb, r0, r0 + 16, slot + pl.up_at, &bar[0]);
            }
            issue_xf(a.xf, [&](int i) { return tok[i]; }, mc, D, sfrag, ssum, &bar[0]);
        }
        if (__syncthreads_or(!mbar_wait_bounded(&bar[0], (uint32_t)pass & 1u))) {
            if (tid == 0) {
                flag(a.status, ST_WAIT_TIMEOUT);
                drain_ring(bar, pass + 1, pass, 1);
            }
            return;
        }
        gateup_tasks<QG, QU, 1>(grows, Lg.stride, urows, Lu.stride, nsb, reinterpret_cast<const uint2*>(sfrag), ssum, mc,
                                part, mpart);
        __syncthreads();
        for (int j = tid; j < 16 * mc; j += blockDim.x) {
            const int r = j / mc, tk = j - r * mc;
            const float ts = __ldg(a.xf.tsc + tok[tk]);
            const float g = tile_value<1>(part, mpart, 0, r, nsb, tk, ts);
            const float u = tile_value<1>(part, mpart, 2 * nsb, r, nsb, tk, ts);
            a.h[(size_t)(s0 + c0 + tk) * FF + r0 + r] = silu_mul(g, u);
        }
        __syncthreads();  // tok and the staged activations are rewritten by the next pass
    }
}

// ------------------------------------------------------------------------------------------------
// down projection: units = (16-row group of D, active expert), contiguous ranges per CTA, so a CTA
// mostly walks the experts of one row group. Expert outputs go to y[slot][D]; the CTA that completes a
// row group (a per-group counter reaches the number of active experts) adds each token's expert
// outputs in ascending expert order, weighted, to the residual (qwen3moe.cpp:1024-1069).
// ------------------------------------------------------------------------------------------------
__host__ __device__ inline GPlan down_plan(int qd, int FF, size_t rb) {
    (void)qd;
    return unit_plan(FF, MPASS, 2 * (FF / 256), 1, slot_bytes(row_layout(rb, true), 16));
}

template <int QD>
__global__ void __launch_bounds__(NTU) k_moe_down(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ int s_last;
    const int D = a.D, FF = a.FF, nsb = FF >> 8, T = a.T, K = a.n_used, tid = threadIdx.x;
    const size_t rb = a.down_rb;
    const GPlan pl = down_plan(QD, FF, rb);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    uint8_t* sfrag = sm + pl.sfrag_off;
    float* ssum = reinterpret_cast<float*>(sm + pl.ssum_off);
    float* part = reinterpret_cast<float*>(sm + pl.part_off);
    float* mpart = reinterpret_cast<float*>(sm + pl.mpart_off);
    uint8_t* slot = sm + pl.slot_off;

    const int nact = a.rw.active[0];
    const int rg = (int)blockIdx.x, ai = (int)blockIdx.y, r0 = 16 * rg;
    if (ai >= nact) return;  // grid.y covers the largest possible number of active experts
    const int e = a.rw.active[1 + ai];
    const int s0 = a.rw.offsets[e], me = a.rw.offsets[e + 1] - s0;
    const uint8_t* w = a.down[e];
    const RowLayout L = layout_of(w, rb);
    const uint8_t* rows = slot + rows_lead(L, w, rb, r0);
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_fence_init();
    }
    for (int c0 = 0, pass = 0; c0 < me; c0 += MPASS, pass++) {
        const int mc = min(MPASS, me - c0);
        __syncthreads();  // the previous pass is done with the staged activations
        if (tid == 0) {
            uint32_t bytes = xf_bytes_of(mc, FF);
            if (pass == 0) bytes += rows_bytes(L, w, rb, r0, r0 + 16);
            mbar_expect_tx(&bar[0], bytes);
            if (pass == 0) issue_rows(L, w, rb, r0, r0 + 16, slot, &bar[0]);
            issue_xf(a.hf, [&](int i) { return s0 + c0 + i; }, mc, FF, sfrag, ssum, &bar[0]);  // xf rows = slots
        }
        if (__syncthreads_or(!mbar_wait_bounded(&bar[0], (uint32_t)pass & 1u))) {
            if (tid == 0) {
                flag(a.status, ST_WAIT_TIMEOUT);
                drain_ring(bar, pass + 1, pass, 1);
            }
            return;
        }
        tile_tasks<QD, 1>(rows, L.stride, nsb, reinterpret_cast<const uint2*>(sfrag), ssum, mc, part, mpart, 0);
        __syncthreads();
        for (int j = tid; j < 16 * mc; j += blockDim.x) {
            const int r = j / mc, tk = j - r * mc;
            const float ts = __ldg(a.hf.tsc + s0 + c0 + tk);
            const float v = tile_value<1>(part, mpart, 0, r, nsb, tk, ts);
            a.y[(size_t)(s0 + c0 + tk) * D + r0 + r] = v;
        }
    }
    // publish this expert's rows of the group; the CTA that completes the group combines it
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.rw.group_done[rg], 1) + 1 == nact);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int j = tid; j < T * 16; j += blockDim.x) {
        const int t = j >> 4, r = j & 15;
        const int* ts = a.rw.token_slots + (size_t)t * K;
        float acc = 0.f;
        for (int k = 0; k < K; k++) {  // ascending slots = ascending experts (qwen3moe.cpp:1025)
            const int s = ts[k];
            acc = fmaf(a.rw.slot_w[s], __ldcg(a.y + (size_t)s * D + r0 + r), acc);
        }
        a.x[(size_t)t * D + r0 + r] += acc;
    }
    if (tid == 0) a.rw.group_done[rg] = 0;  // ready for the next call
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

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
constexpr size_t SMEM_CAP = 227 * 1024;

bool gemv_mma_ok(const QMat& W) {
    return is_kquant(W.type) && W.K % 256 == 0 && W.row_bytes == (size_t)(W.K / 256) * block_bytes(W.type) &&
           gemv_plan(W.type, W.K, W.row_bytes, SETS, TPASS).total <= SMEM_CAP;
}

XF xf_carve(void* base, int rows, int K) {
    uint8_t* p = static_cast<uint8_t*>(base);
    XF x;
    x.frag = reinterpret_cast<const uint2*>(p);
    x.sum = reinterpret_cast<const float*>(p + (size_t)rows * K * 3);
    x.tsc = reinterpret_cast<const float*>(p + (size_t)rows * K * 3 + (size_t)rows * (K / 16) * 4);
    x.nseg = K / 16;
    return x;
}

cudaError_t launch_prep_x(const float* X, int ldx, int rows, int K, const XF& out, cudaStream_t st) {
    if (rows < 1 || K % 32 || ldx % 4 || !aligned16(X)) return cudaErrorInvalidValue;
    k_prep_x<<<rows, PREP_NT, 0, st>>>(X, ldx, K, const_cast<uint2*>(out.frag), const_cast<float*>(out.sum),
                                       const_cast<float*>(out.tsc));
    return cudaGetLastError();
}

// Raises a kernel's dynamic shared-memory limit once per kernel and size (host-side bookkeeping only).
template <typename Kern>
static void smem_attr(Kern k, size_t smem) {
    static std::mutex mu;
    static std::unordered_map<const void*, size_t> done;
    std::lock_guard<std::mutex> g(mu);
    size_t& cur = done[reinterpret_cast<const void*>(k)];
    if (cur < smem) {
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cur = smem;
    }
}

template <int QT, int NSET>
static void gemv_go(const GemvXArgs& a, cudaStream_t st) {
    const GPlan pl = gemv_plan(QT, a.W.K, a.W.row_bytes, NSET, a.m);
    smem_attr(k_gemv<QT, NSET>, pl.total);
    k_gemv<QT, NSET><<<(a.W.rows + 15) / 16, NTU, pl.total, st>>>(a);
}

cudaError_t launch_gemv_xf(const GemvXArgs& a, cudaStream_t st) {
    if (a.m < 1 || a.m > TPASS || !gemv_mma_ok(a.W)) return cudaErrorInvalidValue;
    const bool two = a.m > TOK_PER_SET;
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
    const int threads = a.T <= 4 ? 128 : (a.T <= 32 ? 512 : 1024);  // one warp per token, at most 32
    k_route_permute<<<1, threads, 0, st>>>(a);
    return cudaGetLastError();
}

template <int QG, int QU>
static cudaError_t gateup_as(const MoeArgs& a, cudaStream_t st) {
    const UPlan pl = gateup_plan(QG, QU, a.D, a.gate_rb, a.up_rb);
    if (pl.u.total > SMEM_CAP) return cudaErrorInvalidValue;
    smem_attr(k_moe_gateup<QG, QU>, pl.u.total);
    const int maxact = std::min(a.n_expert, a.T * a.n_used);
    k_moe_gateup<QG, QU><<<maxact * (a.FF / 16), NTU, pl.u.total, st>>>(a);
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
    const GPlan pl = down_plan(QD, a.FF, a.down_rb);
    if (pl.total > SMEM_CAP) return cudaErrorInvalidValue;
    smem_attr(k_moe_down<QD>, pl.total);
    const int maxact = std::min(a.n_expert, a.T * a.n_used);
    k_moe_down<QD><<<dim3(a.D / 16, maxact), NTU, pl.total, st>>>(a);
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
