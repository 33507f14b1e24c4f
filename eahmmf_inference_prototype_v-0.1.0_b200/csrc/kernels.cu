// kernels.cu -- sm_100a kernels of the dense quantized GEMV (the reference's two C entry points and
// eahmmf_cuda_gemv); the MoE block's kernels are in moe.cu.
//
//   k_prep_x            activations -> fragment form (three int8 digits per element, per-16 sums, row
//                       scale; kq.cuh), once per token row, read by every weight tile afterwards.
//   k_gemv<QT,N>        dense K-quant GEMV: one 16-row tile per CTA, staged HBM -> shared memory with the
//                       tokens' XF rows by 1-D TMA bulk copies on an mbarrier, decoded in registers
//                       straight into int8 tensor-core operands (kq.cuh).
//   k_gemv_generic      one warp per row for F32/F16/Q8_0 and for buffers TMA cannot address.
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
    pdl_wait();
    pdl_trigger();
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
// activations -> fragment form (XF, kq.cuh); one CTA per token row
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(PREP_NT) k_prep_x(const float* __restrict__ X, int ldx, int K, uint2* __restrict__ frag,
                                                     float* __restrict__ sum, uint8_t* __restrict__ gs) {
    __shared__ float red[33];
    const int row = blockIdx.x;
    pdl_wait();
    pdl_trigger();
    prep_row(X + (size_t)row * ldx, K, frag + (size_t)row * (K >> 5) * 12, sum + (size_t)row * ((K >> 4) + XF_SUM_PAD),
             gs + (size_t)row * xf_gs_bytes(K), red);
}

// ------------------------------------------------------------------------------------------------
// dense GEMV tile engine: one 16-row tile per CTA, staged with its tokens' XF rows by 1-D TMA copies
// ------------------------------------------------------------------------------------------------
constexpr int SETS = 2;  // MMA column sets per pass of the dense GEMV (TOK_PER_SET tokens each)
constexpr int TPASS = SETS * TOK_PER_SET;  // tokens per pass of the dense GEMV

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
        for (int r = r0; r < r1; r++)
            tma_load_1d(dst + (size_t)(r - r0) * L.stride, base + (size_t)r * rb, (uint32_t)rb, bar);
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

// Bulk-copies the fragment rows and the sums (with the scale) of m tokens into shared memory (sfrag:
// m x K*3 bytes, ssum: m x (K/16 + 4) floats). rows(i) gives token i's xf row; consecutive rows are
// merged into one copy. Returns the bytes in flight on bar.
template <typename Rows>
__device__ __forceinline__ uint32_t issue_xf(const XF& xf, Rows rows, int m, int K, uint8_t* sfrag, float* ssum,
                                             uint64_t* bar) {
    const uint32_t fb = (uint32_t)K * 3, sbytes = (uint32_t)K / 4 + 4 * XF_SUM_PAD;
    const int ss = (K >> 4) + XF_SUM_PAD;
    uint32_t total = 0;
    for (int i = 0; i < m;) {
        int n = 1;
        while (i + n < m && rows(i + n) == rows(i) + n) n++;
        const size_t r = (size_t)rows(i);
        tma_load_1d(sfrag + (size_t)i * fb, reinterpret_cast<const uint8_t*>(xf.frag) + r * fb, n * fb, bar);
        tma_load_1d(ssum + (size_t)i * ss, xf.sum + r * ss, n * sbytes, bar);
        total += n * (fb + sbytes);
        i += n;
    }
    return total;
}
__device__ __forceinline__ uint32_t xf_bytes_of(int m, int K) {
    return (uint32_t)m * ((uint32_t)K * 3 + (uint32_t)K / 4 + 4 * XF_SUM_PAD);
}

// All MMA tasks (super-block, half) of a staged 16-row tile:
//   part[((task0 + task) * NSET + st) * 128 + row * 8 + column] = d * (int32 digit sums)
//   mpart[(task0 + task) * 64 + row * 4 + token]                = group-minimum term
template <int QT, int NSET>
__device__ __forceinline__ void tile_tasks(const uint8_t* rows, int stride, int nsb, const uint8_t* sfrag,
                                           const float* ssum, int m, float* part, float* mpart, int task0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const BPtr<NSET> bp(sfrag, nsb * 8, m);
    const uint8_t* rg = rows + (size_t)g * stride;
    for (int k = warp; k < nsb * 2; k += (int)(blockDim.x >> 5)) {
        const int sb = k >> 1, h = k & 1;
        float o[NSET][4] = {}, mn[2] = {0.f, 0.f};
        const RowsAny R{{rg, rg + 8 * (size_t)stride}};
        kq_task<QT, NSET>(R, sb, h, bp, t < m ? ssum + (size_t)t * (nsb * 16 + XF_SUM_PAD) + sb * 16 : nullptr, o, mn);
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
    p.part_off = al128(p.ssum_off + (size_t)m * (K / 16 + XF_SUM_PAD) * 4);
    p.mpart_off = al128(p.part_off + (size_t)ntask * nset * 512);
    p.slot_off = al128(p.mpart_off + (size_t)ntask * 256);
    p.total = p.slot_off + slot_bytes_total;
    return p;
}
__host__ __device__ inline GPlan gemv_plan(int qt, int K, size_t rb, int nset, int m) {
    (void)qt;
    return unit_plan(K, m, 2 * (K / 256), nset, slot_bytes(row_layout(rb, true), 16));
}
// shared memory of k_gemv's prologue and combine epilogue (after the plan's total): the fp32 row [K], the
// norm weights [K], the XF gs row, the reduction scratch (33 floats), the pending combine's slots and
// weights (32 each), its y values of the block's 16 rows [32][16] and the residual rows [16]
__host__ __device__ inline size_t gemv_pro_bytes(int K) {
    return (size_t)K * 8 + al128(xf_gs_bytes(K)) + 128 * 3 + 256 + (32 * 16 + 16) * 4;
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
    if (tid == 0) {  // the weight rows do not depend on earlier grids: their copy starts before the wait
        mbar_init(&bar[0], 1);
        mbar_fence_init();
        mbar_expect_tx(&bar[0], rows_bytes(L, a.W.w, rb, r0, r1) + (a.pro ? 0u : xf_bytes_of(m, K)));
        issue_rows(L, a.W.w, rb, r0, r1, slot, &bar[0]);
    }
    // prologue scratch after the plan: the fp32 row, the norm weights, the XF gs row, reductions, slots
    float* prow_s = reinterpret_cast<float*>(sm + pl.total);
    float* nw_s = prow_s + K;
    uint8_t* gs_s = reinterpret_cast<uint8_t*>(nw_s + K);
    float* red = reinterpret_cast<float*>(gs_s + al128(xf_gs_bytes(K)));
    int* sl_s = reinterpret_cast<int*>(red + 64);
    float* sw_s = reinterpret_cast<float*>(sl_s + 32);
    float* ey_s = sw_s + 32;  // [32 slots][16 rows] of the epilogue's pending combine
    float* x_s = ey_s + 32 * 16;
    if (a.pro == GEMV_PRO_NORM)  // the norm weights do not depend on earlier grids
        for (int i = tid; i < K / 4; i += NTU)
            reinterpret_cast<float4*>(nw_s)[i] = __ldg(reinterpret_cast<const float4*>(a.pnw) + i);
    pdl_wait();  // the activations (XF or their fp32 row) and, when accumulating, Y come from earlier grids
    pdl_trigger();
    if (a.pro == GEMV_PRO_XF) {
        if (tid == 0) issue_xf(a.xf, [](int i) { return i; }, m, K, sfrag, ssum, &bar[0]);
    } else {  // the token's row in fragment form, formed here exactly as the norm / merge kernels form it
        if (a.pro == GEMV_PRO_NORM) {
            __syncthreads();  // nw_s
            combine_norm_row(a.prow, a.py, a.pslots, a.pw, a.pK, nw_s, a.peps, K, prow_s, nullptr, nullptr, sl_s, sw_s,
                             red);
        } else {  // the row into shared memory first, every thread's loads in flight together
#pragma unroll 4
            for (int i = tid; i < K / 4; i += NTU)
                reinterpret_cast<float4*>(prow_s)[i] = __ldcg(reinterpret_cast<const float4*>(a.prow) + i);
            __syncthreads();
        }
        prep_row(prow_s, K, reinterpret_cast<uint2*>(sfrag), ssum, gs_s, red);
    }
    if (a.ey) {  // the epilogue's pending combine and residual rows, loaded with the prologue's loads
        for (int i = tid; i < a.eK * 16; i += NTU) {
            const int k = i >> 4, r = i & 15, sl = a.eslots ? a.eslots[k] : k;
            ey_s[i] = r0 + r < r1 ? a.ey[(size_t)sl * a.W.rows + r0 + r] : 0.f;
            if (r == 0) sw_s[k] = a.ew[sl];
        }
        if (tid < 16) x_s[tid] = r0 + tid < r1 ? a.Y[r0 + tid] : 0.f;
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
    tile_tasks<QT, NSET>(rows, L.stride, nsb, sfrag, ssum, m, part, mpart, 0);
    __syncthreads();
    for (int j = tid; j < (r1 - r0) * m; j += blockDim.x) {
        const int r = j / m, tk = j - r * m;
        const float v = tile_value<NSET>(part, mpart, 0, r, nsb, tk, ssum[(size_t)tk * (16 * nsb + XF_SUM_PAD) + 16 * nsb]);
        float* y = a.Y + (size_t)tk * a.ldy + r0 + r;
        if (a.accumulate) {
            float base = *y;
            if (a.ey) {  // x + sum_k w_k y_k in the norm kernel's order (combine_norm_row), then + v
                float acc = 0.f;
                for (int k = 0; k < a.eK; k++) acc = fmaf(sw_s[k], ey_s[k * 16 + r], acc);
                base = x_s[r] + acc;
            }
            *y = base + v;
        } else {
            *y = v;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// dense K-quant GEMM over many tokens (prompt passes): the 16-row weight tile is staged once and every
// warp runs four tokens (two column sets) over all of the tile's tasks, fetching the next task's
// activation fragments (global memory, L2-resident) while the current one computes. Each token's value
// is the same sum, in the same order, as k_gemv's (tile_tasks + tile_value), so results do not depend
// on how the tokens are split into passes.
// ------------------------------------------------------------------------------------------------
constexpr int GX_TMAX = 64;                  // tokens per launch
constexpr int GX_NT = 32 * (GX_TMAX / 4);    // one warp per four tokens
constexpr int GX_SCR = 2 * 128 + 64;         // floats of per-warp scratch: two sets' partials, minimums
__host__ __device__ inline size_t gemm_xf_smem(size_t rb, int nwarps) {
    return 128 + slot_bytes(row_layout(rb, true), 16) + (size_t)nwarps * GX_SCR * 4;
}
template <int QT>
__global__ void __launch_bounds__(GX_NT, 1) k_gemm_xf(GemvXArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int K = a.W.K, nsb = K >> 8, m = a.m, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const size_t rb = a.W.row_bytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    uint8_t* slot = sm + 128;
    float* scr = reinterpret_cast<float*>(sm + 128 + slot_bytes(row_layout(rb, true), 16)) + (size_t)warp * GX_SCR;
    const RowLayout L = layout_of(a.W.w, rb);
    const int r0 = 16 * (int)blockIdx.x, r1 = min(a.W.rows, r0 + 16);
    if (tid == 0) {  // the weight rows do not depend on earlier grids: their copy starts before the wait
        mbar_init(&bar[0], 1);
        mbar_fence_init();
        mbar_expect_tx(&bar[0], rows_bytes(L, a.W.w, rb, r0, r1));
        issue_rows(L, a.W.w, rb, r0, r1, slot, &bar[0]);
    }
    pdl_wait();  // the activations (XF) and, when accumulating, Y come from earlier grids
    pdl_trigger();
    __syncthreads();
    if (__syncthreads_or(!mbar_wait_bounded(&bar[0], 0u))) {
        if (tid == 0) {
            flag(a.status, ST_WAIT_TIMEOUT);
            drain_ring(bar, 1, 0, 1);
        }
        return;
    }
    const int tk0 = 4 * warp;
    if (tk0 >= m) return;  // whole warps; no block-wide barrier follows
    const int mw = min(4, m - tk0), ss = (K >> 4) + XF_SUM_PAD;
    const BPtr<2> bp(reinterpret_cast<const uint8_t*>(a.xf.frag) + (size_t)tk0 * K * 3, K >> 5, mw);
    const float* tsum = t < mw ? a.xf.sum + (size_t)(tk0 + t) * ss : nullptr;  // lane t's token
    const uint8_t* rows = slot + rows_lead(L, a.W.w, rb, r0);
    const uint8_t* rg = rows + (size_t)g * L.stride;
    const RowsAny R{{rg, rg + 8 * (size_t)L.stride}};
    float run[2][4] = {}, mnr[2] = {0.f, 0.f};
    auto step = [&](int k, const KqB<QT, 2>& B) {
        float o[2][4] = {}, mn[2] = {0.f, 0.f};
        kq_compute<QT, 2>(R, k >> 1, k & 1, t, B, tsum != nullptr, o, mn);
#pragma unroll
        for (int st = 0; st < 2; st++)
#pragma unroll
            for (int i = 0; i < 4; i++) run[st][i] += o[st][i];
        mnr[0] += mn[0];
        mnr[1] += mn[1];
    };
    auto tsum_at = [&](int k) { return tsum ? tsum + (k >> 1) * 16 : nullptr; };
    KqB<QT, 2> B0, B1;
    kq_load_b<QT, 2>(bp, 0, 0, tsum_at(0), B0);
    for (int k = 0; k < 2 * nsb; k += 2) {  // tasks in super-block order, two per pass (B0, B1 alternate)
        kq_load_b<QT, 2>(bp, (k + 1) >> 1, (k + 1) & 1, tsum_at(k + 1), B1);
        step(k, B0);
        if (k + 2 < 2 * nsb) kq_load_b<QT, 2>(bp, (k + 2) >> 1, (k + 2) & 1, tsum_at(k + 2), B0);
        step(k + 1, B1);
    }
    // the warp's partial sums in tile_tasks' layout (one task), then tile_value's recombination
#pragma unroll
    for (int st = 0; st < 2; st++) {
        *reinterpret_cast<float2*>(scr + st * 128 + g * 8 + 2 * t) = make_float2(run[st][0], run[st][1]);
        *reinterpret_cast<float2*>(scr + st * 128 + (g + 8) * 8 + 2 * t) = make_float2(run[st][2], run[st][3]);
    }
    scr[256 + g * 4 + t] = mnr[0];
    scr[256 + (g + 8) * 4 + t] = mnr[1];
    __syncwarp();
    for (int j = lane; j < 64; j += 32) {
        const int r = j >> 2, tk = j & 3;
        if (tk < mw && r0 + r < r1) {
            const float* p = scr + (tk / TOK_PER_SET) * 128 + r * 8 + 3 * (tk % TOK_PER_SET);
            const float ts = a.xf.sum[(size_t)(tk0 + tk) * ss + (K >> 4)];
            const float v = fmaf(fmaf(fmaf(p[2], 1.0f / DIGIT, p[1]), 1.0f / DIGIT, p[0]), ts, -scr[256 + r * 4 + tk]);
            float* y = a.Y + (size_t)(tk0 + tk) * a.ldy + r0 + r;
            *y = a.accumulate ? *y + v : v;
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

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
constexpr size_t SMEM_CAP = 227 * 1024;

bool gemv_mma_ok(const QMat& W) {
    return is_kquant(W.type) && aligned16(W.w) && W.K % 256 == 0 && W.row_bytes == (size_t)(W.K / 256) * block_bytes(W.type) &&
           gemv_plan(W.type, W.K, W.row_bytes, SETS, TPASS).total <= SMEM_CAP;
}

XF xf_carve(void* base, int rows, int K) {
    uint8_t* p = static_cast<uint8_t*>(base);
    XF x;
    x.frag = reinterpret_cast<const uint2*>(p);
    x.sum = reinterpret_cast<const float*>(p + (size_t)rows * K * 3);
    x.gs = p + (size_t)rows * K * 3 + (size_t)rows * (K / 16 + XF_SUM_PAD) * 4;
    x.nseg = K / 16;
    return x;
}

cudaError_t launch_prep_x(const float* X, int ldx, int rows, int K, const XF& out, cudaStream_t st) {
    if (rows < 1 || K % 256 || ldx % 4 || !aligned16(X)) return cudaErrorInvalidValue;
    return launch_pdl(k_prep_x, dim3(rows), dim3(PREP_NT), 0, st, X, ldx, K, const_cast<uint2*>(out.frag),
                      const_cast<float*>(out.sum), const_cast<uint8_t*>(out.gs));
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
    const size_t smem = pl.total + (a.pro || a.ey ? gemv_pro_bytes(a.W.K) : 0);
    smem_attr(k_gemv<QT, NSET>, smem);
    launch_pdl(k_gemv<QT, NSET>, dim3((a.W.rows + 15) / 16), dim3(NTU), smem, st, a);
}

cudaError_t launch_gemv_xf(const GemvXArgs& a, cudaStream_t st) {
    if (a.m < 1 || a.m > TPASS || !gemv_mma_ok(a.W)) return cudaErrorInvalidValue;
    if ((a.pro && (a.m != 1 || !a.prow || (a.pro == GEMV_PRO_NORM && (!a.pnw || a.pK > 32)) ||
                   gemv_plan(a.W.type, a.W.K, a.W.row_bytes, 1, 1).total + gemv_pro_bytes(a.W.K) > SMEM_CAP)) ||
        (a.ey && (a.m != 1 || !a.accumulate || a.eK > 32 ||
                  gemv_plan(a.W.type, a.W.K, a.W.row_bytes, 1, 1).total + gemv_pro_bytes(a.W.K) > SMEM_CAP)))
        return cudaErrorInvalidValue;
    const bool two = a.m > TOK_PER_SET;
    switch (a.W.type) {
        case T_Q4_K: two ? gemv_go<T_Q4_K, 2>(a, st) : gemv_go<T_Q4_K, 1>(a, st); break;
        case T_Q5_K: two ? gemv_go<T_Q5_K, 2>(a, st) : gemv_go<T_Q5_K, 1>(a, st); break;
        default: two ? gemv_go<T_Q6_K, 2>(a, st) : gemv_go<T_Q6_K, 1>(a, st); break;
    }
    return cudaGetLastError();
}

template <int QT>
static void gemm_xf_go(const GemvXArgs& a, cudaStream_t st) {
    const int nw = (a.m + 3) / 4;
    const size_t smem = gemm_xf_smem(a.W.row_bytes, nw);
    smem_attr(k_gemm_xf<QT>, gemm_xf_smem(a.W.row_bytes, GX_TMAX / 4));
    launch_pdl(k_gemm_xf<QT>, dim3((a.W.rows + 15) / 16), dim3(32 * nw), smem, st, a);
}

bool gemm_xf_ok(const QMat& W) {
    return gemv_mma_ok(W) && gemm_xf_smem(W.row_bytes, GX_TMAX / 4) <= SMEM_CAP;
}

cudaError_t launch_gemm_xf(const GemvXArgs& a, cudaStream_t st) {
    if (a.m < 1 || a.m > GX_TMAX || !gemm_xf_ok(a.W)) return cudaErrorInvalidValue;
    switch (a.W.type) {
        case T_Q4_K: gemm_xf_go<T_Q4_K>(a, st); break;
        case T_Q5_K: gemm_xf_go<T_Q5_K>(a, st); break;
        default: gemm_xf_go<T_Q6_K>(a, st); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t st) {
    if (a.m < 1 || a.m > MT) return cudaErrorInvalidValue;
    return launch_pdl(k_gemv_generic, dim3((a.W.rows * 32 + 255) / 256), dim3(256), 0, st, a);
}

constexpr int F32_NT = 128;
constexpr int F32_PF = 8;  // float4 per thread of the weight row loaded before the grid-dependency wait
__global__ void __launch_bounds__(F32_NT) k_gemv_f32(const float* __restrict__ W, int K, int rows,
                                                     const float* __restrict__ X, int ldx, int m_all,
                                                     float* __restrict__ Y, int ldy, XF xf, int prep,
                                                     const float* __restrict__ nw, float eps) {
    extern __shared__ __align__(16) float nrow[];  // [K] (prep blocks with a norm)
    __shared__ float red[F32_NT / 32][MT];
    __shared__ float red4[4];
    __shared__ float s_sc[MT];
    const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // The row's weights and the norm weights do not depend on earlier grids: the first F32_PF float4 of
    // each thread are loaded before the wait, so the HBM latency overlaps the previous kernel's tail.
    const int n4 = K / 4;
    const float4* w4 = reinterpret_cast<const float4*>(W + (size_t)min(row, rows - 1) * K);
    const float4* g4 = reinterpret_cast<const float4*>(nw);
    float4 wpf[F32_PF], gpf[F32_PF];
#pragma unroll
    for (int j = 0; j < F32_PF; j++) {
        const int i = threadIdx.x + j * F32_NT;
        wpf[j] = row < rows && i < n4 ? __ldg(w4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        gpf[j] = nw && i < n4 ? __ldg(g4 + i) : make_float4(1.f, 1.f, 1.f, 1.f);  // prep blocks too
    }
    pdl_wait();
    pdl_trigger();
    if (row >= rows) {  // blocks past the matrix: token (row - rows) in fragment form for the expert kernels
        __shared__ float pred[33];
        const int t = row - rows;
        if (!(prep && blockIdx.y == 0 && t < m_all)) return;
        const float* xr = X + (size_t)t * ldx;
        if (nw) {  // RMSNorm of the row first (qwen3moe.cpp:527-532); the first F32_PF float4 of the norm
                   // weights per thread were loaded before the wait
            const float sc = 1.0f / sqrtf(row_sumsq128(xr, K, red4) / (float)K + eps);
            const float4* x4 = reinterpret_cast<const float4*>(xr);
            auto norm4 = [&](int i, const float4& g) {
                const float4 v = x4[i];
                reinterpret_cast<float4*>(nrow)[i] = make_float4(__fmul_rn(__fmul_rn(v.x, sc), g.x), __fmul_rn(__fmul_rn(v.y, sc), g.y),
                                                                 __fmul_rn(__fmul_rn(v.z, sc), g.z), __fmul_rn(__fmul_rn(v.w, sc), g.w));
            };
#pragma unroll
            for (int j = 0; j < F32_PF; j++)
                if (threadIdx.x + j * F32_NT < n4) norm4(threadIdx.x + j * F32_NT, gpf[j]);
            for (int i = threadIdx.x + F32_PF * F32_NT; i < n4; i += F32_NT) norm4(i, __ldg(g4 + i));
            __syncthreads();
            xr = nrow;
        }
        prep_row(xr, K, const_cast<uint2*>(xf.frag) + (size_t)t * (K >> 5) * 12,
                 const_cast<float*>(xf.sum) + (size_t)t * ((K >> 4) + XF_SUM_PAD),
                 const_cast<uint8_t*>(xf.gs) + (size_t)t * xf_gs_bytes(K), pred);
        return;
    }
    const int t0 = blockIdx.y * MT, m = min(MT, m_all - t0);  // this block's tokens
    X += (size_t)t0 * ldx;
    Y += (size_t)t0 * ldy;
    if (nw) {
        for (int t = 0; t < m; t++) {
            const float sc = 1.0f / sqrtf(row_sumsq128(X + (size_t)t * ldx, K, red4) / (float)K + eps);
            if (threadIdx.x == 0) s_sc[t] = sc;
        }
        __syncthreads();
    }
    float acc[MT];
#pragma unroll
    for (int t = 0; t < MT; t++) acc[t] = 0.f;
    // element groups i = tid, tid + F32_NT, ... in order (the first F32_PF from the prefetched registers)
    auto step = [&](const float4& w, const float4& g, int i) {
#pragma unroll
        for (int t = 0; t < MT; t++) {
            if (t < m) {
                float4 x = __ldg(reinterpret_cast<const float4*>(X + (size_t)t * ldx) + i);
                if (nw) {  // the normalised element, exactly as the prep blocks form it
                    const float sc = s_sc[t];
                    x.x = __fmul_rn(__fmul_rn(x.x, sc), g.x);
                    x.y = __fmul_rn(__fmul_rn(x.y, sc), g.y);
                    x.z = __fmul_rn(__fmul_rn(x.z, sc), g.z);
                    x.w = __fmul_rn(__fmul_rn(x.w, sc), g.w);
                }
                acc[t] = fmaf(w.x, x.x, fmaf(w.y, x.y, fmaf(w.z, x.z, fmaf(w.w, x.w, acc[t]))));
            }
        }
    };
#pragma unroll
    for (int j = 0; j < F32_PF; j++)
        if (threadIdx.x + j * F32_NT < n4) step(wpf[j], gpf[j], threadIdx.x + j * F32_NT);
#pragma unroll 1
    for (int i = threadIdx.x + F32_PF * F32_NT; i < n4; i += F32_NT)
        step(__ldg(w4 + i), nw ? __ldg(g4 + i) : make_float4(1.f, 1.f, 1.f, 1.f), i);
#pragma unroll
    for (int t = 0; t < MT; t++) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp][t] = v;
    }
    __syncthreads();
    if (threadIdx.x < m) {
        const int t = threadIdx.x;
        Y[(size_t)t * ldy + row] = (red[0][t] + red[1][t]) + (red[2][t] + red[3][t]);
    }
}

// F32 rows (the router, qwen3moe.cpp:1008): one 128-thread block per (row, MT tokens), the four warps
// taking interleaved float4 slices of the row so every thread has all its loads in flight at once; the
// four partial sums are added in a fixed order (deterministic).
cudaError_t launch_router_prep(const float* W, int K, int rows, const float* X, int ldx, int m, float* Y, int ldy,
                               const XF& xf, const float* norm_w, float eps, cudaStream_t st) {
    if (K % 256 || ldx % 4 || (reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(X) & 15) ||
        (norm_w && (reinterpret_cast<uintptr_t>(norm_w) & 15)))
        return cudaErrorInvalidValue;
    const size_t smem = norm_w ? (size_t)K * 4 : 0;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k_gemv_f32, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return launch_pdl(k_gemv_f32, dim3(rows + m, (m + MT - 1) / MT), dim3(F32_NT), smem, st, W, K, rows, X, ldx, m,
                      Y, ldy, xf, 1, norm_w, eps);
}

// F32 rows over more than MT tokens (the router of a prompt pass): one block per (F32_TR rows, F32_TT
// tokens), so that every weight and token float4 read from L2 serves F32_TT (F32_TR) products instead
// of one row's MT tokens. Each (row, token) sum is formed exactly as k_gemv_f32 forms it: thread i owns
// the float4 groups i, i + F32_NT, ... in order with the same fmaf nesting, then the same warp
// butterfly and the same fixed-order sum of the four warps' partials, so the logits are bitwise those
// of the small-batch kernel.
constexpr int F32_TR = 4, F32_TT = 8;
__global__ void __launch_bounds__(F32_NT) k_gemv_f32_tile(const float* __restrict__ W, int K, int rows,
                                                          const float* __restrict__ X, int ldx, int m_all,
                                                          float* __restrict__ Y, int ldy) {
    __shared__ float red[F32_NT / 32][F32_TR][F32_TT];
    const int r0 = blockIdx.x * F32_TR, t0 = blockIdx.y * F32_TT, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nr = min(F32_TR, rows - r0), m = min(F32_TT, m_all - t0), n4 = K / 4;
    const float4* w4 = reinterpret_cast<const float4*>(W) + (size_t)r0 * n4;
    const float4* x4 = reinterpret_cast<const float4*>(X + (size_t)t0 * ldx);
    const int ld4 = ldx / 4;
    pdl_wait();
    pdl_trigger();
    float acc[F32_TR][F32_TT];
#pragma unroll
    for (int r = 0; r < F32_TR; r++)
#pragma unroll
        for (int t = 0; t < F32_TT; t++) acc[r][t] = 0.f;
#pragma unroll 2
    for (int i = threadIdx.x; i < n4; i += F32_NT) {
        float4 w[F32_TR], x[F32_TT];
#pragma unroll
        for (int r = 0; r < F32_TR; r++) w[r] = r < nr ? __ldg(w4 + (size_t)r * n4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int t = 0; t < F32_TT; t++) x[t] = t < m ? __ldg(x4 + (size_t)t * ld4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < F32_TR; r++)
#pragma unroll
            for (int t = 0; t < F32_TT; t++)
                acc[r][t] = fmaf(w[r].x, x[t].x, fmaf(w[r].y, x[t].y, fmaf(w[r].z, x[t].z, fmaf(w[r].w, x[t].w, acc[r][t]))));
    }
#pragma unroll
    for (int r = 0; r < F32_TR; r++)
#pragma unroll
        for (int t = 0; t < F32_TT; t++) {
            float v = acc[r][t];
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red[warp][r][t] = v;
        }
    __syncthreads();
    for (int idx = threadIdx.x; idx < F32_TR * F32_TT; idx += F32_NT) {
        const int r = idx / F32_TT, t = idx - r * F32_TT;
        if (r < nr && t < m)
            Y[(size_t)(t0 + t) * ldy + r0 + r] = (red[0][r][t] + red[1][r][t]) + (red[2][r][t] + red[3][r][t]);
    }
}

cudaError_t launch_f32_gemv(const float* W, int K, int rows, const float* X, int ldx, int m, float* Y, int ldy,
                            cudaStream_t st) {
    const bool vec = K % 4 == 0 && ldx % 4 == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(X) & 15) == 0;
    if (vec && m > MT)
        return launch_pdl(k_gemv_f32_tile, dim3((rows + F32_TR - 1) / F32_TR, (m + F32_TT - 1) / F32_TT), dim3(F32_NT), 0,
                          st, W, K, rows, X, ldx, m, Y, ldy);
    if (vec)
        return launch_pdl(k_gemv_f32, dim3(rows, (m + MT - 1) / MT), dim3(F32_NT), 0, st, W, K, rows, X, ldx, m, Y,
                          ldy, XF{}, 0, static_cast<const float*>(nullptr), 0.f);
    for (int t0 = 0; t0 < m; t0 += MT) {  // other layouts: the per-row kernel, MT tokens per pass
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
