// moe.cu -- the MoE block (qwen3moe.cpp:1006-1069) on sm_100a as three launches chained by programmatic
// dependent launch (each starts while its predecessor finishes and waits in griddepcontrol.wait):
//
//   k_moe_route       block 0: router softmax + top-k + renormalisation (warp per token, the CPU
//                     comparator of qwen3moe.cpp:1016), then the token->expert grouping: per-expert
//                     token bitmasks (histogram), exclusive scan, stable scatter into expert-major slots,
//                     and the work list: groups of up to MU consecutive slots of one expert, each with
//                     its expert's weight pointers and tokens (GroupRec).
//                     blocks 1..T: the tokens' activations in fragment form (XF).
//   k_moe_gateup<G,U> persistent, one CTA per SM: units (group, 16 rows of FF) in contiguous ranges per
//                     CTA. A producer warp streams each unit's gate and up rows HBM -> shared memory
//                     through a ring of mbarrier-guarded stages, with the group's XF rows when the group
//                     changes; 16 consumer warps run the int8 tensor-core GEMV (kq.cuh) with register
//                     accumulators and read nothing from global memory; the last warp to finish a unit
//                     reduces it and writes SiLU(g)*u. A 1-D bulk copy costs about the same time
//                     whether it moves 1 KB or 9 KB (one copy per ~0.2 us per SM), so a matrix's 16 rows
//                     come as two 8-row copies, the second placed 32 bytes off the first's bank
//                     alignment, instead of sixteen row copies.
//   (Up to FUSED_ROUTE_TMAX tokens, the gate/up kernel routes the tokens itself from the logits and its
//   CTA 0 publishes the groups and slot maps for the down kernel and the combine.)
//   k_moe_down<D>     persistent likewise over units (group, 64 rows of D) with 12 consumer warps. The
//                     consumers put each group's h rows in fragment form in shared memory themselves
//                     (the first group's while the first weight tiles are in flight). Each unit's reducer
//                     only stores its y rows: no counters or dependent loads in the pipelined loop.
//   k_moe_combine     adds each token's K expert outputs, weighted, in ascending expert order
//                     (qwen3moe.cpp:1025-1069) to the residual once the down grid has completed.
//
// Every mbarrier wait is bounded; a timeout flags ST_WAIT_TIMEOUT, stops the producer, drains the copies
// already in flight (bounded) and ends the CTA.
#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.cuh"
#include "kq.cuh"
#include "ksb.cuh"

namespace eb {

namespace {

__device__ __forceinline__ void set_flag(int* status, int bits) {
    if (status) atomicOr(status, bits);
}
__host__ __device__ constexpr size_t al128(size_t x) { return (x + 127) & ~(size_t)127; }
__device__ __forceinline__ bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Row placement of a staged tile (as in the dense GEMV): rows whose stride is a multiple of 32 words
// are copied one bulk copy per row into a 16-byte padded stride (bank spread); other strides as one
// contiguous span from the 16-byte boundary at or below the first row.
struct Rows {
    int per_row;
    int stride;
};
__host__ __device__ inline Rows rows_of(size_t rb) {
    if (rb % 16 == 0 && (rb % 128) % 32 == 0) return {1, (int)rb + 16};
    return {0, (int)rb};
}
__host__ __device__ inline size_t rows_slot(size_t rb, int n) { return al128((size_t)n * rows_of(rb).stride + 64); }
__device__ __forceinline__ uint32_t rows_copy_bytes(const Rows& L, const uint8_t* base, size_t rb, int r0, int n) {
    if (L.per_row) return (uint32_t)(n * rb);
    const uintptr_t s = reinterpret_cast<uintptr_t>(base) + (size_t)r0 * rb, e = s + (size_t)n * rb;
    return (uint32_t)(((e + 15) & ~(uintptr_t)15) - (s & ~(uintptr_t)15));
}
__device__ __forceinline__ uint32_t rows_lead(const Rows& L, const uint8_t* base, size_t rb, int r0) {
    return L.per_row ? 0u : (uint32_t)((reinterpret_cast<uintptr_t>(base) + (size_t)r0 * rb) & 15);
}
__device__ __forceinline__ void rows_issue(const Rows& L, const uint8_t* base, size_t rb, int r0, int n, uint8_t* dst,
                                           uint64_t* bar) {
    if (L.per_row) {
        for (int r = 0; r < n; r++)
            tma_load_1d(dst + (size_t)r * L.stride, base + (size_t)(r0 + r) * rb, (uint32_t)rb, bar);
        return;
    }
    const uintptr_t s = reinterpret_cast<uintptr_t>(base) + (size_t)r0 * rb;
    tma_load_1d(dst, reinterpret_cast<const void*>(s & ~(uintptr_t)15), rows_copy_bytes(L, base, rb, r0, n), bar);
}

// Staging buffer of G XF rows of K elements (G: slots per work group): frag rows (K*3 bytes each), then
// the rows' scale and group sums (XF gs rows, 16 + K/8 bytes each).
__host__ __device__ constexpr size_t xs_gs_off(int K, int G = MU) { return (size_t)G * K * 3; }
__host__ __device__ constexpr size_t xs_bytes(int K, int G = MU) { return al128(xs_gs_off(K, G) + (size_t)G * xf_gs_bytes(K)); }

// Bulk copy of the XF rows of a group's mc tokens (tok[0..mc)) into a staging buffer of G rows; runs of
// consecutive token rows go as one copy per array.
template <int G>
__device__ __forceinline__ void xf_issue(const XF& xf, const int* tok, int mc, int K, uint8_t* dst, uint64_t* bar) {
    const uint32_t fb = (uint32_t)K * 3, sb = (uint32_t)xf_gs_bytes(K);
    const uint8_t* F = reinterpret_cast<const uint8_t*>(xf.frag);
    const uint8_t* Sg = xf.gs;
    for (int k = 0; k < mc;) {
        int n = 1;
        while (k + n < mc && tok[k + n] == tok[k] + n) n++;
        tma_load_1d(dst + (size_t)k * fb, F + (size_t)tok[k] * fb, n * fb, bar);
        tma_load_1d(dst + xs_gs_off(K, G) + (size_t)k * sb, Sg + (size_t)tok[k] * sb, n * sb, bar);
        k += n;
    }
}

// After a failed wait: every stage that may still have copies in flight gets one more bounded wait.
__device__ void drain(uint64_t* full, int issued, int consumed, int S) {
    for (int i = consumed; i < issued; i++) mbar_wait_bounded(&full[i % S], (uint32_t)(i / S) & 1u);
}

// ---- shared-memory plan of the persistent kernels ---------------------------------------------------
//   [0, 128)     mbarriers: full[4], empty[4], done[4], the down kernel's consumer barrier
//   info         per-stage unit descriptors (int4)
//   cnt          per-stage finished-warp counters
//   xf           two XF staging buffers (double-buffered by group)
//   part         per-stage, per-warp partial results [S][NWC][16 rows][G]
//   comb         combine scratch of the down kernel (slots and weights of T*K (token, k) pairs)
//   stages       the ring
struct Plan {
    int S;
    size_t info_off, cnt_off, xf_off, xfb, part_off, comb_off, stage_off, stage_bytes, extra_off, total;
};
constexpr size_t SMEM_CAP = 227 * 1024;
__host__ __device__ inline Plan make_plan(int nwc, int K, size_t stage_bytes, size_t comb_bytes, size_t extra = 0,
                                         int G = MU) {
    Plan p;
    p.info_off = 128;
    p.cnt_off = p.info_off + 4 * 16;
    p.xf_off = al128(p.cnt_off + 4 * 4);
    p.xfb = xs_bytes(K, G);
    p.part_off = al128(p.xf_off + 2 * p.xfb);
    const size_t part_bytes = (size_t)nwc * 16 * G * 4;
    p.stage_bytes = al128(stage_bytes);
    p.S = 4;
    for (;; p.S--) {
        p.comb_off = al128(p.part_off + (size_t)p.S * part_bytes);
        p.stage_off = al128(p.comb_off + comb_bytes);
        p.extra_off = al128(p.stage_off + (size_t)p.S * p.stage_bytes);
        p.total = p.extra_off + extra;
        if (p.total <= SMEM_CAP || p.S == 2) break;
    }
    return p;
}
constexpr int NWC_GU = 16;   // consumer warps of the gate/up kernel
constexpr int NWC_DN = 12;   // consumer warps of the down kernel
constexpr int DN_ROWS = 64;  // rows of D per down unit
// 8-element items of a group's h rows per consumer thread of the down kernel: G * FF <= 8 * 32 * NWC_DN * this
__host__ __device__ constexpr int dn_prep_items(int G) { return G <= 2 ? 2 : 4; }
// Gate/up tiles: 16 rows of a matrix. Rows of a multiple of 16 bytes come as two 8-row copies, the
// second at split8_off(rb) (32 bytes past a 128-byte boundary, so that rows 0..7 and 8..15 start on
// different banks); other rows as one contiguous span copy.
__host__ __device__ inline bool split8(size_t rb) { return rb % 16 == 0; }
__host__ __device__ inline size_t split8_off(size_t rb) { return al128(8 * rb) + 32; }
__host__ __device__ inline size_t gu_slot(size_t rb) { return split8(rb) ? al128(split8_off(rb) + 8 * rb) : al128(16 * rb + 64); }
__host__ __device__ inline Plan gateup_plan(int D, size_t rbg, size_t rbu, size_t route_bytes = 0, int G = MU) {
    return make_plan(NWC_GU, D, gu_slot(rbg) + gu_slot(rbu), 0, route_bytes, G);
}
__host__ __device__ inline Plan down_plan(int FF, size_t rbd, size_t route_bytes = 0, int G = MU) {
    return make_plan(NWC_DN, FF, rows_slot(rbd, DN_ROWS), 0, route_bytes, G);
}
// the down kernel's shared-memory copy of the group list (small batches, whose gate/up kernel routed)
__host__ __device__ inline size_t down_cache_bytes(const MoeArgs& a) {
    return a.fused_route ? (size_t)a.T * a.n_used * sizeof(GroupRec) : 0;
}

// info word y: xf buffer (bit 0), slots in the group (bits 4-7), weights usable (bit 8), first unit of
// the group in this CTA (bit 9)
__device__ __forceinline__ int info_bits(int xb, int mc, bool ok, bool fresh) {
    return xb | (mc << 4) | (ok ? 256 : 0) | (fresh ? 512 : 0);
}

// Per-warp epilogue of a 16-row block (one column set, <= 2 tokens): the lane's digit columns are
// recombined across lanes, value = (a + b/254 + c/254^2 - min) * s; lanes t = 0, 1 end up with token
// t's values of MMA rows g and g+8, which hold the block's rows row0 and row1. Stored to
// part[row * G + slot0 + t] (part: [16][G]; the set's tokens are the group's slots slot0, slot0 + 1).
__device__ __forceinline__ void warp_values(const float (&acc)[1][4], const float (&mn)[2], float ts, float* part,
                                            int row0, int row1, int G = MU, int slot0 = 0) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const float A0 = __shfl_down_sync(0xffffffffu, acc[0][0], 1), B0 = __shfl_down_sync(0xffffffffu, acc[0][1], 1);
    const float A1 = __shfl_down_sync(0xffffffffu, acc[0][2], 1), B1 = __shfl_down_sync(0xffffffffu, acc[0][3], 1);
    constexpr float R = 1.0f / DIGIT;
    float v0, v1;
    if (t == 0) {  // token 0: columns 0, 1 (own), 2 (lane t+1's first)
        v0 = fmaf(fmaf(A0, R, acc[0][1]), R, acc[0][0]);
        v1 = fmaf(fmaf(A1, R, acc[0][3]), R, acc[0][2]);
    } else {  // token 1: column 3 (own second), 4, 5 (lane t+1's)
        v0 = fmaf(fmaf(B0, R, A0), R, acc[0][1]);
        v1 = fmaf(fmaf(B1, R, A1), R, acc[0][3]);
    }
    (void)g;
    if (t < 2) {
        part[row0 * G + slot0 + t] = (v0 - mn[0]) * ts;
        part[row1 * G + slot0 + t] = (v1 - mn[1]) * ts;
    }
}

// Item i of a row in fragment form (block j = i / 4, lane t = i % 4: elements 8i .. 8i + 7, held in u, w):
// its three digit planes into frag and, from lane t = 0 of each block, the group sum into gs. All 32
// lanes of the warp take part (shuffles).
__device__ __forceinline__ void prep_item(const float4& u, const float4& w, int i, float inv, uint2* __restrict__ frag,
                                          uint8_t* __restrict__ gs) {
    const int j = i >> 2, t = i & 3;
    const float xv[8] = {u.x, u.y, u.z, u.w, w.x, w.y, w.z, w.w};
    uint2 pl[3];
    digits8(xv, inv, pl);
    uint2* o = frag + (size_t)j * 12 + t;
#pragma unroll
    for (int p = 0; p < 3; p++) o[p * 4] = pl[p];
    float s8 = ((u.x + u.y) + (u.z + u.w)) + ((w.x + w.y) + (w.z + w.w));
    s8 += __shfl_xor_sync(0xffffffffu, s8, 1);
    s8 += __shfl_xor_sync(0xffffffffu, s8, 2);
    if (t == 0) put_group_sum(gs, j, s8 * inv);
}

// The super-blocks sb0, sb0 + step, ... of one warp on a staged 16-row block (rows.r[0], rows.r[1]: the
// block's rows held by MMA rows g and g+8), accumulated in registers (ksb.cuh).
template <int QT>
__device__ __forceinline__ void block_tasks(const RowsAny& rows, int nsb, int sb0, int step, const BPtr<1>& bp,
                                            const uint8_t* mq, float (&acc)[1][4], float (&mn)[2]) {
    const int t = threadIdx.x & 3;
    for (int sb = sb0; sb < nsb; sb += step) {
        const uint8_t* r0 = rows.r[0] + (size_t)sb * block_bytes(QT);
        const uint8_t* r1 = rows.r[1] + (size_t)sb * block_bytes(QT);
        if constexpr (QT == T_Q6_K) {
            const uint8_t* bq = bp.p[0] + 4 * t + 768 * sb;
            const bool m0 = (smem_u32(r0) & 2u) != 0, m1 = (smem_u32(r1) & 2u) != 0;  // warp-uniform
            if (m0) {
                if (m1) sb_q6<true, true>(r0, r1, bq, t, acc[0]);
                else sb_q6<true, false>(r0, r1, bq, t, acc[0]);
            } else {
                if (m1) sb_q6<false, true>(r0, r1, bq, t, acc[0]);
                else sb_q6<false, false>(r0, r1, bq, t, acc[0]);
            }
        } else {
            sb_q45<QT>(r0, r1, bp.p[0] + 8 * t + 768 * sb, mq + 32 * sb, t, acc[0], mn);
        }
    }
}
// block_tasks over NS column sets at once (sets of a larger group): each super-block's weights are
// decoded once for all sets; per set the sums are bitwise block_tasks' (ksb.cuh: sb_q45m, sb_q6m).
// bq[s]: set s's B-fragment base (BPtr<1>::p[0]); mq[s]: its minimum-term operand (Q4_K/Q5_K).
template <int QT, int NS>
__device__ __forceinline__ void block_tasks_m(const RowsAny& rows, int nsb, int sb0, int step,
                                              const uint8_t* const (&bq)[NS], const uint8_t* const (&mq)[NS],
                                              float (&acc)[NS][4], float (&mn)[NS][2]) {
    const int t = threadIdx.x & 3;
    for (int sb = sb0; sb < nsb; sb += step) {
        const uint8_t* r0 = rows.r[0] + (size_t)sb * block_bytes(QT);
        const uint8_t* r1 = rows.r[1] + (size_t)sb * block_bytes(QT);
        const uint8_t* b[NS];
        if constexpr (QT == T_Q6_K) {
#pragma unroll
            for (int k = 0; k < NS; k++) b[k] = bq[k] + 4 * t + 768 * sb;
            const bool m0 = (smem_u32(r0) & 2u) != 0, m1 = (smem_u32(r1) & 2u) != 0;  // warp-uniform
            if (m0) {
                if (m1) sb_q6m<true, true, NS>(r0, r1, b, t, acc);
                else sb_q6m<true, false, NS>(r0, r1, b, t, acc);
            } else {
                if (m1) sb_q6m<false, true, NS>(r0, r1, b, t, acc);
                else sb_q6m<false, false, NS>(r0, r1, b, t, acc);
            }
        } else {
            const uint8_t* m[NS];
#pragma unroll
            for (int k = 0; k < NS; k++) {
                b[k] = bq[k] + 8 * t + 768 * sb;
                m[k] = mq[k] + 32 * sb;
            }
            sb_q45m<QT, NS>(r0, r1, b, m, t, acc, mn);
        }
    }
}
// The lane's B operand base of the minimum-term MMA (ksb.cuh) in a staging buffer's gs rows: token g/2
// for g < 4 (token 0 beyond the group's slots or for g >= 4: those columns are never read), f16 high
// parts for even g, residues for odd g.
__device__ __forceinline__ const uint8_t* min_operand(const uint8_t* gs_rows, int K, int mc) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    int tok = g >> 1;
    if (g >= 4 || tok >= mc) tok = 0;
    return gs_rows + (size_t)tok * xf_gs_bytes(K) + 16 + (g & 1) * 16 + 4 * t;
}
// Rows 2g, 2g+1 of a tile staged with a row stride (lead: bytes before row 0)
__device__ __forceinline__ RowsAny rows_pair(const uint8_t* tile, int stride) {
    const int g = (threadIdx.x & 31) >> 2;
    const uint8_t* r0 = tile + (size_t)(2 * g) * stride;
    return RowsAny{{r0, r0 + stride}};
}
// A gate/up tile (16 rows of rb bytes). Split copies: MMA row g takes row p(g) = g/2 + 8 (g & 1), row
// g+8 takes p(g) + 4, so each half-warp's four rows start on two different bank offsets. Span copies:
// rows 2g, 2g+1 behind the lead bytes.
__device__ __forceinline__ RowsAny rows_gu(const uint8_t* slot, size_t rb, uint32_t lead) {
    const int g = (threadIdx.x & 31) >> 2;
    if (split8(rb)) {
        const int p = (g >> 1) + ((g & 1) ? 8 : 0);
        const uint8_t* hi = slot + split8_off(rb);
        const uint8_t* r0 = (g & 1) ? hi + (size_t)(g >> 1) * rb : slot + (size_t)(g >> 1) * rb;
        (void)p;
        return RowsAny{{r0, r0 + 4 * rb}};
    }
    const uint8_t* r0 = slot + lead + (size_t)(2 * g) * rb;
    return RowsAny{{r0, r0 + rb}};
}
// Tile row held by MMA row g (i = 0) or g+8 (i = 1) of a gate/up tile
__device__ __forceinline__ int gu_row(size_t rb, int g, int i) {
    if (split8(rb)) return (g >> 1) + ((g & 1) ? 8 : 0) + 4 * i;
    return 2 * g + i;
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// routing, grouping and activation prep
// ------------------------------------------------------------------------------------------------
// Orderable key of a float: a larger float has a larger key; only one NaN pattern maps to 0, which is
// reserved for "no entry".
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
// Top-k of one token by the reference's ranking (qwen3moe.cpp:1012-1020): r = expf(l - max) computed as
// the correctly rounded exponential of the fp32 difference, order (r desc, index asc), weights r / sum
// of the k r in rank order. Lane j < k returns the j-th expert and its weight.
//
// exp is monotone, so the top k by r are the top k by d = l - max unless entries of different d round
// to the same r. Candidates are therefore ranked by (d desc, index asc) without exponentials; if any
// other entry lies within 2^-20 of the k-th d (it could round to the same r) or the k-th r is below
// 2^-100 (where rounding groups wider ranges), every entry's r is computed and ranked instead. Otherwise
// the k candidates take one exponential each (one lane each) and are re-sorted by (r desc, index asc),
// which only reorders runs of equal r. rk: 64 words of shared scratch of this warp.
template <int PER>
__device__ void route_token(const float* __restrict__ lg, int E, int K, int lane, uint32_t* rk, int& out_e,
                            float& out_w) {
    float d[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int e = lane + 32 * i;
        d[i] = e < E ? __ldg(lg + e) : -INFINITY;
        mx = fmaxf(mx, d[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    uint32_t key[PER];
#pragma unroll
    for (int i = 0; i < PER; i++) {
        d[i] = d[i] - mx;  // the CPU's fp32 difference
        key[i] = (lane + 32 * i) < E ? fkey(d[i]) : 0u;
    }
    // (d desc, index asc) top k; lane j keeps the j-th (d, e)
    float cd = 0.f, dk = 0.f;
    int ce = 0;
    for (int k = 0; k < K; k++) {
        uint32_t lb = 0;
        int li = 0;
#pragma unroll
        for (int i = 0; i < PER; i++)
            if (key[i] > lb) {
                lb = key[i];
                li = i;
            }
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, lb);
        const uint32_t emin = __reduce_min_sync(0xffffffffu, lb == kmax ? (uint32_t)(lane + 32 * li) : 0xffffffffu);
        float dsel = 0.f;
#pragma unroll
        for (int i = 0; i < PER; i++)
            if ((int)(emin & 31) == lane && i == (int)(emin >> 5)) {
                dsel = d[i];
                key[i] = 0u;
            }
        dsel = __shfl_sync(0xffffffffu, dsel, (int)(emin & 31));
        if (lane == k) {
            cd = dsel;
            ce = (int)emin;
        }
        dk = dsel;
    }
    const float rK = (float)exp((double)dk);
    bool near = false;
#pragma unroll
    for (int i = 0; i < PER; i++) near |= key[i] != 0u && d[i] >= dk - 9.5367431640625e-07f;  // 2^-20
    if (!__any_sync(0xffffffffu, near) && rK >= 7.888609052210118e-31f) {  // 2^-100
        // one exponential per candidate, then rank (r desc, index asc) among the k
        const float r = lane < K ? (float)exp((double)cd) : -1.0f;
        int rank = 0;
        for (int j = 0; j < K; j++) {
            const float rj = __shfl_sync(0xffffffffu, r, j);
            const int ej = __shfl_sync(0xffffffffu, ce, j);
            rank += (rj > r) || (rj == r && ej < ce);
        }
        if (lane < K) {
            rk[2 * rank] = __float_as_uint(r);
            rk[2 * rank + 1] = (uint32_t)ce;
        }
    } else {
        // every entry's r, then k rounds of (r desc, index asc)
        uint32_t* rkey = key;  // the logit keys are spent
#pragma unroll
        for (int i = 0; i < PER; i++)
            rkey[i] = (lane + 32 * i) < E ? __float_as_uint((float)exp((double)d[i])) + 1u : 0u;
        for (int k = 0; k < K; k++) {
            uint32_t lb = 0;
            int li = 0;
#pragma unroll
            for (int i = 0; i < PER; i++)
                if (rkey[i] > lb) {
                    lb = rkey[i];
                    li = i;
                }
            const uint32_t kmax = __reduce_max_sync(0xffffffffu, lb);
            const uint32_t emin = __reduce_min_sync(0xffffffffu, lb == kmax ? (uint32_t)(lane + 32 * li) : 0xffffffffu);
#pragma unroll
            for (int i = 0; i < PER; i++)
                if ((int)(emin & 31) == lane && i == (int)(emin >> 5)) rkey[i] = 0u;
            if (lane == 0) {
                rk[2 * k] = kmax - 1u;
                rk[2 * k + 1] = emin;
            }
        }
    }
    __syncwarp();
    float tot = 0.f;
    for (int k = 0; k < K; k++) tot += __uint_as_float(rk[2 * k]);  // rank-order sum, identical on every lane
    if (lane < K) {
        out_e = (int)rk[2 * lane + 1];
        out_w = __fdiv_rn(__uint_as_float(rk[2 * lane]), tot);
    }
    __syncwarp();
}

// Shared-memory views of one block's routing of T <= MOE_TMAX tokens (E <= MAX_EXPERTS experts).
constexpr int RT_TEAMS = 4;  // tokens ranked at once by a routing block (128 threads each)
// 32-bit words of one token group's ranking scratch (spl teams per token; see route_block)
__host__ __device__ constexpr int rt_group_words(int E, int spl) {
    return 2 * ((E + 7) & ~7) + (spl > 1 ? spl * ((E + 7) & ~7) : 0) + 72;
}
__host__ __device__ constexpr int rt_max(int a, int b) { return a > b ? a : b; }
// ranking scratch: RT_TEAMS single-team groups or one group of RT_TEAMS teams, or 64 words per warp of
// route_token (k_moe_route)
__host__ __device__ constexpr int rt_scr_words(int E) {
    return rt_max(rt_max(RT_TEAMS * rt_group_words(E, 1), rt_group_words(E, RT_TEAMS)), (ROUTE_NT / 32 + 2) * 64);
}
static_assert(RT_TEAMS == 4, "route_block's team split");
static_assert(ROUTE_NT >= MAX_EXPERTS && ROUTE_NT % 128 == 0, "route_block: one thread per expert");
static_assert((NWC_GU + 1) * 32 >= MAX_EXPERTS, "route_block in the gate/up kernel: one thread per expert");
struct RouteSm {
    int *cnt, *off, *goff;        // [E] slots, slot offset, group offset per expert
    unsigned long long* mask;     // [E] tokens routed to the expert
    int* s_ids;                   // [T*K] routed experts, rank order
    float* s_w;                   // [T*K] their weights
    float* scr;                   // [rt_scr_words(E)] ranking scratch (16-byte aligned)
    int* g_info;                  // optional [G][4]: expert, first slot, slots, unused; G <= T*K
    int* g_tok;                   // optional [G][MU]
    const uint8_t** g_w;          // optional [G][3]: gate, up and down matrices of the group's expert
    const uint8_t** tab;          // optional [3][E]: the gate, up and down matrix of every expert
    int* G;                       // number of groups
};
// bytes of a RouteSm for E experts and TK = T*K slots; with_groups adds the shared-memory group list
// and the experts' matrix table
__host__ __device__ constexpr size_t route_sm_bytes(int E, int TK, bool with_groups) {
    return (size_t)E * (8 + 4 + 4 + 4) + (size_t)TK * 8 + 16 + (size_t)rt_scr_words(E) * 4 + 16 +
           (with_groups ? 16 + (size_t)TK * (24 + 16 + 4 * MU) + (size_t)E * 24 : 0);  // 16: alignment
}
__device__ inline RouteSm route_sm_carve(uint8_t* p, int E, int TK, bool with_groups) {
    RouteSm r;
    r.mask = reinterpret_cast<unsigned long long*>(p);  // 8-byte aligned at the start
    p += (size_t)E * 8;
    r.cnt = reinterpret_cast<int*>(p);
    r.off = r.cnt + E;
    r.goff = r.off + E;
    r.s_ids = r.goff + E;
    r.s_w = reinterpret_cast<float*>(r.s_ids + TK);
    r.scr = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(r.s_w + TK) + 15) & ~(uintptr_t)15);
    r.G = reinterpret_cast<int*>(r.scr + rt_scr_words(E));
    p = reinterpret_cast<uint8_t*>(r.G + 4);  // 16 bytes
    p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 15) & ~(uintptr_t)15);
    if (with_groups) {
        r.g_w = reinterpret_cast<const uint8_t**>(p);
        r.g_info = reinterpret_cast<int*>(p + (size_t)TK * 24);
        r.g_tok = r.g_info + 4 * TK;
        r.tab = reinterpret_cast<const uint8_t**>(r.g_tok + MU * TK);  // 8-byte aligned: TK * (40 + 4 MU)
    } else {
        r.g_w = nullptr;
        r.g_info = nullptr;
        r.g_tok = nullptr;
        r.tab = nullptr;
    }
    return r;
}

// The routing of the T tokens by every thread of the block (qwen3moe.cpp:1009-1029): top-k per token,
// per-expert counts and token masks, scans, work groups of up to MU slots per expert (expert ascending),
// slot maps. With `global` the results go to a.rw (routing outputs, groups and slot maps for the later
// kernels); with r.g_info the group list also stays in shared memory. TEAMS: a few tokens, each ranked
// by a team of 128 threads (latency); otherwise one warp per token (route_token; throughput).
// Requires blockDim.x >= E (one thread per expert in the scans).
// Levels K0..K1 (powers of two) of the bitonic sorting network over 32 keys, one per lane. After level k
// every block of k lanes is sorted, descending when (lane & k) == 0, ascending otherwise; after level 32
// the warp is sorted descending (lane i holds the i-th largest).
template <int K0, int K1>
__device__ __forceinline__ uint64_t warp_bitonic(uint64_t key) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = K0; k <= K1; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const uint64_t o = __shfl_xor_sync(0xffffffffu, key, j);
            const bool desc = (lane & k) == 0, lower = (lane & j) == 0;
            key = (lower == desc) ? (key > o ? key : o) : (key < o ? key : o);
        }
    }
    return key;
}
// 32 keys sorted descending across the warp; lane i returns the i-th largest.
__device__ __forceinline__ uint64_t warp_sort_desc(uint64_t key) { return warp_bitonic<2, 32>(key); }
// Four descending runs of 8 keys (one per warp of a team) in the lane layout the network has after level
// 8: run w in lanes 8w..8w+7, reversed (ascending) for odd w. Levels 16 and 32 finish the sort: the
// result is the same sorted sequence a full sort of the 32 keys gives.
__device__ __forceinline__ int run8_slot(int w, int i) { return 8 * w + ((w & 1) ? 7 - i : i); }
__device__ __forceinline__ uint64_t warp_merge_runs8(uint64_t key) { return warp_bitonic<16, 32>(key); }

// The routing of one token (E <= 128, k <= 8) by the block's first four warps, and its work list: the
// sorting-team ranking (see route_block), then the first warp sorts its k picks by expert id, so that
// pick i is slot i, group i (one slot) and the token's i-th slot in expert order. With `global` the
// routing (rank order), groups, slot maps, offsets and active list go to a.rw as route_block writes them.
// All threads call it; the results in r (group list) are visible after the caller's __syncthreads.
__device__ void route_one(const MoeArgs& a, RouteSm r, bool global) {
    const int E = a.n_expert, K = a.n_used, tid = threadIdx.x, lane = tid & 31, wt = tid >> 5;
    float* wmax = r.scr;  // [4] warp maxima, a NaN flag, 32 candidate keys, 4 mask words
    int* nan_flag = reinterpret_cast<int*>(wmax + 4);
    uint64_t* cand = reinterpret_cast<uint64_t*>(wmax + 8);
    uint32_t* selm = reinterpret_cast<uint32_t*>(wmax + 8 + 64);
    if (tid < 128) {
        auto team_sync = []() { asm volatile("bar.sync 1, 128;" ::: "memory"); };
        const float l = tid < E ? __ldg(a.logits + tid) : -INFINITY;
        float mx = l;
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) wmax[wt] = mx;
        if (tid == 0) *nan_flag = 0;
        if (tid < 4) selm[tid] = 0u;
        team_sync();
        mx = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
        const float rv = (float)exp((double)(l - mx));
        const bool isnan_e = tid < E && rv != rv;
        uint64_t key = tid < E && !isnan_e ? ((uint64_t)__float_as_uint(rv) << 32) | (uint32_t)~(uint32_t)tid : 0ull;
        key = warp_sort_desc(key);
        if (lane < 8) cand[run8_slot(wt, lane)] = key;
        if (__any_sync(0xffffffffu, isnan_e) && lane == 0) *nan_flag = 1;
        team_sync();
        if (wt == 0) {
            key = warp_merge_runs8(cand[lane]);
            const float rk = __uint_as_float((uint32_t)(key >> 32));
            float tot = 0.f;
            for (int k = 0; k < K; k++) tot += __shfl_sync(0xffffffffu, rk, k);  // rank-order sum
            int my_e = *nan_flag || key == 0ull ? -1 : (int)~(uint32_t)key;
            const float my_w = __fdiv_rn(rk, tot);
            if (lane < K) {
                if (my_e < 0 || my_e >= E) {  // only reachable with NaN logits
                    if (global) set_flag(a.status, ST_BAD_INDEX);
                    my_e = 0;
                }
                r.s_ids[lane] = my_e;
                r.s_w[lane] = my_w;
                if (global) {
                    a.rw.ids[lane] = my_e;
                    a.rw.wts[lane] = my_w;
                }
            }
            // the k picks in ascending expert order (id + 1 in the high word, above the empty lanes' 0; the
            // weight travels in the low word)
            uint64_t k2 = lane < K ? ((uint64_t)(uint32_t)(my_e + 1) << 32) | __float_as_uint(my_w) : 0ull;
            // lanes 0..7 hold every key (the others 0): levels 2..8 sort them descending, so pick i of the
            // ascending order sits in lane K - 1 - i
            k2 = warp_bitonic<2, 8>(k2);
            const int i = K - 1 - lane;
            if (lane < K) {
                const int e = (int)(k2 >> 32) - 1;
                const float w = __uint_as_float((uint32_t)k2);
                const uint8_t* wg = r.tab ? r.tab[e] : a.gate[e];
                const uint8_t* wu = r.tab ? r.tab[E + e] : a.up[e];
                const uint8_t* wd = r.tab ? r.tab[2 * E + e] : a.down[e];
                r.off[e] = i;
                r.goff[e] = i;
                atomicOr(&selm[e >> 5], 1u << (e & 31));
                if (r.g_info) {
                    r.g_info[4 * i] = e;
                    r.g_info[4 * i + 1] = i;
                    r.g_info[4 * i + 2] = 1;
                    for (int k = 0; k < MU; k++) r.g_tok[MU * i + k] = 0;
                    r.g_w[3 * i] = wg;
                    r.g_w[3 * i + 1] = wu;
                    r.g_w[3 * i + 2] = wd;
                }
                if (global) {
                    GroupRec& g = a.rw.groups[i];
                    g.w[0] = wg;
                    g.w[1] = wu;
                    g.w[2] = wd;
                    g.e = e;
                    g.s0 = i;
                    g.mc = 1;
                    for (int k = 0; k < MU; k++) g.tok[k] = 0;
                    a.rw.slot_token[i] = 0;
                    a.rw.slot_w[i] = w;
                    a.rw.token_slots[i] = i;
                    a.rw.active[1 + i] = e;
                }
            }
            if (lane == 0) {
                *r.G = K;
                if (global) {
                    a.rw.ngroups[0] = K;
                    a.rw.active[0] = K;
                    a.rw.offsets[E] = K;
                }
            }
        }
    }
    __syncthreads();
    if (global)  // slot offsets: the picks below each expert id
        for (int e = tid; e < E; e += blockDim.x) {
            int c = __popc(selm[e >> 5] & ((1u << (e & 31)) - 1u));
            for (int w = 0; w < (e >> 5); w++) c += __popc(selm[w]);
            a.rw.offsets[e] = c;
        }
}

// GIVEN: the experts of every slot come from a.given (weight 1, entries < 0 absent) instead of a top-k.
template <bool TEAMS, int GS = MU, bool GIVEN = false>
__device__ void route_block(const MoeArgs& a, RouteSm r, bool global) {
    static_assert(GS >= MU && GS <= 32, "group size");
    const int T = a.T, E = a.n_expert, K = a.n_used, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, nwarp = blockDim.x >> 5;
    if constexpr (TEAMS) {
        if (T == 1 && E <= 128 && K <= 8) {  // one token (a decode step): no counts, scans or scatter
            route_one(a, r, global);
            return;
        }
    }
    for (int i = tid; i < E; i += blockDim.x) {
        r.cnt[i] = 0;
        r.mask[i] = 0ull;
    }
    __syncthreads();
    // ---- softmax numerators, top-k, renormalisation (qwen3moe.cpp:1012-1022). A team of 128 threads
    // (4 warps, named barrier 1 + team) ranks one token: every entry's r = (float)exp((double)(l - max))
    // with the difference in fp32 as on the CPU, then each entry's rank under the comparator (r desc,
    // index asc) of std::partial_sort by counting the entries ahead of it; ranks < K are the top k, summed
    // in rank order for the weights r / sum.
    const int nteam = nwarp >= 16 ? 4 : nwarp >= 8 ? 2 : 1, team = warp >> 2, tt = tid & 127;  // RT_TEAMS = 4
    if constexpr (!TEAMS) {
        for (int t = warp; t < T; t += nwarp) {
            int my_e = 0;
            float my_w = 0.f;
            uint32_t* rk = reinterpret_cast<uint32_t*>(r.scr) + warp * 64;
            if constexpr (GIVEN) {  // assigned experts (expert-parallel receiver): weight 1, no ranking
                if (lane < K) {
                    my_e = __ldg(a.given + (size_t)t * K + lane);
                    my_w = 1.0f;
                }
            } else if (E <= 128) route_token<4>(a.logits + (size_t)t * E, E, K, lane, rk, my_e, my_w);
            else if (E <= 256) route_token<8>(a.logits + (size_t)t * E, E, K, lane, rk, my_e, my_w);
            else route_token<16>(a.logits + (size_t)t * E, E, K, lane, rk, my_e, my_w);
            if (GIVEN && lane < K && my_e < 0) {  // an absent slot (padding row of the receiver): no slot
                r.s_ids[t * K + lane] = -1;
                if (global) a.rw.ids[(size_t)t * K + lane] = -1;
            } else if (lane < K) {
                if (my_e < 0 || my_e >= E) {  // NaN logits or a given id out of range
                    if (global) set_flag(a.status, ST_BAD_INDEX);
                    my_e = 0;
                }
                r.s_ids[t * K + lane] = my_e;
                r.s_w[t * K + lane] = my_w;
                if (global) {
                    a.rw.ids[(size_t)t * K + lane] = my_e;
                    a.rw.wts[(size_t)t * K + lane] = my_w;
                }
                atomicAdd(&r.cnt[my_e], 1);
                atomicOr(&r.mask[my_e], 1ull << t);
            }
        }
    } else if (team < nteam && E <= 128 && K <= 8) {
        // Sorting teams (E <= 128, k <= 8; the Qwen3 shapes): one team of 128 threads per token, one entry
        // per thread. Key of entry e: (bits of r) << 32 | ~e, so that a larger key ranks first under
        // (r desc, index asc) (r >= 0: its bits order as the floats do); NaN and absent entries key 0.
        // Each warp sorts its 32 keys (bitonic, descending), the team's four top-8 lists are merged by the
        // team's first warp (the network's last two levels): its lanes 0..k-1 hold the top k in rank order.
        float* wmax = r.scr + (size_t)team * 80;  // [4] warp maxima, a NaN flag, then 32 candidate keys
        int* nan_flag = reinterpret_cast<int*>(wmax + 4);
        uint64_t* cand = reinterpret_cast<uint64_t*>(wmax + 8);
        const int wt = tt >> 5;  // warp within the team
        auto team_sync = [&]() { asm volatile("bar.sync %0, 128;" ::"r"(1 + team) : "memory"); };
        for (int t = team; t < T; t += nteam) {
            const float l = tt < E ? __ldg(a.logits + (size_t)t * E + tt) : -INFINITY;
            float mx = l;
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0) wmax[wt] = mx;
            if (tt == 0) *nan_flag = 0;
            team_sync();
            mx = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
            const float rv = (float)exp((double)(l - mx));
            const bool isnan_e = tt < E && rv != rv;
            uint64_t key = tt < E && !isnan_e ? ((uint64_t)__float_as_uint(rv) << 32) | (uint32_t)~(uint32_t)tt : 0ull;
            key = warp_sort_desc(key);
            if (lane < 8) cand[run8_slot(wt, lane)] = key;
            if (__any_sync(0xffffffffu, isnan_e) && lane == 0) *nan_flag = 1;
            team_sync();
            if (wt == 0) {
                key = warp_merge_runs8(cand[lane]);
                const float rk = __uint_as_float((uint32_t)(key >> 32));
                float tot = 0.f;
                for (int k = 0; k < K; k++) tot += __shfl_sync(0xffffffffu, rk, k);  // rank-order sum
                if (lane < K) {
                    int my_e = *nan_flag || key == 0ull ? -1 : (int)~(uint32_t)key;
                    const float my_w = __fdiv_rn(rk, tot);
                    if (my_e < 0 || my_e >= E) {  // only reachable with NaN logits
                        if (global) set_flag(a.status, ST_BAD_INDEX);
                        my_e = 0;
                    }
                    r.s_ids[t * K + lane] = my_e;
                    r.s_w[t * K + lane] = my_w;
                    if (global) {
                        a.rw.ids[(size_t)t * K + lane] = my_e;
                        a.rw.wts[(size_t)t * K + lane] = my_w;
                    }
                    atomicAdd(&r.cnt[my_e], 1);
                    atomicOr(&r.mask[my_e], 1ull << t);
                }
            }
            team_sync();  // the scratch is reused by the team's next token
        }
    } else if (team < nteam) {
        // One token per group of spl teams: spl = nteam for a single token (the decode case), else 1.
        // Group scratch: [E8] 64-bit keys, [spl][E8] partial ranks (spl > 1), [4] warp maxima, [32] r and
        // [32] ids by rank, a NaN flag. Key of entry e: (bits of r) << 32 | ~e, so that a larger key ranks
        // first under (r desc, index asc) (r >= 0: its bits order as the floats do).
        const int spl = T == 1 ? nteam : 1, ngrp = nteam / spl, grp = team / spl, q = team % spl;
        const int E8 = (E + 7) & ~7;
        uint64_t* keys = reinterpret_cast<uint64_t*>(r.scr + (size_t)grp * rt_group_words(E, spl));
        int* part = reinterpret_cast<int*>(keys + E8);
        float* wmax = reinterpret_cast<float*>(part + (spl > 1 ? spl * E8 : 0));
        float* sel_r = wmax + 4;
        int* sel_e = reinterpret_cast<int*>(sel_r + 32);
        int* nan_flag = sel_e + 32;
        auto team_sync = [&]() { asm volatile("bar.sync %0, 128;" ::"r"(1 + team) : "memory"); };
        auto group_sync = [&]() {
            if (spl == 1) team_sync();
            else asm volatile("bar.sync %0, %1;" ::"r"(5 + grp), "r"(128 * spl) : "memory");
        };
        const int ept = (E + 127) >> 7;  // entries per thread: e = tt + 128 j
        for (int t0 = 0; t0 < T; t0 += ngrp) {
            const int t = t0 + grp;
            if (t >= T) break;  // whole groups
            bool nanv[4] = {false, false, false, false};
            if (q == 0) {  // the group's first team: numerators and keys
                const float* lg = a.logits + (size_t)t * E;
                float l[4];
                float mx = -INFINITY;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int e = tt + 128 * j;
                    l[j] = j < ept && e < E ? __ldg(lg + e) : -INFINITY;
                    mx = fmaxf(mx, l[j]);
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                if (lane == 0) wmax[tt >> 5] = mx;
                if (tt < 32) sel_e[tt] = -1;
                if (tt == 0) *nan_flag = 0;
                team_sync();
                mx = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int e = tt + 128 * j;
                    if (j < ept && e < E8) {
                        uint64_t k = 0;  // padding entries and NaN: below every real key
                        if (e < E) {
                            const float rv = (float)exp((double)(l[j] - mx));
                            if (rv != rv) {
                                nanv[j] = true;
                                *nan_flag = 1;
                            } else {
                                k = ((uint64_t)__float_as_uint(rv) << 32) | (uint32_t)~(uint32_t)e;
                            }
                        }
                        keys[e] = k;
                    }
                }
            }
            group_sync();
            // ranks: entry e's count of larger keys among this team's share [q E8 / spl, (q+1) E8 / spl)
            const int f0 = q * (E8 / spl), f1 = f0 + E8 / spl;
            int rk[4] = {0, 0, 0, 0};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int e = tt + 128 * j;
                if (j < ept && e < E) {
                    const uint64_t me = keys[e];
                    int c0 = 0, c1 = 0;
#pragma unroll 4
                    for (int f = f0; f < f1; f += 2) {
                        const ulonglong2 kk = *reinterpret_cast<const ulonglong2*>(keys + f);
                        c0 += kk.x > me;
                        c1 += kk.y > me;
                    }
                    rk[j] = c0 + c1;
                    if (spl > 1) part[q * E8 + e] = rk[j];
                }
            }
            if (spl > 1) group_sync();
            if (q == 0) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int e = tt + 128 * j;
                    if (j < ept && e < E && !nanv[j]) {
                        int rank = rk[j];
                        for (int qq = 1; qq < spl; qq++) rank += part[qq * E8 + e];
                        if (rank < K) {
                            sel_r[rank] = __uint_as_float((uint32_t)(keys[e] >> 32));
                            sel_e[rank] = e;
                        }
                    }
                }
                team_sync();
                if (tt < K) {
                    float tot = 0.f;
                    for (int k = 0; k < K; k++) tot += sel_r[k];  // rank-order sum
                    int my_e = *nan_flag ? -1 : sel_e[tt];
                    const float my_w = __fdiv_rn(sel_r[tt], tot);
                    if (my_e < 0 || my_e >= E) {  // only reachable with NaN logits
                        if (global) set_flag(a.status, ST_BAD_INDEX);
                        my_e = 0;
                    }
                    r.s_ids[t * K + tt] = my_e;
                    r.s_w[t * K + tt] = my_w;
                    if (global) {
                        a.rw.ids[(size_t)t * K + tt] = my_e;
                        a.rw.wts[(size_t)t * K + tt] = my_w;
                    }
                    atomicAdd(&r.cnt[my_e], 1);
                    atomicOr(&r.mask[my_e], 1ull << t);
                }
            }
            group_sync();  // the scratch is reused by the group's next token
        }
    }
    __syncthreads();
    // ---- exclusive scans over the experts (thread e: slots, groups of ceil(count / MU), active flag);
    // E <= blockDim.x
    {
        int* wtot = reinterpret_cast<int*>(r.scr);  // [3][32] per-warp totals (the ranking scratch is free)
        const int e = tid;
        const int c = e < E ? r.cnt[e] : 0, g = (c + GS - 1) / GS, ac = c > 0;
        int cx = c, gx = g, ax = ac;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, cx, o), gv = __shfl_up_sync(0xffffffffu, gx, o),
                      av = __shfl_up_sync(0xffffffffu, ax, o);
            if (lane >= o) {
                cx += v;
                gx += gv;
                ax += av;
            }
        }
        if (lane == 31) {
            wtot[warp] = cx;
            wtot[32 + warp] = gx;
            wtot[64 + warp] = ax;
        }
        __syncthreads();
        int cb = 0, gb = 0, ab = 0;
        for (int w = 0; w < warp; w++) {
            cb += wtot[w];
            gb += wtot[32 + w];
            ab += wtot[64 + w];
        }
        if (e < E) {
            r.off[e] = cb + cx - c;
            r.goff[e] = gb + gx - g;
            if (global) {
                a.rw.offsets[e] = cb + cx - c;
                if (ac) a.rw.active[1 + ab + ax - 1] = e;
            }
        }
        if (e == E - 1) {
            *r.G = gb + gx;
            if (global) {
                a.rw.offsets[E] = cb + cx;
                a.rw.active[0] = ab + ax;
                a.rw.ngroups[0] = gb + gx;
            }
        }
    }
    __syncthreads();
    // ---- work list: groups of up to MU consecutive slots of one expert, expert ascending. Expert threads
    // write each group's expert, first slot and size (and zero token entries past the size); the
    // (token, k) threads below fill in the tokens.
    for (int e = tid; e < E; e += blockDim.x) {
        const int c = r.cnt[e];
        if (c == 0) continue;
        const uint8_t* wg = r.tab ? r.tab[e] : a.gate[e];
        const uint8_t* wu = r.tab ? r.tab[E + e] : a.up[e];
        const uint8_t* wd = r.tab ? r.tab[2 * E + e] : a.down[e];
        for (int j = 0; j * GS < c; j++) {
            const int gi = r.goff[e] + j, s0 = r.off[e] + j * GS, mc = min(GS, c - j * GS);
            if (global) {
                GroupRec& g = a.rw.groups[gi];
                g.w[0] = wg;
                g.w[1] = wu;
                g.w[2] = wd;
                g.e = e;
                g.s0 = s0;
                g.mc = mc;
                if (GS == MU)  // wider groups take their tokens from the slot map
                    for (int k = mc; k < MU; k++) g.tok[k] = 0;
            }
            if (r.g_info) {
                r.g_info[4 * gi] = e;
                r.g_info[4 * gi + 1] = s0;
                r.g_info[4 * gi + 2] = mc;
                for (int k = mc; k < MU; k++) r.g_tok[MU * gi + k] = 0;
                r.g_w[3 * gi] = wg;
                r.g_w[3 * gi + 1] = wu;
                r.g_w[3 * gi + 2] = wd;
            }
        }
    }
    // ---- one thread per (token, k): the slot is offset[e] + the earlier tokens routed to e (stable
    // scatter); its group and place in the group follow; the token's slots in ascending order (= expert
    // order) by rank among its k experts
    for (int i = tid; i < T * K; i += blockDim.x) {
        const int t = i / K;
        const int e = r.s_ids[i];
        if (GIVEN && e < 0) continue;  // absent slot
        const int pos = __popcll(r.mask[e] & ((1ull << t) - 1ull)), sl = r.off[e] + pos;
        const int gi = r.goff[e] + pos / GS;
        if (r.g_tok) r.g_tok[MU * gi + pos % GS] = t;
        if (global) {
            if (GS == MU) a.rw.groups[gi].tok[pos % MU] = t;
            a.rw.slot_token[sl] = t;
            a.rw.slot_w[sl] = r.s_w[i];
            int rank = 0;
            for (int j = 0; j < K; j++) rank += r.s_ids[t * K + j] < e;
            a.rw.token_slots[(size_t)t * K + rank] = sl;
        }
    }
}

template <bool GIVEN, int GS>
__global__ void __launch_bounds__(ROUTE_NT) k_moe_route(MoeArgs a) {
    pdl_wait();     // logits and activations come from the previous grids
    pdl_trigger();
    if (blockIdx.x > 0) {  // activation prep of token blockIdx.x - 1
        __shared__ float red[33];
        const int row = blockIdx.x - 1;
        prep_row(a.xn + (size_t)row * a.D, a.D, const_cast<uint2*>(a.xf.frag) + (size_t)row * (a.D >> 5) * 12,
                 const_cast<float*>(a.xf.sum) + (size_t)row * ((a.D >> 4) + XF_SUM_PAD),
                 const_cast<uint8_t*>(a.xf.gs) + (size_t)row * xf_gs_bytes(a.D), red);
        return;
    }
    __shared__ __align__(16) uint8_t rsm[route_sm_bytes(MAX_EXPERTS, MOE_TMAX * 32, false) + 16];
    route_block<false, GS, GIVEN>(a, route_sm_carve(rsm, a.n_expert, a.T * a.n_used, false), true);
}

// ------------------------------------------------------------------------------------------------
// gate + up + SiLU*mul
// ------------------------------------------------------------------------------------------------
template <int QG, int QU, int G>
__global__ void __launch_bounds__((NWC_GU + 1) * 32, 1) k_moe_gateup(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int D = a.D, FF = a.FF, nsb = D >> 8, NRB = FF >> 4, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int TK = a.T * a.n_used;
    const bool fused = G == MU && a.fused_route;  // routing inside (small batches; groups of MU slots)
    const Plan pl = gateup_plan(D, a.gate_rb, a.up_rb, fused ? route_sm_bytes(a.n_expert, TK, true) : 0, G);
    const int S = pl.S;
    uint64_t* full = reinterpret_cast<uint64_t*>(sm);
    uint64_t* empty = full + 4;
    uint64_t* done = full + 8;  // per stage: every consumer warp has stored its partial results
    int4* info = reinterpret_cast<int4*>(sm + pl.info_off);
    __shared__ int abort_flag;
    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NWC_GU);
            mbar_init(&done[s], NWC_GU);
        }
        abort_flag = 0;
        mbar_fence_init();
    }
    RouteSm rt{};
    if (fused) {  // the experts' matrix table does not depend on earlier grids
        rt = route_sm_carve(sm + pl.extra_off, a.n_expert, TK, true);
        const int E = a.n_expert;
        for (int i = tid; i < 3 * E; i += blockDim.x) rt.tab[i] = i < E ? a.gate[i] : i < 2 * E ? a.up[i - E] : a.down[i - 2 * E];
    }
    __syncthreads();
    pdl_wait();  // routing results (or the logits) and the XF of the tokens come from the previous grids
    pdl_trigger();
    // small batches: every CTA routes the tokens itself into shared memory (CTA 0 also publishes the
    // routing, groups and slot maps for the down kernel and the combine)
    if constexpr (G == MU) {
        if (fused) {
            route_block<true>(a, rt, blockIdx.x == 0);
            __syncthreads();
        }
    }
    const int NG = fused ? *rt.G : a.rw.ngroups[0];
    auto group = [&](int gi) {
        if (!fused) return a.rw.groups[gi];
        GroupRec g{};
        g.w[0] = rt.g_w[3 * gi];
        g.w[1] = rt.g_w[3 * gi + 1];
        g.w[2] = rt.g_w[3 * gi + 2];
        g.e = rt.g_info[4 * gi];
        g.s0 = rt.g_info[4 * gi + 1];
        g.mc = rt.g_info[4 * gi + 2];
#pragma unroll
        for (int k = 0; k < MU; k++) g.tok[k] = rt.g_tok[MU * gi + k];
        return g;
    };
    const int nunits = NG * NRB;
    const int u0 = (int)((long long)blockIdx.x * nunits / gridDim.x), u1 = (int)((long long)(blockIdx.x + 1) * nunits / gridDim.x);
    const size_t rbg = a.gate_rb, rbu = a.up_rb, up_at = gu_slot(rbg);
    const Rows Lg = rows_of(rbg), Lu = rows_of(rbu);  // span layouts (rows that are not 16-byte multiples)

    if (warp == NWC_GU) {  // ---------------- producer
        if (lane != 0) return;
        int cur = -1, xb = 1, i = 0;
        GroupRec rec{}, nxt{};
        if (u0 < u1) nxt = group(u0 / NRB);
        for (int u = u0; u < u1; u++, i++) {
            const int s = i % S;
            if (i >= S && !mbar_wait_bounded(&empty[s], (uint32_t)(i / S - 1) & 1u)) {
                set_flag(a.status, ST_WAIT_TIMEOUT);
                atomicExch(&abort_flag, 1);
                break;
            }
            if (*(volatile int*)&abort_flag) break;
            const int gi = u / NRB, rb = u - gi * NRB, r0 = 16 * rb;
            const bool fresh = gi != cur;
            if (fresh) {
                rec = nxt;
                cur = gi;
                xb ^= 1;
                if ((gi + 1) * NRB < u1) nxt = group(gi + 1);  // the next group's record, ahead of use
            }
            const bool ok = al16(rec.w[0]) && al16(rec.w[1]);
            if (!ok) set_flag(a.status, ST_BAD_ARG);
            uint8_t* stage = sm + pl.stage_off + (size_t)s * pl.stage_bytes;
            const uint32_t lg = (!split8(rbg) && ok) ? rows_lead(Lg, rec.w[0], rbg, r0) : 0u;
            const uint32_t lu = (!split8(rbu) && ok) ? rows_lead(Lu, rec.w[1], rbu, r0) : 0u;
            info[s] = make_int4(rb, info_bits(xb, rec.mc, ok, fresh), rec.s0, (int)(lg | (lu << 8)));
            uint32_t bytes = fresh ? (uint32_t)rec.mc * ((uint32_t)D * 3 + (uint32_t)xf_gs_bytes(D)) : 0u;
            if (ok) {
                bytes += split8(rbg) ? (uint32_t)(16 * rbg) : rows_copy_bytes(Lg, rec.w[0], rbg, r0, 16);
                bytes += split8(rbu) ? (uint32_t)(16 * rbu) : rows_copy_bytes(Lu, rec.w[1], rbu, r0, 16);
            }
            mbar_expect_tx(&full[s], bytes);
            if (fresh) {
                int tok[G];
                for (int k = 0; k < rec.mc; k++) tok[k] = G == MU ? rec.tok[k < MU ? k : 0] : a.rw.slot_token[rec.s0 + k];
                xf_issue<G>(a.xf, tok, rec.mc, D, sm + pl.xf_off + (size_t)xb * pl.xfb, &full[s]);
            }
            if (ok) {
                if (split8(rbg)) {
                    tma_load_1d(stage, rec.w[0] + (size_t)r0 * rbg, (uint32_t)(8 * rbg), &full[s]);
                    tma_load_1d(stage + split8_off(rbg), rec.w[0] + (size_t)(r0 + 8) * rbg, (uint32_t)(8 * rbg), &full[s]);
                } else {
                    rows_issue(Lg, rec.w[0], rbg, r0, 16, stage, &full[s]);
                }
                if (split8(rbu)) {
                    tma_load_1d(stage + up_at, rec.w[1] + (size_t)r0 * rbu, (uint32_t)(8 * rbu), &full[s]);
                    tma_load_1d(stage + up_at + split8_off(rbu), rec.w[1] + (size_t)(r0 + 8) * rbu, (uint32_t)(8 * rbu),
                                &full[s]);
                } else {
                    rows_issue(Lu, rec.w[1], rbu, r0, 16, stage + up_at, &full[s]);
                }
            }
        }
        // wait (bounded) until the consumers have released every issued stage, so that no copy is in
        // flight when the CTA retires (after a consumer timeout: drain the copies instead)
        const int issued = i;
        for (int k = (issued > S ? issued - S : 0); k < issued; k++) {
            if (!mbar_wait_bounded(&empty[k % S], (uint32_t)(k / S) & 1u)) {
                drain(full, issued, k, S);
                break;
            }
        }
        return;
    }

    // ---------------- consumers: warp w works on matrix w / 8 (gate, up), super-blocks w % 8 + 8j
    const int mtx = warp >> 3, wsub = warp & 7, g = lane >> 2, t = lane & 3;
    const size_t rbm = mtx ? rbu : rbg;
    const int prow0 = gu_row(rbm, g, 0), prow1 = gu_row(rbm, g, 1);
    int i = 0;
    for (int u = u0; u < u1; u++, i++) {
        const int s = i % S;
        if (!mbar_wait_bounded(&full[s], (uint32_t)(i / S) & 1u)) {
            set_flag(a.status, ST_WAIT_TIMEOUT);
            atomicExch(&abort_flag, 1);
            return;  // the producer drains what it issued
        }
        const int4 in = info[s];
        const int rb = in.x, xb = in.y & 1, mc = (in.y >> 4) & 15, s0 = in.z;
        const uint8_t* xs = sm + pl.xf_off + (size_t)xb * pl.xfb;
        float* part = reinterpret_cast<float*>(sm + pl.part_off) + ((size_t)s * NWC_GU + warp) * 16 * G;
        const uint8_t* stage = sm + pl.stage_off + (size_t)s * pl.stage_bytes;
        for (int st = 0; 2 * st < mc;) {  // column sets: slots 2 st, 2 st + 1 of the group
            const int ms = mc - 2 * st;
            const uint8_t* xg = xs + xs_gs_off(D, G) + (size_t)(2 * st) * xf_gs_bytes(D);
            if (G > MU && ms > 2) {  // sets st, st + 1 over one decode of the weights
                const uint8_t* xg1 = xg + 2 * (size_t)xf_gs_bytes(D);
                float acc[2][4] = {}, mn[2][2] = {};
                if (in.y & 256) {
                    const uint8_t* bq[2] = {BPtr<1>(xs + (size_t)(2 * st) * D * 3, D >> 5, ms).p[0],
                                            BPtr<1>(xs + (size_t)(2 * st + 2) * D * 3, D >> 5, ms - 2).p[0]};
                    const uint8_t* mq[2] = {min_operand(xg, D, ms), min_operand(xg1, D, ms - 2)};
                    if (mtx == 0)
                        block_tasks_m<QG, 2>(rows_gu(stage, rbg, in.w & 255), nsb, wsub, 8, bq, mq, acc, mn);
                    else
                        block_tasks_m<QU, 2>(rows_gu(stage + up_at, rbu, (in.w >> 8) & 255), nsb, wsub, 8, bq, mq, acc, mn);
                }
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    const float a1[1][4] = {{acc[k][0], acc[k][1], acc[k][2], acc[k][3]}};
                    const float ts = t < ms - 2 * k ? *reinterpret_cast<const float*>(xg + (size_t)(2 * k + t) * xf_gs_bytes(D)) : 0.f;
                    warp_values(a1, mn[k], ts, part, prow0, prow1, G, 2 * st + 2 * k);
                }
                st += 2;
                continue;
            }
            float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}}, mn[2] = {0.f, 0.f};
            if (in.y & 256) {
                const BPtr<1> bp(xs + (size_t)(2 * st) * D * 3, D >> 5, ms);
                const uint8_t* mq = min_operand(xg, D, ms);
                if (mtx == 0)
                    block_tasks<QG>(rows_gu(stage, rbg, in.w & 255), nsb, wsub, 8, bp, mq, acc, mn);
                else
                    block_tasks<QU>(rows_gu(stage + up_at, rbu, (in.w >> 8) & 255), nsb, wsub, 8, bp, mq, acc, mn);
            }
            const float ts = t < ms ? *reinterpret_cast<const float*>(xg + (size_t)t * xf_gs_bytes(D)) : 0.f;
            warp_values(acc, mn, ts, part, prow0, prow1, G, 2 * st);
            st++;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&done[s]);
        if (warp == i % NWC_GU) {  // this unit's reducer (round robin): SiLU*mul of the summed partials
            if (!mbar_wait_bounded(&done[s], (uint32_t)(i / S) & 1u)) {
                set_flag(a.status, ST_WAIT_TIMEOUT);
                atomicExch(&abort_flag, 1);
                return;
            }
            const float* P = reinterpret_cast<const float*>(sm + pl.part_off) + (size_t)s * NWC_GU * 16 * G;
            for (int j = lane; j < 16 * G; j += 32) {
                const int r = j / G, tk = j - r * G;
                if (tk < mc) {
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int w = 0; w < 8; w++) {
                        gv += P[(w * 16 + r) * G + tk];
                        uv += P[((8 + w) * 16 + r) * G + tk];
                    }
                    a.h[(size_t)(s0 + tk) * FF + 16 * rb + r] = silu_mul(gv, uv);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// ------------------------------------------------------------------------------------------------
// gate + up + SiLU*mul for small batches (T <= FUSED_ROUTE_TMAX, the decode steps): every CTA routes the
// tokens itself and stages all T tokens' XF rows once (two bulk copies); the 16 consumer warps form
// FS_GROUPS independent pipelines of 4 warps, group q taking the CTA's units q, q + 4, ... from ring
// stage q, so up to four units are computed at once. Within a group, warp k takes matrix k / 2 and the
// super-block subsets ("virtual warps") 4 (k % 2) .. 4 (k % 2) + 3, each subset accumulated and
// recombined exactly as one consumer warp of k_moe_gateup does it, and the group's first warp sums the
// eight subsets per matrix in the same order: per-slot results are bitwise those of k_moe_gateup.
// ------------------------------------------------------------------------------------------------
constexpr int FS_GROUPS = 4;
struct FsPlan {
    size_t info_off, xf_off, xf_gs_off, part_off, stage_off, stage_bytes, extra_off, total;
};
__host__ __device__ inline FsPlan gateup_fs_plan(int T, int D, size_t rbg, size_t rbu, size_t route_bytes) {
    FsPlan p;
    p.info_off = 128;
    p.xf_off = 256;
    p.xf_gs_off = p.xf_off + (size_t)T * D * 3;
    p.part_off = al128(p.xf_gs_off + (size_t)T * xf_gs_bytes(D));
    p.stage_bytes = al128(gu_slot(rbg) + gu_slot(rbu));
    p.stage_off = al128(p.part_off + (size_t)FS_GROUPS * 16 * 16 * MU * 4);
    p.extra_off = al128(p.stage_off + (size_t)FS_GROUPS * p.stage_bytes);
    p.total = p.extra_off + route_bytes;
    return p;
}

template <int QG, int QU>
__global__ void __launch_bounds__((NWC_GU + 1) * 32, 1) k_moe_gateup_fs(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int D = a.D, FF = a.FF, nsb = D >> 8, NRB = FF >> 4, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, TK = T * a.n_used;
    const FsPlan pl = gateup_fs_plan(T, D, a.gate_rb, a.up_rb, route_sm_bytes(a.n_expert, TK, true));
    constexpr int S = FS_GROUPS;
    uint64_t* full = reinterpret_cast<uint64_t*>(sm);
    uint64_t* empty = full + 4;
    uint64_t* done = full + 8;  // per stage: the group's four warps have stored their partial results
    uint64_t* xfbar = full + 12;
    int4* info = reinterpret_cast<int4*>(sm + pl.info_off);
    __shared__ int abort_flag;
    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 4);
            mbar_init(&done[s], 4);
        }
        mbar_init(xfbar, 1);
        abort_flag = 0;
        mbar_fence_init();
    }
    RouteSm rt = route_sm_carve(sm + pl.extra_off, a.n_expert, TK, true);
    {  // the experts' matrix table does not depend on earlier grids
        const int E = a.n_expert;
        for (int i = tid; i < 3 * E; i += blockDim.x) rt.tab[i] = i < E ? a.gate[i] : i < 2 * E ? a.up[i - E] : a.down[i - 2 * E];
    }
    __syncthreads();
    pdl_wait();  // the logits and the tokens' XF come from the previous grid
    pdl_trigger();
    const uint32_t xfg = (uint32_t)xf_gs_bytes(D);
    if (tid == 0) {  // all T tokens' XF rows: fragments and group sums, one bulk copy each
        mbar_expect_tx(xfbar, (uint32_t)T * ((uint32_t)D * 3 + xfg));
        tma_load_1d(sm + pl.xf_off, a.xf.frag, (uint32_t)T * D * 3, xfbar);
        tma_load_1d(sm + pl.xf_gs_off, a.xf.gs, (uint32_t)T * xfg, xfbar);
    }
    route_block<true>(a, rt, blockIdx.x == 0);
    __syncthreads();
    const int G = *rt.G;
    const int nunits = G * NRB;
    const int u0 = (int)((long long)blockIdx.x * nunits / gridDim.x), u1 = (int)((long long)(blockIdx.x + 1) * nunits / gridDim.x);
    const size_t rbg = a.gate_rb, rbu = a.up_rb, up_at = gu_slot(rbg);
    const Rows Lg = rows_of(rbg), Lu = rows_of(rbu);

    if (warp == NWC_GU) {  // ---------------- producer: weight tiles only
        if (lane != 0) return;
        int i = 0;
        for (int u = u0; u < u1; u++, i++) {
            const int s = i % S;
            if (i >= S && !mbar_wait_bounded(&empty[s], (uint32_t)(i / S - 1) & 1u)) {
                set_flag(a.status, ST_WAIT_TIMEOUT);
                atomicExch(&abort_flag, 1);
                break;
            }
            if (*(volatile int*)&abort_flag) break;
            const int gi = u / NRB, rb = u - gi * NRB, r0 = 16 * rb;
            const uint8_t* wg = rt.g_w[3 * gi];
            const uint8_t* wu = rt.g_w[3 * gi + 1];
            const int mc = rt.g_info[4 * gi + 2];
            const bool ok = al16(wg) && al16(wu);
            if (!ok) set_flag(a.status, ST_BAD_ARG);
            uint8_t* stage = sm + pl.stage_off + (size_t)s * pl.stage_bytes;
            const uint32_t lg = (!split8(rbg) && ok) ? rows_lead(Lg, wg, rbg, r0) : 0u;
            const uint32_t lu = (!split8(rbu) && ok) ? rows_lead(Lu, wu, rbu, r0) : 0u;
            info[s] = make_int4(rb | (gi << 12), info_bits(0, mc, ok, false), rt.g_info[4 * gi + 1], (int)(lg | (lu << 8)));
            uint32_t bytes = 0;
            if (ok) {
                bytes += split8(rbg) ? (uint32_t)(16 * rbg) : rows_copy_bytes(Lg, wg, rbg, r0, 16);
                bytes += split8(rbu) ? (uint32_t)(16 * rbu) : rows_copy_bytes(Lu, wu, rbu, r0, 16);
            }
            mbar_expect_tx(&full[s], bytes);
            if (ok) {
                if (split8(rbg)) {
                    tma_load_1d(stage, wg + (size_t)r0 * rbg, (uint32_t)(8 * rbg), &full[s]);
                    tma_load_1d(stage + split8_off(rbg), wg + (size_t)(r0 + 8) * rbg, (uint32_t)(8 * rbg), &full[s]);
                } else {
                    rows_issue(Lg, wg, rbg, r0, 16, stage, &full[s]);
                }
                if (split8(rbu)) {
                    tma_load_1d(stage + up_at, wu + (size_t)r0 * rbu, (uint32_t)(8 * rbu), &full[s]);
                    tma_load_1d(stage + up_at + split8_off(rbu), wu + (size_t)(r0 + 8) * rbu, (uint32_t)(8 * rbu),
                                &full[s]);
                } else {
                    rows_issue(Lu, wu, rbu, r0, 16, stage + up_at, &full[s]);
                }
            }
        }
        const int issued = i;
        for (int k = (issued > S ? issued - S : 0); k < issued; k++) {
            if (!mbar_wait_bounded(&empty[k % S], (uint32_t)(k / S) & 1u)) {
                drain(full, issued, k, S);
                break;
            }
        }
        return;
    }

    // ---------------- consumers: group q = warp / 4 runs units q, q + 4, ... on stage q
    const int q = warp >> 2, k4 = warp & 3, mtx = k4 >> 1, vw0 = 4 * (k4 & 1), g = lane >> 2, t = lane & 3;
    const size_t rbm = mtx ? rbu : rbg;
    const int prow0 = gu_row(rbm, g, 0), prow1 = gu_row(rbm, g, 1);
    if (!mbar_wait_bounded(xfbar, 0u)) {  // the tokens' XF rows
        set_flag(a.status, ST_WAIT_TIMEOUT);
        atomicExch(&abort_flag, 1);
        return;
    }
    const uint8_t* xfr = sm + pl.xf_off;
    const uint8_t* xgs = sm + pl.xf_gs_off;
    float* part = reinterpret_cast<float*>(sm + pl.part_off) + (size_t)q * 16 * 16 * MU;  // [16 subsets][16 rows][MU]
    int n = 0;  // uses of this group's stage
    for (int i = q; u0 + i < u1; i += S, n++) {
        const int s = q;
        if (!mbar_wait_bounded(&full[s], (uint32_t)n & 1u)) {
            set_flag(a.status, ST_WAIT_TIMEOUT);
            atomicExch(&abort_flag, 1);
            return;  // the producer drains what it issued
        }
        const int4 in = info[s];
        const int rb = in.x & 0xfff, gi = in.x >> 12, mc = (in.y >> 4) & 15, s0 = in.z;
        const int tok0 = rt.g_tok[MU * gi], tok1 = mc > 1 ? rt.g_tok[MU * gi + 1] : tok0;
        // the lane's B operands over the staged rows of the group's tokens (as BPtr<1> / min_operand)
        BPtr<1> bp(xfr, D >> 5, 1);
        {
            int ti = g / 3, pg = g % 3;
            if (g >= 6 || ti >= mc) ti = pg = 0;
            bp.p[0] = xfr + ((size_t)(ti ? tok1 : tok0) * (D >> 5) * 3 + pg) * 32;
        }
        int mt = g >> 1;
        if (g >= 4 || mt >= mc) mt = 0;
        const uint8_t* mq = xgs + (size_t)(mt ? tok1 : tok0) * xfg + 16 + (g & 1) * 16 + 4 * t;
        const float ts = t < mc ? *reinterpret_cast<const float*>(xgs + (size_t)(t ? tok1 : tok0) * xfg) : 0.f;
        const uint8_t* stage = sm + pl.stage_off + (size_t)s * pl.stage_bytes;
#pragma unroll 2
        for (int v = 0; v < 4; v++) {
            const int vw = vw0 + v;
            float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}}, mn[2] = {0.f, 0.f};
            if (in.y & 256) {
                if (mtx == 0)
                    block_tasks<QG>(rows_gu(stage, rbg, in.w & 255), nsb, vw, 8, bp, mq, acc, mn);
                else
                    block_tasks<QU>(rows_gu(stage + up_at, rbu, (in.w >> 8) & 255), nsb, vw, 8, bp, mq, acc, mn);
            }
            warp_values(acc, mn, ts, part + (size_t)(mtx * 8 + vw) * 16 * MU, prow0, prow1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&done[s]);
        if (k4 == 0) {  // the group's reducer: SiLU*mul of the summed subsets
            if (!mbar_wait_bounded(&done[s], (uint32_t)n & 1u)) {
                set_flag(a.status, ST_WAIT_TIMEOUT);
                atomicExch(&abort_flag, 1);
                return;
            }
            const int r = lane >> 1, tk = lane & 1;
            if (tk < mc) {
                float gv = 0.f, uv = 0.f;
#pragma unroll
                for (int w = 0; w < 8; w++) {
                    gv += part[(w * 16 + r) * MU + tk];
                    uv += part[((8 + w) * 16 + r) * MU + tk];
                }
                a.h[(size_t)(s0 + tk) * FF + 16 * rb + r] = silu_mul(gv, uv);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// ------------------------------------------------------------------------------------------------
// down projection + weighted combine + residual add
// ------------------------------------------------------------------------------------------------
template <int QD, int G>
__global__ void __launch_bounds__((NWC_DN + 1) * 32, 1) k_moe_down(MoeArgs a) {
    constexpr int PI = dn_prep_items(G);
    extern __shared__ __align__(128) uint8_t sm[];
    const int D = a.D, FF = a.FF, nsb = FF >> 8, NRG = D / DN_ROWS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t rb = a.down_rb;
    const Plan pl = down_plan(FF, rb, down_cache_bytes(a), G);
    const int S = pl.S;
    uint64_t* full = reinterpret_cast<uint64_t*>(sm);
    uint64_t* empty = full + 4;
    uint64_t* done = full + 8;     // per stage: every consumer warp has stored its partial results
    uint64_t* cbar = full + 12;    // the consumer warps' barrier of the h-row prep (one arrival per warp)
    int4* info = reinterpret_cast<int4*>(sm + pl.info_off);
    __shared__ int abort_flag;
    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NWC_DN);
            mbar_init(&done[s], NWC_DN);
        }
        mbar_init(cbar, NWC_DN);
        abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_wait();  // h and the routing come from the previous grids
    pdl_trigger();
    // small batches: the whole group list (at most T*K records) is read into shared memory in the same
    // round trip as its length
    GroupRec* gcache = G == MU && a.fused_route ? reinterpret_cast<GroupRec*>(sm + pl.extra_off) : nullptr;
    if (gcache) {
        const int4* src = reinterpret_cast<const int4*>(a.rw.groups);
        int4* dst = reinterpret_cast<int4*>(gcache);
        for (int i = tid; i < a.T * a.n_used * (int)(sizeof(GroupRec) / 16); i += blockDim.x) dst[i] = __ldcg(src + i);
    }
    const int NG = a.rw.ngroups[0];
    if (gcache) __syncthreads();
    auto group = [&](int gi) { return gcache ? gcache[gi] : a.rw.groups[gi]; };
    const int nunits = NG * NRG;
    const int u0 = (int)((long long)blockIdx.x * nunits / gridDim.x), u1 = (int)((long long)(blockIdx.x + 1) * nunits / gridDim.x);
    const Rows L = rows_of(rb);

    if (warp == NWC_DN) {  // ---------------- producer
        if (lane != 0) return;
        int cur = -1, xb = 1, i = 0;
        GroupRec rec{}, nxt{};
        if (u0 < u1) nxt = group(u0 / NRG);
        for (int u = u0; u < u1; u++, i++) {
            const int s = i % S;
            if (i >= S && !mbar_wait_bounded(&empty[s], (uint32_t)(i / S - 1) & 1u)) {
                set_flag(a.status, ST_WAIT_TIMEOUT);
                atomicExch(&abort_flag, 1);
                break;
            }
            if (*(volatile int*)&abort_flag) break;
            const int gi = u / NRG, rg = u - gi * NRG;
            const bool fresh = gi != cur;
            if (fresh) {
                rec = nxt;
                cur = gi;
                xb ^= 1;
                if ((gi + 1) * NRG < u1) nxt = group(gi + 1);
            }
            const uint8_t* w = rec.w[2];
            const bool ok = al16(w);
            if (!ok) set_flag(a.status, ST_BAD_ARG);
            info[s] = make_int4(rg, info_bits(xb, rec.mc, ok, fresh), rec.s0,
                                ok ? (int)rows_lead(L, w, rb, DN_ROWS * rg) : 0);
            const uint32_t bytes = ok ? rows_copy_bytes(L, w, rb, DN_ROWS * rg, DN_ROWS) : 0u;
            mbar_expect_tx(&full[s], bytes);
            if (ok) rows_issue(L, w, rb, DN_ROWS * rg, DN_ROWS, sm + pl.stage_off + (size_t)s * pl.stage_bytes, &full[s]);
        }
        const int issued = i;
        for (int k = (issued > S ? issued - S : 0); k < issued; k++) {
            if (!mbar_wait_bounded(&empty[k % S], (uint32_t)(k / S) & 1u)) {
                drain(full, issued, k, S);
                break;
            }
        }
        return;
    }

    // ---------------- consumers: warp w works on rows 16 (w / 3) .. +15 of the unit, super-blocks w % 3 + 3j
    const int rbk = warp / 3, wsub = warp - 3 * rbk, t = lane & 3;
    // h rows of a group -> fragment form in XF buffer xb, by all consumer warps (bounded waits on cbar):
    // each thread loads up to DN_PREP_ITEMS items of 8 elements (every warp's items belong to one row),
    // the rows' max |h| are combined across the warps, then each thread writes its items' digits and
    // sums. False after a timed-out wait (flagged; the caller ends the warp).
    __shared__ float s_pmax[G][NWC_DN * PI];
    uint32_t cphase = 0;
    auto consumers_sync = [&]() {
        __syncwarp();
        if (lane == 0) mbar_arrive(cbar);
        if (!mbar_wait_bounded(cbar, cphase & 1u)) {
            set_flag(a.status, ST_WAIT_TIMEOUT);
            atomicExch(&abort_flag, 1);
            return false;
        }
        cphase++;
        return true;
    };
    auto prep_group = [&](int xb, int s0, int mc) {
        uint8_t* xs = sm + pl.xf_off + (size_t)xb * pl.xfb;
        const int nit = FF >> 3, tot = mc * nit;  // nit % 32 == 0: warp-uniform rows and bounds
        float4 u[PI], w[PI];
#pragma unroll
        for (int k = 0; k < PI; k++) {
            const int it = tid + NWC_DN * 32 * k, tk = it < tot ? it / nit : 0, i = it - tk * nit;
            float m = 0.f;
            if (it < tot) {
                const float4* x4 = reinterpret_cast<const float4*>(a.h + (size_t)(s0 + tk) * FF);
                u[k] = __ldcg(x4 + 2 * i);
                w[k] = __ldcg(x4 + 2 * i + 1);
                m = fmaxf(fmaxf(fmaxf(fabsf(u[k].x), fabsf(u[k].y)), fmaxf(fabsf(u[k].z), fabsf(u[k].w))),
                          fmaxf(fmaxf(fabsf(w[k].x), fabsf(w[k].y)), fmaxf(fabsf(w[k].z), fabsf(w[k].w))));
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane < G) s_pmax[lane][warp * PI + k] = (it < tot && lane == tk) ? m : 0.f;
        }
        if (!consumers_sync()) return false;
        auto row_max = [&](int tk) {  // max |h| of row tk over every warp's items
            float mx = 0.f;
            for (int j = 0; j < NWC_DN * PI; j++) mx = fmaxf(mx, s_pmax[tk][j]);
            return (!(mx > 0.f) || mx == INFINITY) ? 127.f : mx;
        };
        if (tid < mc)
            *reinterpret_cast<float4*>(xs + xs_gs_off(FF, G) + (size_t)tid * xf_gs_bytes(FF)) =
                make_float4(row_max(tid) / 127.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < PI; k++) {
            const int it = tid + NWC_DN * 32 * k;
            if (it < tot) {  // warp-uniform
                const int tk = it / nit;
                prep_item(u[k], w[k], it - tk * nit, 127.f / row_max(tk), reinterpret_cast<uint2*>(xs + (size_t)tk * FF * 3),
                          xs + xs_gs_off(FF, G) + (size_t)tk * xf_gs_bytes(FF));
            }
        }
        return consumers_sync();  // the group's rows are ready for every consumer warp (and s_pmax is free)
    };
    if (u0 < u1) {  // the first group's h rows, while the first weight tiles are in flight
        const GroupRec r0 = group(u0 / NRG);
        if (!prep_group(0, r0.s0, r0.mc)) return;
    }
    int i = 0;
    for (int u = u0; u < u1; u++, i++) {
        const int s = i % S;
        if (!mbar_wait_bounded(&full[s], (uint32_t)(i / S) & 1u)) {
            set_flag(a.status, ST_WAIT_TIMEOUT);
            atomicExch(&abort_flag, 1);
            return;
        }
        const int4 in = info[s];
        const int rg = in.x, xb = in.y & 1, mc = (in.y >> 4) & 15, s0 = in.z;
        if ((in.y & 512) && u != u0 && !prep_group(xb, s0, mc)) return;  // a later group's first unit here
        const uint8_t* xs = sm + pl.xf_off + (size_t)xb * pl.xfb;
        float* part = reinterpret_cast<float*>(sm + pl.part_off) + ((size_t)s * NWC_DN + warp) * 16 * G;
        for (int st = 0; 2 * st < mc;) {  // column sets: slots 2 st, 2 st + 1 of the group
            const int ms = mc - 2 * st;
            const uint8_t* xg = xs + xs_gs_off(FF, G) + (size_t)(2 * st) * xf_gs_bytes(FF);
            const RowsAny rows =
                rows_pair(sm + pl.stage_off + (size_t)s * pl.stage_bytes + in.w + (size_t)(16 * rbk) * L.stride, L.stride);
            if (G > MU && ms > 2) {  // sets st, st + 1 over one decode of the weights
                const uint8_t* xg1 = xg + 2 * (size_t)xf_gs_bytes(FF);
                float acc[2][4] = {}, mn[2][2] = {};
                if (in.y & 256) {
                    const uint8_t* bq[2] = {BPtr<1>(xs + (size_t)(2 * st) * FF * 3, FF >> 5, ms).p[0],
                                            BPtr<1>(xs + (size_t)(2 * st + 2) * FF * 3, FF >> 5, ms - 2).p[0]};
                    const uint8_t* mq[2] = {min_operand(xg, FF, ms), min_operand(xg1, FF, ms - 2)};
                    block_tasks_m<QD, 2>(rows, nsb, wsub, 3, bq, mq, acc, mn);
                }
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    const float a1[1][4] = {{acc[k][0], acc[k][1], acc[k][2], acc[k][3]}};
                    const float ts = t < ms - 2 * k ? *reinterpret_cast<const float*>(xg + (size_t)(2 * k + t) * xf_gs_bytes(FF)) : 0.f;
                    warp_values(a1, mn[k], ts, part, 2 * ((lane >> 2) & 7), 2 * ((lane >> 2) & 7) + 1, G, 2 * st + 2 * k);
                }
                st += 2;
                continue;
            }
            float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}}, mn[2] = {0.f, 0.f};
            if (in.y & 256) {
                const BPtr<1> bp(xs + (size_t)(2 * st) * FF * 3, FF >> 5, ms);
                block_tasks<QD>(rows, nsb, wsub, 3, bp, min_operand(xg, FF, ms), acc, mn);
            }
            const float ts = t < ms ? *reinterpret_cast<const float*>(xg + (size_t)t * xf_gs_bytes(FF)) : 0.f;
            warp_values(acc, mn, ts, part, 2 * ((lane >> 2) & 7), 2 * ((lane >> 2) & 7) + 1, G, 2 * st);
            st++;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&done[s]);
        const bool reducer = warp == i % NWC_DN;
        if (reducer) {  // this unit's reducer (round robin): y rows of the unit's slots
            if (!mbar_wait_bounded(&done[s], (uint32_t)(i / S) & 1u)) {
                set_flag(a.status, ST_WAIT_TIMEOUT);
                atomicExch(&abort_flag, 1);
                return;
            }
            const float* P = reinterpret_cast<const float*>(sm + pl.part_off) + (size_t)s * NWC_DN * 16 * G;
            for (int j = lane; j < DN_ROWS * G; j += 32) {
                const int r = j / G, tk = j - r * G;
                if (tk < mc) {
                    const int rk = r >> 4, rr = r & 15;
                    const float v = (P[((3 * rk) * 16 + rr) * G + tk] + P[((3 * rk + 1) * 16 + rr) * G + tk]) +
                                    P[((3 * rk + 2) * 16 + rr) * G + tk];
                    a.y[(size_t)(s0 + tk) * D + DN_ROWS * rg + r] = v;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// ------------------------------------------------------------------------------------------------
// weighted combine + residual add: x[t] += sum_k w_k y[slot_k] over token t's slots in ascending slot
// (= expert) order (qwen3moe.cpp:1024, :1062-1069). Grid (D / (2 * COMB_NT), T); each thread owns two
// consecutive elements of one token row.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(COMB_NT) k_moe_combine(MoeArgs a) {
    __shared__ int s_sl[32];
    __shared__ float s_w[32];
    const int t = blockIdx.y, K = a.n_used, D = a.D;
    pdl_wait();  // y and the routing come from the previous grids
    if (a.given && __ldg(a.given + t) < 0) return;  // an absent row (given ids have K == 1)
    if (threadIdx.x < K) {
        const int sl = a.rw.token_slots[t * K + threadIdx.x];
        s_sl[threadIdx.x] = sl;
        s_w[threadIdx.x] = a.rw.slot_w[sl];
    }
    __syncthreads();
    const int c = 2 * (blockIdx.x * COMB_NT + threadIdx.x);
    if (c >= D) return;
    float2 acc = make_float2(0.f, 0.f);
    for (int k = 0; k < K; k++) {
        const float2 v = *reinterpret_cast<const float2*>(a.y + (size_t)s_sl[k] * D + c);
        acc.x = fmaf(s_w[k], v.x, acc.x);
        acc.y = fmaf(s_w[k], v.y, acc.y);
    }
    float2* xp = reinterpret_cast<float2*>(a.x + (size_t)t * D + c);
    float2 xv = *xp;
    xv.x += acc.x;
    xv.y += acc.y;
    *xp = xv;
}

// ------------------------------------------------------------------------------------------------
// ragged batches of any size (the grouped tensor-core path): routing without the 64-token masks.
// Slot order inside an expert follows the count atomics (not token order); every slot's result depends
// only on its own token, and the combine visits a token's slots in expert order, so the outputs are
// the same for any slot order.
// ------------------------------------------------------------------------------------------------
constexpr int BIG_NT = 128;
// One warp per token. The slot counts are gathered per block first (shared-memory atomics), then one
// global atomic per (block, expert) reserves the block's range of the expert's slots: under skewed
// routing a few popular experts take a large share of every token's k slots, and one global atomic per
// slot on their counters serialises.
template <bool GIVEN>
__global__ void __launch_bounds__(BIG_NT) k_route_big(MoeArgs a, int* __restrict__ cnt, int* __restrict__ local) {
    __shared__ uint32_t s_rk[(BIG_NT / 32) * 64];
    __shared__ int s_cnt[MAX_EXPERTS];  // this block's slots per expert, then the block's first slot index
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * (BIG_NT / 32) + warp, E = a.n_expert, K = a.n_used;
    if (cnt) {
        for (int i = threadIdx.x; i < E; i += BIG_NT) s_cnt[i] = 0;
        __syncthreads();
    }
    int my_e = 0, pos = -1;  // pos: this slot's place among the block's slots of my_e (-1: not counted)
    float my_w = 0.f;
    if (t < a.T) {  // whole warps
        const float* lg = a.logits + (size_t)t * E;
        if constexpr (GIVEN) {  // assigned experts (expert-parallel receiver): weight 1, no ranking
            if (lane < K) {
                my_e = __ldg(a.given + (size_t)t * K + lane);
                my_w = 1.0f;
            }
        } else if (E <= 128) route_token<4>(lg, E, K, lane, s_rk + warp * 64, my_e, my_w);
        else if (E <= 256) route_token<8>(lg, E, K, lane, s_rk + warp * 64, my_e, my_w);
        else route_token<16>(lg, E, K, lane, s_rk + warp * 64, my_e, my_w);
        if (lane < K) {
            if (GIVEN && my_e < 0) {  // an absent slot (padding row of the receiver)
                a.rw.ids[(size_t)t * K + lane] = -1;
            } else {
                if (my_e < 0 || my_e >= E) {  // NaN logits or a given id out of range
                    set_flag(a.status, ST_BAD_INDEX);
                    my_e = 0;
                }
                a.rw.ids[(size_t)t * K + lane] = my_e;
                a.rw.wts[(size_t)t * K + lane] = my_w;
                if (cnt) pos = atomicAdd(&s_cnt[my_e], 1);
            }
        }
    }
    if (!cnt) return;  // routing alone (the same for the whole block)
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += BIG_NT) {
        const int n = s_cnt[i];
        if (n) s_cnt[i] = atomicAdd(&cnt[i], n);
    }
    __syncthreads();
    if (pos >= 0) local[(size_t)t * K + lane] = s_cnt[my_e] + pos;
}

// One block: slot offsets, tile prefixes of the two GEMMs, active list.
__global__ void __launch_bounds__(512) k_plan_big(MoeArgs a, const int* __restrict__ cnt, int* __restrict__ tiles_gu,
                                                  int* __restrict__ tiles_dn) {
    __shared__ int ws[3][16];
    pdl_wait();
    pdl_trigger();
    const int E = a.n_expert, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c = tid < E ? cnt[tid] : 0;
    const int nt = (c + 127) / 128;
    int v[3] = {c, nt, c > 0 ? 1 : 0};
    int incl[3];
#pragma unroll
    for (int q = 0; q < 3; q++) {
        int x = v[q];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        incl[q] = x;
        if (lane == 31) ws[q][warp] = x;
    }
    __syncthreads();
    int base[3] = {0, 0, 0};
#pragma unroll
    for (int q = 0; q < 3; q++)
        for (int w = 0; w < warp; w++) base[q] += ws[q][w];
    const int off = base[0] + incl[0] - v[0], toff = base[1] + incl[1] - v[1], aoff = base[2] + incl[2] - v[2];
    const int RTg = a.FF / GU_TILE_ROWS, RTd = a.D / DN_TILE_ROWS;
    if (tid < E) {
        a.rw.offsets[tid] = off;
        tiles_gu[tid] = RTg * toff;
        tiles_dn[tid] = RTd * toff;
        if (c > 0) a.rw.active[1 + aoff] = tid;
    }
    if (tid == E - 1) {
        a.rw.offsets[E] = off + c;
        tiles_gu[E] = RTg * (toff + nt);
        tiles_dn[E] = RTd * (toff + nt);
        a.rw.active[0] = aoff + v[2];
        a.rw.ngroups[0] = toff + nt;
    }
}

// One thread per (token, k): slot = offset[e] + its count index; the token's slots by expert order.
// (cnt / local may be null for routing alone.)
__global__ void __launch_bounds__(256) k_scatter_big(MoeArgs a, const int* __restrict__ local) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * 256 + threadIdx.x, K = a.n_used;
    if (i >= a.T * K) return;
    const int t = i / K;
    const int e = a.rw.ids[i];
    if (e < 0) return;  // absent slot (given ids only)
    const int slot = a.rw.offsets[e] + local[i];
    a.rw.slot_token[slot] = t;
    a.rw.slot_w[slot] = a.rw.wts[i];
    int rank = 0;
    for (int j = 0; j < K; j++) rank += a.rw.ids[(size_t)t * K + j] < e;
    a.rw.token_slots[(size_t)t * K + rank] = slot;
}

// ------------------------------------------------------------------------------------------------
// launchers
// ------------------------------------------------------------------------------------------------
namespace {
template <typename Kern>
void smem_attr(Kern k, size_t smem) {
    static std::mutex mu;
    static std::unordered_map<const void*, size_t> done;
    std::lock_guard<std::mutex> lk(mu);
    size_t& cur = done[reinterpret_cast<const void*>(k)];
    if (cur < smem) {
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cur = smem;
    }
}
int max_groups(const MoeArgs& a) {
    const int g = a.gsz == GW ? GW : MU;
    return std::min(a.T * a.n_used, a.n_expert * ((a.T + g - 1) / g));
}

}  // namespace

size_t moe_smem_gateup(int D, size_t rbg, size_t rbu) { return gateup_plan(D, rbg, rbu).total; }
int moe_chunk_group_size(int D, int FF, size_t rbg, size_t rbu, size_t rbd) {
    const bool wide = gateup_plan(D, rbg, rbu, 0, GW).total <= SMEM_CAP && down_plan(FF, rbd, 0, GW).total <= SMEM_CAP &&
                      GW * (FF / 8) <= dn_prep_items(GW) * NWC_DN * 32 && (FF >> 4) >= gateup_plan(D, rbg, rbu, 0, GW).S &&
                      D / DN_ROWS >= down_plan(FF, rbd, 0, GW).S;
    return wide ? GW : MU;
}
size_t moe_smem_down(int FF, size_t rbd) { return down_plan(FF, rbd).total; }

cudaError_t launch_moe_route(const MoeArgs& a, cudaStream_t st) {
    if (a.T < 1 || a.T > MOE_TMAX || a.n_expert > MAX_EXPERTS || a.n_used > 32 || a.n_used > a.n_expert ||
        a.D % 256 || a.D % DN_ROWS)
        return cudaErrorInvalidValue;
    const dim3 grid(1 + a.T), block(ROUTE_NT);
    if (a.gsz == GW)
        return a.given ? launch_pdl(k_moe_route<true, GW>, grid, block, 0, st, a)
                       : launch_pdl(k_moe_route<false, GW>, grid, block, 0, st, a);
    return a.given ? launch_pdl(k_moe_route<true, MU>, grid, block, 0, st, a)
                   : launch_pdl(k_moe_route<false, MU>, grid, block, 0, st, a);
}

template <int QG, int QU, int G>
static cudaError_t gateup_as(const MoeArgs& a, cudaStream_t st) {
    const bool fused = G == MU && a.fused_route;
    const Plan pl = gateup_plan(a.D, a.gate_rb, a.up_rb, fused ? route_sm_bytes(a.n_expert, a.T * a.n_used, true) : 0, G);
    if (pl.total > SMEM_CAP || (a.FF >> 4) < pl.S) return cudaErrorInvalidValue;
    smem_attr(k_moe_gateup<QG, QU, G>, pl.total);
    const int units = max_groups(a) * (a.FF >> 4);
    return launch_pdl(k_moe_gateup<QG, QU, G>, dim3(std::min(sm_count(), units)), (NWC_GU + 1) * 32, pl.total, st, a);
}
template <int QG, int QU>
static cudaError_t gateup_pick(const MoeArgs& a, cudaStream_t st) {
    if (a.fused_route && a.FF < (1 << 16)) {  // unit info packs the row block in 12 bits
        const FsPlan pl = gateup_fs_plan(a.T, a.D, a.gate_rb, a.up_rb, route_sm_bytes(a.n_expert, a.T * a.n_used, true));
        if (pl.total <= SMEM_CAP) {
            smem_attr(k_moe_gateup_fs<QG, QU>, pl.total);
            const int units = max_groups(a) * (a.FF >> 4);
            return launch_pdl(k_moe_gateup_fs<QG, QU>, dim3(std::min(sm_count(), units)), (NWC_GU + 1) * 32, pl.total, st,
                              a);
        }
    }
    return a.gsz == GW ? gateup_as<QG, QU, GW>(a, st) : gateup_as<QG, QU, MU>(a, st);
}
template <int QG>
static cudaError_t gateup_g(const MoeArgs& a, cudaStream_t st) {
    switch (a.up_type) {
        case T_Q4_K: return gateup_pick<QG, T_Q4_K>(a, st);
        case T_Q5_K: return gateup_pick<QG, T_Q5_K>(a, st);
        case T_Q6_K: return gateup_pick<QG, T_Q6_K>(a, st);
        default: return cudaErrorInvalidValue;
    }
}
cudaError_t launch_moe_gateup(const MoeArgs& a, cudaStream_t st) {
    if (a.D % 256 || a.FF % 256) return cudaErrorInvalidValue;
    switch (a.gate_type) {
        case T_Q4_K: return gateup_g<T_Q4_K>(a, st);
        case T_Q5_K: return gateup_g<T_Q5_K>(a, st);
        case T_Q6_K: return gateup_g<T_Q6_K>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

template <int QD, int G>
static cudaError_t down_as(const MoeArgs& a, cudaStream_t st) {
    const Plan pl = down_plan(a.FF, a.down_rb, G == MU ? down_cache_bytes(a) : 0, G);
    if (pl.total > SMEM_CAP || a.D / DN_ROWS < pl.S || G * (a.FF / 8) > dn_prep_items(G) * NWC_DN * 32)
        return cudaErrorInvalidValue;
    smem_attr(k_moe_down<QD, G>, pl.total);
    const int units = max_groups(a) * (a.D / DN_ROWS);
    return launch_pdl(k_moe_down<QD, G>, dim3(std::min(sm_count(), units)), (NWC_DN + 1) * 32, pl.total, st, a);
}
cudaError_t launch_moe_down(const MoeArgs& a, cudaStream_t st, bool combine) {
    if (a.FF % 256 || a.D % DN_ROWS || a.T > MOE_TMAX) return cudaErrorInvalidValue;
    cudaError_t e;
    const bool w = a.gsz == GW;
    switch (a.down_type) {
        case T_Q4_K: e = w ? down_as<T_Q4_K, GW>(a, st) : down_as<T_Q4_K, MU>(a, st); break;
        case T_Q5_K: e = w ? down_as<T_Q5_K, GW>(a, st) : down_as<T_Q5_K, MU>(a, st); break;
        case T_Q6_K: e = w ? down_as<T_Q6_K, GW>(a, st) : down_as<T_Q6_K, MU>(a, st); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess || !combine) return e;
    return launch_moe_combine(a, st);
}

cudaError_t launch_moe_combine(const MoeArgs& a, cudaStream_t st) {
    const int bx = (a.D / 2 + COMB_NT - 1) / COMB_NT;
    return launch_pdl(k_moe_combine, dim3(bx, a.T), dim3(COMB_NT), 0, st, a);
}

cudaError_t launch_route_big(const MoeArgs& a, int* cnt, int* local, cudaStream_t st) {
    if (a.T < 1 || a.n_expert > MAX_EXPERTS || a.n_used > 32 || a.n_used > a.n_expert) return cudaErrorInvalidValue;
    const int per = BIG_NT / 32;
    const dim3 grid((a.T + per - 1) / per);
    return a.given ? launch_pdl(k_route_big<true>, grid, dim3(BIG_NT), 0, st, a, cnt, local)
                   : launch_pdl(k_route_big<false>, grid, dim3(BIG_NT), 0, st, a, cnt, local);
}
cudaError_t launch_plan_big(const MoeArgs& a, const int* cnt, int* tiles_gu, int* tiles_dn, cudaStream_t st) {
    if (a.n_expert > 512 || a.FF % 64 || a.D % 128) return cudaErrorInvalidValue;
    return launch_pdl(k_plan_big, dim3(1), dim3(512), 0, st, a, cnt, tiles_gu, tiles_dn);
}
cudaError_t launch_scatter_big(const MoeArgs& a, const int* local, cudaStream_t st) {
    return launch_pdl(k_scatter_big, dim3((a.T * a.n_used + 255) / 256), dim3(256), 0, st, a, local);
}

}  // namespace eb
