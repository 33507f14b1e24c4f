// decode.cu -- the non-expert kernels of a qwen3moe forward pass (Engine::forward, qwen3moe.cpp:929-1074)
// on sm_100a: embedding rows, RMSNorm, QK-norm + NeoX RoPE + KV-cache append, causal GQA attention
// split over the context with a merge that also preps the o-projection's activations, first-maximum argmax,
// and the device-side decode state.
//
// Every kernel that depends on the position reads it from device memory (`DecodeState.pos`), so one
// captured CUDA graph serves every decode step: the argmax kernel writes the next token and advances
// the position for the following replay.
//
// These kernels are memory- or latency-bound (a few KB to a few MB per call); the weight GEMVs around
// them (kernels.cu, moe.cu) carry the bytes.
#include <float.h>
#include <math.h>

#include "decode.cuh"
#include "kq.cuh"

namespace eb {

// ---- dequantisation of single rows (embedding lookup), the reference decoders (qwen3moe.cpp:128-202)
__device__ __forceinline__ float f16_at(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& sc, int& mn) {
    if (j < 4) {
        sc = q[j] & 63;
        mn = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}
// Element i of a row of `type` (block-granular random access).
__device__ float dq_elem(const uint8_t* row, int type, int i) {
    switch (type) {
        case T_F32: return reinterpret_cast<const float*>(row)[i];
        case T_F16: return f16_at(row + 2 * i);
        case T_Q8_0: {
            const uint8_t* b = row + (i >> 5) * 34;
            return f16_at(b) * (float)(int8_t)b[2 + (i & 31)];
        }
        case T_Q4_K:
        case T_Q5_K: {
            const bool q5 = type == T_Q5_K;
            const uint8_t* b = row + (i >> 8) * (q5 ? 176 : 144);
            const int e = i & 255, c = e >> 6, hi = (e >> 5) & 1, l = e & 31;
            int sc, mn;
            scale_min_k4(2 * c + hi, b + 4, sc, mn);
            const uint8_t* qs = b + (q5 ? 48 : 16);
            int q = hi ? (qs[32 * c + l] >> 4) : (qs[32 * c + l] & 0x0f);
            if (q5) q += ((b[16 + l] >> (2 * c + hi)) & 1) << 4;
            const float d = f16_at(b) * (float)sc, o = f16_at(b + 2) * (float)mn;
            return d * (float)q - o;
        }
        case T_Q6_K: {
            const uint8_t* b = row + (i >> 8) * 210;
            const int e = i & 255, h = e >> 7, r = e & 127, quad = r >> 5, l = r & 31;
            const uint8_t* ql = b + 64 * h;
            const uint8_t* qh = b + 128 + 32 * h;
            const int8_t* s = reinterpret_cast<const int8_t*>(b + 192) + 8 * h;
            const uint8_t lo = (quad & 1) ? ql[l + 32] : ql[l];
            const int q = (int)(((quad & 2) ? (lo >> 4) : (lo & 0x0f)) | (((qh[l] >> (2 * quad)) & 3) << 4)) - 32;
            return f16_at(b + 208) * (float)s[l / 16 + 2 * quad] * (float)q;
        }
        default: return 0.f;
    }
}

__global__ void k_embed(const uint8_t* __restrict__ W, int type, size_t row_bytes, int D, int n_rows,
                        const int* __restrict__ toks, int nb, float* __restrict__ x, int* status) {
    const int t = blockIdx.x;
    pdl_wait();
    pdl_trigger();
    if (t >= nb) return;
    const int id = toks[t];
    if (id < 0 || id >= n_rows) {
        if (threadIdx.x == 0) atomicOr(status, ST_BAD_INDEX);
        for (int i = threadIdx.x; i < D; i += blockDim.x) x[(size_t)t * D + i] = 0.f;
        return;
    }
    const uint8_t* row = W + (size_t)id * row_bytes;
    for (int i = threadIdx.x; i < D; i += blockDim.x) x[(size_t)t * D + i] = dq_elem(row, type, i);
}

// ---- RMSNorm (qwen3moe.cpp:527-532): out = x * (1 / sqrtf(mean(x^2) + eps)) * w, one block per row
// (128 threads: the sum of squares in row_sumsq128's order, shared with the router launch's fused norm)
__global__ void __launch_bounds__(128) k_rmsnorm(const float* __restrict__ x, int ldx, const float* __restrict__ w,
                                                 float* __restrict__ out, int ldo, int n, float eps) {
    __shared__ float red4[4];
    pdl_wait();
    pdl_trigger();
    const float* xr = x + (size_t)blockIdx.x * ldx;
    const float sc = 1.0f / sqrtf(row_sumsq128(xr, n, red4) / (float)n + eps);
    float* o = out + (size_t)blockIdx.x * ldo;
    for (int i = threadIdx.x; i < n; i += 128) o[i] = __fmul_rn(__fmul_rn(xr[i], sc), w[i]);
}

// ---- fused: [combine of the previous MoE block] + RMSNorm + activation prep, one CTA per token row
// x[t] += sum_k w_k y[slot_k] (ascending expert order, as k_moe_combine), then xn = x * (1 / sqrtf(
// mean(x^2) + eps)) * w (qwen3moe.cpp:527-532), then xn in fragment form (XF) for the next GEMV and,
// optionally, xn itself. The row stays in shared memory between the steps.
constexpr int NP_NT = 1024;  // one thread per element pair of a 2048-wide row: every load in flight at once
__global__ void __launch_bounds__(NP_NT) k_norm_prep(NormPrepArgs a) {
    extern __shared__ __align__(16) float row[];  // [n]
    __shared__ float red[33];
    __shared__ int s_sl[32];
    __shared__ float s_w[32];
    pdl_wait();
    pdl_trigger();
    const int t = a.t0 + blockIdx.x, n = a.n;
    float* xr = a.x + (size_t)t * a.ldx;
    combine_norm_row(xr, a.y, a.y ? a.token_slots + (size_t)t * a.K : nullptr, a.slot_w, a.K, a.w, a.eps, n, row,
                     xr, a.xn ? a.xn + (size_t)blockIdx.x * n : nullptr, s_sl, s_w, red);
    const int r = blockIdx.x;  // XF row
    prep_row(row, n, const_cast<uint2*>(a.xf.frag) + (size_t)r * (n >> 5) * 12,
             const_cast<float*>(a.xf.sum) + (size_t)r * ((n >> 4) + XF_SUM_PAD),
             const_cast<uint8_t*>(a.xf.gs) + (size_t)r * xf_gs_bytes(n), red);
}

// ---- rotary table: cos/sin of (p0 + t) * inv_freq[i] in double, rounded to float (qwen3moe.cpp:937-943)
__global__ void k_rope_table(const DecodeState* st, const float* __restrict__ inv_freq, int half, int nb,
                             float2* __restrict__ cs) {
    const int t = blockIdx.x;
    pdl_wait();
    pdl_trigger();
    const int p = tok_pos(st, t);
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const double ang = (double)p * (double)inv_freq[i];
        cs[(size_t)t * half + i] = make_float2((float)cos(ang), (float)sin(ang));
    }
}

// One head (lane l holds elements l, l+32, ...): per-head RMSNorm with weights nw, then NeoX rotation
// with the row's cos/sin pairs (qwen3moe.cpp:951-972).
template <int HD>
__device__ __forceinline__ void head_norm_rope(float (&v)[HD / 32], const float* __restrict__ nw, float eps,
                                               const float2* __restrict__ cs_row, int lane) {
    constexpr int PER = HD / 32;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) ss = fmaf(v[j], v[j], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float sc = 1.0f / sqrtf(ss / (float)HD + eps);
#pragma unroll
    for (int j = 0; j < PER; j++) v[j] = __fmul_rn(__fmul_rn(v[j], sc), nw[lane + 32 * j]);
#pragma unroll
    for (int j = 0; j < PER / 2; j++) {
        const float2 r = cs_row[lane + 32 * j];
        const float a = v[j], b = v[j + PER / 2];
        v[j] = a * r.x - b * r.y;
        v[j + PER / 2] = a * r.y + b * r.x;
    }
}

// ---- per-head RMSNorm + NeoX rotation of q and k, KV-cache append (qwen3moe.cpp:951-972)
// qkv: [nb x (QD + 2 KD)] rows as the fused q|k|v projection writes them. One warp per (token, head)
// over the n_head q heads, n_kv k heads and n_kv v heads; lane l holds elements l, l+32, ... of the head.
template <int HD>
__global__ void k_qk_rope_kv(const float* __restrict__ qkv, int n_head, int n_kv, const float* __restrict__ qn,
                             const float* __restrict__ kn, float eps, const float2* __restrict__ cs,
                             const DecodeState* st, int nb, float* __restrict__ q_out, float* __restrict__ kc,
                             float* __restrict__ vc) {
    constexpr int PER = HD / 32, HALF = HD / 2;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nh = n_head + 2 * n_kv, QD = n_head * HD, KD = n_kv * HD;
    pdl_wait();
    pdl_trigger();
    if (gw >= nb * nh) return;
    const int t = gw / nh, h = gw - t * nh;
    const float* src = qkv + (size_t)t * (QD + 2 * KD) + (size_t)h * HD;
    const int pos = tok_pos(st, t);
    const size_t row = tok_base(st, t) + (size_t)pos;  // the token's cache row
    float v[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) v[j] = src[lane + 32 * j];
    if (h >= n_head + n_kv) {  // v head: copied into the cache unchanged
        float* dst = vc + row * KD + (size_t)(h - n_head - n_kv) * HD;
#pragma unroll
        for (int j = 0; j < PER; j++) dst[lane + 32 * j] = v[j];
        return;
    }
    head_norm_rope<HD>(v, h < n_head ? qn : kn, eps, cs + (size_t)t * HALF, lane);  // pairs (e, e + HD/2)
    float* dst = h < n_head ? q_out + (size_t)t * QD + (size_t)h * HD
                            : kc + row * KD + (size_t)(h - n_head) * HD;
#pragma unroll
    for (int j = 0; j < PER; j++) dst[lane + 32 * j] = v[j];
}

// ---- causal GQA attention (qwen3moe.cpp:976-1001), split over the context
// Block (kv head h, split y, token t) runs the GRP q heads sharing kv head h over context chunks
// y, y + nsplit, ... of ATT_CH positions with an online softmax and writes one partial (max, sum,
// unnormalised output) per q head; splits y >= ceil(np / ATT_CH) hold no positions of the token and write
// nothing. K/V chunks are staged in shared memory with cp.async (every thread's 16-byte copies in flight
// at once), rows padded by 4 floats for conflict-free row-parallel score reads. k_attn_merge_prep merges
// the splits of every head of a token row and puts the row in fragment form for the o-projection. The
// merges read the min(nsplit, ceil(np / ATT_CH)) records that exist: a split without positions would
// add exact zeros (weight 0, sum 0) and leave the maximum unchanged, so the merged row is the same as
// a merge over all nsplit records.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// One warp merges the nsplit partial records [m, l, o[HD]] of one (token, q head) (p: the first record):
// lane y holds split y's m and l (nsplit <= 128); v[j] = element lane + 32 j of sum_y e_y o_y / sum_y e_y l_y,
// e_y = expf(m_y - max m) (splits without positions weigh 0), the o sum in split order. The records are
// read eight splits at a time (independent loads in flight), or with EARLY and up to 16 splits all of
// them together with the m, l loads (64 more registers); CG: through L2 only (records written by other
// blocks of the same grid).
template <int HD, bool CG, bool EARLY>
__device__ __forceinline__ void merge_head(const float* __restrict__ p, int nsplit, float (&v)[HD / 32]) {
    constexpr int PER = HD / 32;
    const int lane = threadIdx.x & 31;
    auto ld = [](const float* a) { return CG ? __ldcg(a) : *a; };
    auto load8 = [&](int y0, float (&r)[8][PER]) {  // the o records of splits y0 .. y0 + 7
#pragma unroll
        for (int u = 0; u < 8; u++)
#pragma unroll
            for (int j = 0; j < PER; j++)
                r[u][j] = y0 + u < nsplit ? ld(p + (size_t)(y0 + u) * (HD + 2) + 2 + lane + 32 * j) : 0.f;
    };
    float mq[4], lq[4], M = -INFINITY;
#pragma unroll
    for (int q4 = 0; q4 < 4; q4++) {
        const int yy = lane + 32 * q4;
        mq[q4] = yy < nsplit ? ld(p + (size_t)yy * (HD + 2)) : -INFINITY;
        lq[q4] = yy < nsplit ? ld(p + (size_t)yy * (HD + 2) + 1) : 0.f;
    }
    float r0[8][PER], r1[8][PER];
    if (EARLY && nsplit <= 16) {  // up to 16 splits: every record's loads in flight together with m and l
        load8(0, r0);
        load8(8, r1);
    }
#pragma unroll
    for (int q4 = 0; q4 < 4; q4++) M = fmaxf(M, mq[q4]);
#pragma unroll
    for (int off = 16; off; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float eq[4], L = 0.f;
#pragma unroll
    for (int q4 = 0; q4 < 4; q4++) {
        eq[q4] = mq[q4] == -INFINITY ? 0.f : expf(mq[q4] - M);  // splits without positions weigh 0
        L = fmaf(lq[q4], eq[q4], L);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    float o[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) o[j] = 0.f;
    auto accumulate = [&](int y0, const float (&r)[8][PER]) {  // splits y0 .. y0 + 7 in order
        const int q4 = y0 >> 5;  // the eight splits share one lane group of eq
        const float eg = q4 == 0 ? eq[0] : q4 == 1 ? eq[1] : q4 == 2 ? eq[2] : eq[3];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const float e = __shfl_sync(0xffffffffu, eg, (y0 + u) & 31);
            if (y0 + u < nsplit && e != 0.f) {  // warp-uniform
#pragma unroll
                for (int j = 0; j < PER; j++) o[j] = fmaf(r[u][j], e, o[j]);
            }
        }
    };
    if (EARLY && nsplit <= 16) {
        accumulate(0, r0);
        accumulate(8, r1);
    } else {
        for (int y0 = 0; y0 < nsplit; y0 += 8) {
            float r[8][PER];
            load8(y0, r);
            accumulate(y0, r);
        }
    }
    const float inv = 1.0f / L;
#pragma unroll
    for (int j = 0; j < PER; j++) v[j] = o[j] * inv;
}

// One split holding a single chunk of n positions (the usual case: the context fits in nsplit chunks),
// for the grp q heads of a block, with the whole block. Scores: thread (position p, heads 2i, 2i+1), so a
// K float4 serves two heads; the softmax of head hq: warp hq % 8 with positions lane, lane + 32 per lane;
// PV: warp (four heads, elements lane + 32 j), so a V element serves four heads. Every record equals the
// one k_attention's per-warp loop writes for a first (and only) chunk: dots as four fmaf chains over
// d = i mod 4 then (a0 + a1) + (a2 + a3), times scale; m = the maximum; p = expf(s - m); l = the lane sums
// p[lane] + p[lane + 32] reduced by the same butterfly (= 0 * 0 + ls); o = even and odd fmaf chains from +0,
// then added. S: [grp][ATT_CH] scores, P: [ATT_CH][4 ceil(grp / 4)] probabilities. rec0: the record of the
// group's first head for this split; head hq's is at rec0 + hq * rstride.
template <int HD>
__device__ __forceinline__ void attn_one_chunk(const float* __restrict__ Ks, const float* __restrict__ Vs,
                                               const float* __restrict__ Qs, float* __restrict__ S,
                                               float* __restrict__ P, int grp, int n, float scale,
                                               float* __restrict__ rec0, size_t rstride) {
    constexpr int PER = HD / 32, RS = HD + 4;
    static_assert(ATT_CH == 64, "positions lane, lane + 32");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int GP2 = (grp + 1) / 2, GQ = (grp + 3) / 4, GP = 4 * GQ;
    for (int it = tid; it < GP2 * ATT_CH; it += ATT_NT) {
        const int p = it & (ATT_CH - 1), h0 = 2 * (it / ATT_CH);
        const float* q0 = Qs + h0 * HD;
        const float* q1 = h0 + 1 < grp ? q0 + HD : q0;
        float a[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        if (p < n) {
            const float* kr = Ks + p * RS;
#pragma unroll 8
            for (int d = 0; d < HD; d += 4) {
                const float4 kv4 = *reinterpret_cast<const float4*>(kr + d);
                const float4 qa = *reinterpret_cast<const float4*>(q0 + d);
                const float4 qb = *reinterpret_cast<const float4*>(q1 + d);
                a[0][0] = fmaf(qa.x, kv4.x, a[0][0]);
                a[0][1] = fmaf(qa.y, kv4.y, a[0][1]);
                a[0][2] = fmaf(qa.z, kv4.z, a[0][2]);
                a[0][3] = fmaf(qa.w, kv4.w, a[0][3]);
                a[1][0] = fmaf(qb.x, kv4.x, a[1][0]);
                a[1][1] = fmaf(qb.y, kv4.y, a[1][1]);
                a[1][2] = fmaf(qb.z, kv4.z, a[1][2]);
                a[1][3] = fmaf(qb.w, kv4.w, a[1][3]);
            }
        }
#pragma unroll
        for (int k = 0; k < 2; k++)
            if (h0 + k < grp) S[(h0 + k) * ATT_CH + p] = p < n ? ((a[k][0] + a[k][1]) + (a[k][2] + a[k][3])) * scale : -INFINITY;
    }
    __syncthreads();
    for (int hq = warp; hq < grp; hq += ATT_NT / 32) {
        const float s0 = S[hq * ATT_CH + lane], s1 = S[hq * ATT_CH + lane + 32];
        float mc = fmaxf(fmaxf(-INFINITY, s0), s1);
#pragma unroll
        for (int o = 16; o; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
        const float p0 = lane < n ? expf(s0 - mc) : 0.f, p1 = lane + 32 < n ? expf(s1 - mc) : 0.f;
        P[lane * GP + hq] = p0;
        P[(lane + 32) * GP + hq] = p1;
        float ls = 0.f;
        ls += p0;
        ls += p1;
#pragma unroll
        for (int o = 16; o; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
        if (lane == 0) {
            rec0[hq * rstride] = mc;
            rec0[hq * rstride + 1] = ls;
        }
    }
    __syncthreads();
    for (int it = warp; it < GQ * PER; it += ATT_NT / 32) {
        const int qd = it % GQ, e = lane + 32 * (it / GQ);
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        int r = 0;
#pragma unroll 4
        for (; r + 1 < n; r += 2) {
            const float4 pe = *reinterpret_cast<const float4*>(P + r * GP + 4 * qd);
            const float4 po = *reinterpret_cast<const float4*>(P + (r + 1) * GP + 4 * qd);
            const float v0 = Vs[r * RS + e], v1 = Vs[(r + 1) * RS + e];
            acc[0][0] = fmaf(pe.x, v0, acc[0][0]);
            acc[0][1] = fmaf(pe.y, v0, acc[0][1]);
            acc[0][2] = fmaf(pe.z, v0, acc[0][2]);
            acc[0][3] = fmaf(pe.w, v0, acc[0][3]);
            acc[1][0] = fmaf(po.x, v1, acc[1][0]);
            acc[1][1] = fmaf(po.y, v1, acc[1][1]);
            acc[1][2] = fmaf(po.z, v1, acc[1][2]);
            acc[1][3] = fmaf(po.w, v1, acc[1][3]);
        }
        if (r < n) {
            const float4 pe = *reinterpret_cast<const float4*>(P + r * GP + 4 * qd);
            const float v0 = Vs[r * RS + e];
            acc[0][0] = fmaf(pe.x, v0, acc[0][0]);
            acc[0][1] = fmaf(pe.y, v0, acc[0][1]);
            acc[0][2] = fmaf(pe.z, v0, acc[0][2]);
            acc[0][3] = fmaf(pe.w, v0, acc[0][3]);
        }
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (4 * qd + k < grp) rec0[(4 * qd + k) * rstride + 2 + e] = acc[0][k] + acc[1][k];
    }
}

template <int HD>
__global__ void __launch_bounds__(ATT_NT) k_attention(const float* __restrict__ q, float* __restrict__ kc,
                                                       float* __restrict__ vc, int n_head, int n_kv, float scale,
                                                       const DecodeState* st, int nsplit, float* __restrict__ part,
                                                       RopeFuse rf) {
    constexpr int PER = HD / 32, RS = HD + 4;
    extern __shared__ __align__(16) float smf[];
    float* Ks = smf;                          // [ATT_CH][RS]
    float* Vs = Ks + ATT_CH * RS;             // [ATT_CH][RS]
    float* Ps = Vs + ATT_CH * RS;             // [ATT_NT/32][ATT_CH] probabilities of the warp's current head
    float* Qs = Ps + (ATT_NT / 32) * ATT_CH;  // [GRP][HD]
    const int h = blockIdx.x, y = blockIdx.y, t = blockIdx.z;
    const int grp = n_head / n_kv, QD = n_head * HD, KD = n_kv * HD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = ATT_NT / 32;
    // A single-token step reads the position and stages its first chunk before the grid-dependency wait:
    // the position and the cache rows of earlier positions were written by kernels that completed before
    // the previous grid passed its own wait, and the step's own row is replaced below from the q|k|v row.
    // A prompt pass's rows come from the previous grid (k_qk_rope_kv): its copies start after the wait.
    int np = 0, nch = 0;
    size_t base = 0;  // first cache row of the token's sequence
    auto stage_chunk = [&](int c) {  // K/V rows of chunk c -> shared memory (cp.async, 16 bytes each)
        const int p0 = c * ATT_CH, n = min(ATT_CH, np - p0);
        for (int i = threadIdx.x; i < n * (HD / 4); i += ATT_NT) {
            const int r = i / (HD / 4), c4 = i - r * (HD / 4);
            const size_t g = (base + (size_t)(p0 + r)) * KD + (size_t)h * HD + 4 * c4;
            cp_async16(Ks + r * RS + 4 * c4, kc + g);
            cp_async16(Vs + r * RS + 4 * c4, vc + g);
        }
    };
    if (rf.qkv) {
        np = st->pos + t + 1;
        nch = (np + ATT_CH - 1) / ATT_CH;
        if (y < nch) stage_chunk(y);
    }
    pdl_wait();
    pdl_trigger();
    if (!rf.qkv) {
        np = tok_pos(st, t) + 1;  // causal: positions 0 .. the token's own
        nch = (np + ATT_CH - 1) / ATT_CH;
        base = tok_base(st, t);
    }
    // splits y >= nch hold no positions of this token: no record (the merges read the first
    // min(nsplit, nch) records only); a single-token step still counts the block for its merge
    if (y >= nch && !rf.cnt) return;
    if (!rf.qkv && y < nch) stage_chunk(y);  // the first chunk's copies fly while the q heads are prepared
    if (y >= nch) {
    } else if (rf.qkv) {  // single-token step: the group's q heads normalised and rotated here, from the q|k|v row
        for (int hq = warp; hq < grp; hq += nwarp) {
            const float* src = rf.qkv + (size_t)(h * grp + hq) * HD;
            float v[PER];
#pragma unroll
            for (int j = 0; j < PER; j++) v[j] = src[lane + 32 * j];
            head_norm_rope<HD>(v, rf.qn, rf.eps, rf.cs, lane);
#pragma unroll
            for (int j = 0; j < PER; j++) Qs[hq * HD + lane + 32 * j] = v[j];
        }
    } else {
        for (int i = threadIdx.x; i < grp * HD; i += ATT_NT) Qs[i] = q[(size_t)t * QD + (size_t)h * grp * HD + i];
    }
    // each warp owns q heads warp, warp + nwarp, ... (at most ATT_MAXH per warp)
    float m_run[ATT_MAXH], l_run[ATT_MAXH], o_run[ATT_MAXH][PER];
#pragma unroll
    for (int k = 0; k < ATT_MAXH; k++) {
        m_run[k] = -INFINITY;
        l_run[k] = 0.f;
#pragma unroll
        for (int j = 0; j < PER; j++) o_run[k][j] = 0.f;
    }
    for (int c = y; c < nch; c += nsplit) {
        const int p0 = c * ATT_CH, n = min(ATT_CH, np - p0);
        if (c != y) {
            __syncthreads();  // previous chunk fully consumed
            stage_chunk(c);
        }
        cp_async_wait_all();
        __syncthreads();  // every thread's copies have landed (the fused row below must not be overwritten)
        if (rf.qkv && np - 1 >= p0 && np - 1 < p0 + n && warp < 2) {
            // the step's own position lies in this chunk: its k (normalised, rotated) and v come straight
            // from the q|k|v row into the staged chunk and into the cache
            const int r = np - 1 - p0;
            const float* src = rf.qkv + (size_t)(n_head + (warp == 0 ? 0 : n_kv) + h) * HD;
            float v[PER];
#pragma unroll
            for (int j = 0; j < PER; j++) v[j] = src[lane + 32 * j];
            if (warp == 0) head_norm_rope<HD>(v, rf.kn, rf.eps, rf.cs, lane);
            float* srow = (warp == 0 ? Ks : Vs) + r * RS;
            float* grow = (warp == 0 ? kc : vc) + (size_t)(np - 1) * KD + (size_t)h * HD;
#pragma unroll
            for (int j = 0; j < PER; j++) {
                srow[lane + 32 * j] = v[j];
                grow[lane + 32 * j] = v[j];
            }
        }
        __syncthreads();
        if (nch <= nsplit) {  // this split's only chunk (block-uniform): the block-wide layout writes the records
            attn_one_chunk<HD>(Ks, Vs, Qs, Qs + grp * HD, Qs + grp * HD + grp * ATT_CH, grp, n, scale,
                               part + (((size_t)t * n_head + (size_t)h * grp) * nsplit + y) * (HD + 2),
                               (size_t)nsplit * (HD + 2));
            break;
        }
#pragma unroll
        for (int k = 0; k < ATT_MAXH; k++) {
            const int hq = warp + k * nwarp;
            if (hq >= grp) break;
            const float* qh = Qs + hq * HD;
            // scores: lane handles chunk positions lane, lane + 32
            float s[ATT_CH / 32];
            float mc = -INFINITY;
#pragma unroll
            for (int r = 0; r < ATT_CH / 32; r++) {
                const int pr = lane + 32 * r;
                float acc = 0.f;
                if (pr < n) {
                    const float* kr = Ks + pr * RS;
                    float a4[4] = {0.f, 0.f, 0.f, 0.f};  // four chains: the dot is latency-bound otherwise
#pragma unroll 8
                    for (int d = 0; d < HD; d += 4) {
                        const float4 kv4 = *reinterpret_cast<const float4*>(kr + d);
                        const float4 q4 = *reinterpret_cast<const float4*>(qh + d);
                        a4[0] = fmaf(q4.x, kv4.x, a4[0]);
                        a4[1] = fmaf(q4.y, kv4.y, a4[1]);
                        a4[2] = fmaf(q4.z, kv4.z, a4[2]);
                        a4[3] = fmaf(q4.w, kv4.w, a4[3]);
                    }
                    acc = (a4[0] + a4[1]) + (a4[2] + a4[3]);
                    s[r] = acc * scale;
                    mc = fmaxf(mc, s[r]);
                } else {
                    s[r] = -INFINITY;
                }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
            const float m_new = fmaxf(m_run[k], mc);
            const float alpha = expf(m_run[k] - m_new);  // 0 on the first chunk (m_run = -inf)
            float ls = 0.f;
#pragma unroll
            for (int r = 0; r < ATT_CH / 32; r++) {
                const float p = (lane + 32 * r) < n ? expf(s[r] - m_new) : 0.f;
                Ps[warp * ATT_CH + lane + 32 * r] = p;
                ls += p;
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
            l_run[k] = l_run[k] * alpha + ls;
            m_run[k] = m_new;
            __syncwarp();
            float acc[2][PER];  // even / odd positions: two chains per element
#pragma unroll
            for (int j = 0; j < PER; j++) {
                acc[0][j] = o_run[k][j] * alpha;
                acc[1][j] = 0.f;
            }
            int r = 0;
#pragma unroll 4
            for (; r + 1 < n; r += 2) {
                const float p0 = Ps[warp * ATT_CH + r], p1 = Ps[warp * ATT_CH + r + 1];
                const float* v0 = Vs + r * RS;
                const float* v1 = v0 + RS;
#pragma unroll
                for (int j = 0; j < PER; j++) {
                    acc[0][j] = fmaf(p0, v0[lane + 32 * j], acc[0][j]);
                    acc[1][j] = fmaf(p1, v1[lane + 32 * j], acc[1][j]);
                }
            }
            if (r < n) {
                const float p0 = Ps[warp * ATT_CH + r];
#pragma unroll
                for (int j = 0; j < PER; j++) acc[0][j] = fmaf(p0, Vs[r * RS + lane + 32 * j], acc[0][j]);
            }
#pragma unroll
            for (int j = 0; j < PER; j++) o_run[k][j] = acc[0][j] + acc[1][j];
            __syncwarp();
        }
    }
    // partial record per (token, q head, split): [m, l, o[HD]]
#pragma unroll
    for (int k = 0; k < ATT_MAXH; k++) {
        const int hq = warp + k * nwarp;
        if (hq >= grp || y >= nch || nch <= nsplit) break;  // (nch <= nsplit: written by attn_one_chunk)
        float* pr = part + (((size_t)t * n_head + (size_t)h * grp + hq) * nsplit + y) * (HD + 2);
        if (lane == 0) {
            pr[0] = m_run[k];
            pr[1] = l_run[k];
        }
#pragma unroll
        for (int j = 0; j < PER; j++) pr[2 + lane + 32 * j] = o_run[k][j];
    }
    if (rf.cnt) {  // single-token step: the last split block of (t, kv head h) merges the group's q heads
        __shared__ bool s_last;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = atomicAdd(&rf.cnt[t * n_kv + h], 1) == (int)gridDim.y - 1;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        for (int hq = warp; hq < grp; hq += nwarp) {
            float v[PER];
            merge_head<HD, true, true>(part + ((size_t)t * n_head + (size_t)h * grp + hq) * nsplit * (HD + 2),
                                       min(nsplit, nch), v);
#pragma unroll
            for (int j = 0; j < PER; j++) rf.att[(size_t)t * QD + (size_t)(h * grp + hq) * HD + lane + 32 * j] = v[j];
        }
        if (threadIdx.x == 0) rf.cnt[t * n_kv + h] = 0;  // counted again by the next launch
    }
}

// ---- prompt-pass attention when every split holds one chunk (nch <= nsplit for every token of the pass)
// Block (kv head h, chunk c, tokens 8z .. 8z + 7) stages chunk c's K/V rows once for its tokens; warp w
// takes q heads 4 (w % WPT) .. + 3 of one token (WPT = ceil(grp / 4) warps per token, 8 / WPT tokens at
// a time). Each K float4 a lane loads serves four heads' dot products and each V element four heads'
// sums, so shared-memory traffic per head is about a quarter of k_attention's. The record of (token,
// head, split c) is k_attention's for a split with the single chunk c, operation for operation: scores
// as four fmaf chains over d = i mod 4 then (a0 + a1) + (a2 + a3), times scale; the maximum over the
// chunk; p = expf(s - m); the sum as lane value p[lane] + p[lane + 32] reduced by the same butterfly;
// o as two fmaf chains over even and odd positions from +0, then added. The merge therefore sees the
// same records whichever kernel wrote them.
constexpr int AC_TG = 8;  // tokens per block
size_t attn_chunk_smem(int hd, int grp) {
    return ((size_t)2 * ATT_CH * (hd + 4) + (size_t)AC_TG * grp * (hd + 4) + (size_t)(ATT_NT / 32) * ATT_CH * 4) *
           sizeof(float);
}
template <int HD>
__global__ void __launch_bounds__(ATT_NT) k_attn_chunk(const float* __restrict__ q, const float* __restrict__ kc,
                                                        const float* __restrict__ vc, int n_head, int n_kv, float scale,
                                                        const DecodeState* st, int nb, int nsplit,
                                                        float* __restrict__ part) {
    constexpr int PER = HD / 32, RS = HD + 4, QS = HD + 4;
    extern __shared__ __align__(16) float smf[];
    const int grp = n_head / n_kv, QD = n_head * HD, KD = n_kv * HD;
    float* Ks = smf;                          // [ATT_CH][RS]
    float* Vs = Ks + ATT_CH * RS;             // [ATT_CH][RS]
    float* Qs = Vs + ATT_CH * RS;             // [AC_TG][grp][QS]
    float* Ps = Qs + AC_TG * grp * QS;        // [warp][ATT_CH][4]
    const int h = blockIdx.x, c = blockIdx.y, t0 = blockIdx.z * AC_TG;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    const int pos = st->pos, p0 = c * ATT_CH, tn = min(AC_TG, nb - t0);
    // token t has positions 0 .. pos + t: chunk c holds some of them iff pos + t >= p0
    const int tf = max(t0, p0 - pos);
    if (tf >= t0 + tn) return;
    const int n_max = min(ATT_CH, pos + t0 + tn - p0);
    for (int i = threadIdx.x; i < n_max * (HD / 4); i += ATT_NT) {
        const int r = i / (HD / 4), c4 = i - r * (HD / 4);
        const size_t g = (size_t)(p0 + r) * KD + (size_t)h * HD + 4 * c4;
        cp_async16(Ks + r * RS + 4 * c4, kc + g);
        cp_async16(Vs + r * RS + 4 * c4, vc + g);
    }
    for (int i = threadIdx.x; i < tn * grp * (HD / 4); i += ATT_NT) {
        const int row = i / (HD / 4), c4 = i - row * (HD / 4), tt = row / grp, hq = row - tt * grp;
        cp_async16(Qs + row * QS + 4 * c4, q + (size_t)(t0 + tt) * QD + (size_t)(h * grp + hq) * HD + 4 * c4);
    }
    cp_async_wait_all();
    __syncthreads();
    const int wpt = (grp + 3) / 4, nslot = (ATT_NT / 32) / wpt, slot = warp / wpt, h4 = 4 * (warp - slot * wpt);
    if (slot >= nslot) return;
    float* pw = Ps + warp * ATT_CH * 4;
    for (int t = tf + slot; t < t0 + tn; t += nslot) {
        const int n = min(ATT_CH, pos + t + 1 - p0);  // positions of token t in this chunk
        const float* qb = Qs + ((t - t0) * grp + h4) * QS;
        // scores of positions lane, lane + 32 for the warp's four heads
        float s[2][4];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int pr = lane + 32 * r;
            float a[4][4];
#pragma unroll
            for (int k = 0; k < 4; k++) a[k][0] = a[k][1] = a[k][2] = a[k][3] = 0.f;
            if (pr < n) {
                const float* kr = Ks + pr * RS;
#pragma unroll 4
                for (int d = 0; d < HD; d += 4) {
                    const float4 kv4 = *reinterpret_cast<const float4*>(kr + d);
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const float4 q4 = *reinterpret_cast<const float4*>(qb + k * QS + d);
                        a[k][0] = fmaf(q4.x, kv4.x, a[k][0]);
                        a[k][1] = fmaf(q4.y, kv4.y, a[k][1]);
                        a[k][2] = fmaf(q4.z, kv4.z, a[k][2]);
                        a[k][3] = fmaf(q4.w, kv4.w, a[k][3]);
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < 4; k++) s[r][k] = pr < n ? ((a[k][0] + a[k][1]) + (a[k][2] + a[k][3])) * scale : -INFINITY;
        }
        float m[4], l[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float mc = fmaxf(s[0][k], s[1][k]);
#pragma unroll
            for (int o = 16; o; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
            m[k] = mc;
            float ls = 0.f;
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const float p = (lane + 32 * r) < n ? expf(s[r][k] - mc) : 0.f;
                pw[(lane + 32 * r) * 4 + k] = p;
                ls += p;
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
            l[k] = ls;
        }
        __syncwarp();
        float acc[2][4][PER];
#pragma unroll
        for (int e = 0; e < 2; e++)
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int j = 0; j < PER; j++) acc[e][k][j] = 0.f;
        int r = 0;
#pragma unroll 2
        for (; r + 1 < n; r += 2) {
            const float4 pe = *reinterpret_cast<const float4*>(pw + r * 4), po = *reinterpret_cast<const float4*>(pw + r * 4 + 4);
            const float pev[4] = {pe.x, pe.y, pe.z, pe.w}, pov[4] = {po.x, po.y, po.z, po.w};
#pragma unroll
            for (int j = 0; j < PER; j++) {
                const float v0 = Vs[r * RS + lane + 32 * j], v1 = Vs[(r + 1) * RS + lane + 32 * j];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    acc[0][k][j] = fmaf(pev[k], v0, acc[0][k][j]);
                    acc[1][k][j] = fmaf(pov[k], v1, acc[1][k][j]);
                }
            }
        }
        if (r < n) {
            const float4 pe = *reinterpret_cast<const float4*>(pw + r * 4);
            const float pev[4] = {pe.x, pe.y, pe.z, pe.w};
#pragma unroll
            for (int j = 0; j < PER; j++) {
                const float v0 = Vs[r * RS + lane + 32 * j];
#pragma unroll
                for (int k = 0; k < 4; k++) acc[0][k][j] = fmaf(pev[k], v0, acc[0][k][j]);
            }
        }
        __syncwarp();  // pw is rewritten by the warp's next token
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if (h4 + k >= grp) break;
            float* pr = part + (((size_t)t * n_head + (size_t)h * grp + h4 + k) * nsplit + c) * (HD + 2);
            if (lane == 0) {
                pr[0] = m[k];
                pr[1] = l[k];
            }
#pragma unroll
            for (int j = 0; j < PER; j++) pr[2 + lane + 32 * j] = acc[0][k][j] + acc[1][k][j];
        }
    }
}

// ---- split merge of every head of a token row: out = sum_y o_y e^(m_y - M) / sum_y l_y e^(m_y - M),
// written to att (fp32) and, in fragment form, to xf for the o-projection. One CTA per token row
// (32 warps, warp w merges heads w, w + 32, ...; the row stays in shared memory for the prep).
constexpr int MP_NT = 1024;
template <int HD>
__global__ void __launch_bounds__(MP_NT) k_attn_merge_prep(const float* __restrict__ part, int n_head, int nsplit,
                                                           const DecodeState* st, float* __restrict__ att, XF xf) {
    constexpr int PER = HD / 32;
    extern __shared__ __align__(16) float mrow[];  // [n_head * HD]
    __shared__ float red[33];
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, QD = n_head * HD;
    const int nvalid = min(nsplit, (tok_pos(st, t) + ATT_CH) / ATT_CH);  // splits holding positions 0 .. pos
    for (int hq = warp; hq < n_head; hq += MP_NT / 32) {
        float v[PER];
        merge_head<HD, false, false>(part + ((size_t)t * n_head + hq) * nsplit * (HD + 2), nvalid, v);
#pragma unroll
        for (int j = 0; j < PER; j++) {
            mrow[hq * HD + lane + 32 * j] = v[j];
            att[(size_t)t * QD + hq * HD + lane + 32 * j] = v[j];
        }
    }
    __syncthreads();
    prep_row(mrow, QD, const_cast<uint2*>(xf.frag) + (size_t)t * (QD >> 5) * 12,
             const_cast<float*>(xf.sum) + (size_t)t * ((QD >> 4) + XF_SUM_PAD),
             const_cast<uint8_t*>(xf.gs) + (size_t)t * xf_gs_bytes(QD), red);
}

// ---- argmax: first maximum, as std::max_element (qwen3moe.cpp:1103)
// Blocks reduce strided slices to (value, index); the last block to finish reduces the block results,
// records the token in the decode state (next input, output history) and advances the position.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__global__ void __launch_bounds__(ARGMAX_NT) k_argmax(const float* __restrict__ lg, int n, float2* __restrict__ blk,
                                                       DecodeState* st, int advance) {
    __shared__ float sv[ARGMAX_NT / 32];
    __shared__ int si[ARGMAX_NT / 32];
    __shared__ bool last;
    pdl_wait();
    pdl_trigger();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = blockIdx.x * ARGMAX_NT + threadIdx.x; i < n; i += gridDim.x * ARGMAX_NT) {
        const float v = lg[i];
        if (better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    auto warp_best = [&]() {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
    };
    auto block_best = [&]() {
        warp_best();
        const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
        __syncthreads();
        if (lane == 0) {
            sv[w] = bv;
            si[w] = bi;
        }
        __syncthreads();
        bv = lane < ARGMAX_NT / 32 ? sv[lane] : -INFINITY;
        bi = lane < ARGMAX_NT / 32 ? si[lane] : 0x7fffffff;
        warp_best();
    };
    block_best();
    if (threadIdx.x == 0) {
        blk[blockIdx.x] = make_float2(bv, __int_as_float(bi));
        __threadfence();
        last = atomicAdd(&st->ticket, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    bv = -INFINITY;
    bi = 0x7fffffff;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += ARGMAX_NT) {
        const float2 r = __ldcg(blk + b);
        const int ri = __float_as_int(r.y);
        if (better(r.x, ri, bv, bi)) {
            bv = r.x;
            bi = ri;
        }
    }
    block_best();
    if (threadIdx.x == 0) {
        if (bi == 0x7fffffff) bi = 0;  // every logit NaN: max_element returns the first element
        st->ticket = 0;
        st->token = bi;
        if (st->n_out < st->cap_out) st->out[st->n_out] = bi;
        st->n_out++;
        if (advance) st->pos += 1;
    }
}

// One block per row: the first maximum of the row (the order `better` defines), for multi-sequence steps.
__global__ void __launch_bounds__(ARGMAX_NT) k_argmax_rows(const float* __restrict__ lg, int n, int ld,
                                                            int* __restrict__ out) {
    __shared__ float sv[ARGMAX_NT / 32];
    __shared__ int si[ARGMAX_NT / 32];
    pdl_wait();
    pdl_trigger();
    const float* row = lg + (size_t)blockIdx.x * ld;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += ARGMAX_NT) {
        const float v = row[i];
        if (better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[w] = bv;
        si[w] = bi;
    }
    __syncthreads();
    if (w == 0) {
        bv = lane < ARGMAX_NT / 32 ? sv[lane] : -INFINITY;
        bi = lane < ARGMAX_NT / 32 ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
    }
}

// pos += n (host-enqueued position advance after a prompt chunk, kept on the device)
__global__ void k_advance(DecodeState* st, int n) {
    pdl_wait();
    st->pos += n;
}

// ---- launchers ---------------------------------------------------------------------------------
cudaError_t launch_embed(const uint8_t* W, int type, size_t rb, int D, int n_rows, const int* toks, int nb, float* x,
                         int* status, cudaStream_t s) {
    return launch_pdl(k_embed, dim3(nb), dim3(256), 0, s, W, type, rb, D, n_rows, toks, nb, x, status);
}
cudaError_t launch_rmsnorm(const float* x, int ldx, const float* w, float* out, int ldo, int rows, int n, float eps,
                           cudaStream_t s) {
    if (n % 4 || ldx % 4) return cudaErrorInvalidValue;
    return launch_pdl(k_rmsnorm, dim3(rows), dim3(128), 0, s, x, ldx, w, out, ldo, n, eps);
}
cudaError_t launch_norm_prep(const NormPrepArgs& a, int rows, cudaStream_t s) {
    if (rows < 1 || a.n % 256 || (a.y && (a.K < 1 || a.K > 32))) return cudaErrorInvalidValue;
    const size_t smem = (size_t)a.n * 4;
    if (smem > 48 * 1024) {
        static size_t cur = 0;
        if (smem > cur) {
            cudaError_t e = cudaFuncSetAttribute(k_norm_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            cur = smem;
        }
    }
    return launch_pdl(k_norm_prep, dim3(rows), dim3(NP_NT), smem, s, a);
}
cudaError_t launch_rope_table(const DecodeState* st, const float* inv_freq, int half, int nb, float2* cs,
                              cudaStream_t s) {
    return launch_pdl(k_rope_table, dim3(nb), dim3(64), 0, s, st, inv_freq, half, nb, cs);
}
cudaError_t launch_qk_rope_kv(int hd, const float* qkv, int n_head, int n_kv, const float* qn, const float* kn,
                              float eps, const float2* cs, const DecodeState* st, int nb, float* q_out, float* kc,
                              float* vc, cudaStream_t s) {
    const int warps = nb * (n_head + 2 * n_kv), grid = (warps + 7) / 8;
    if (hd == 128)
        return launch_pdl(k_qk_rope_kv<128>, dim3(grid), dim3(256), 0, s, qkv, n_head, n_kv, qn, kn, eps, cs, st, nb,
                          q_out, kc, vc);
    if (hd == 64)
        return launch_pdl(k_qk_rope_kv<64>, dim3(grid), dim3(256), 0, s, qkv, n_head, n_kv, qn, kn, eps, cs, st, nb,
                          q_out, kc, vc);
    return cudaErrorInvalidValue;
}
size_t attn_smem(int hd, int grp) {  // K, V, per-warp P, Q, then attn_one_chunk's S and P
    return ((size_t)2 * ATT_CH * (hd + 4) + (size_t)(ATT_NT / 32) * ATT_CH + (size_t)grp * hd + (size_t)grp * ATT_CH +
            (size_t)ATT_CH * 4 * ((grp + 3) / 4)) *
           sizeof(float);
}
template <int HD>
static cudaError_t attn_as(const float* q, float* kc, float* vc, int n_head, int n_kv, float scale,
                           const DecodeState* st, int nb, int nsplit, float* part, float* att, const XF& xf,
                           const RopeFuse& rf, int pos_host, cudaStream_t s) {
    cudaError_t e;
    const int nch_max = pos_host >= 0 ? (pos_host + nb + ATT_CH - 1) / ATT_CH : 0;
    if (!rf.qkv && !rf.cnt && nb > 1 && pos_host >= 0 && nch_max <= nsplit && n_head / n_kv <= 32) {
        // prompt pass at a known position, one chunk per split: chunk-shared kernel
        const size_t smem = attn_chunk_smem(HD, n_head / n_kv);
        static size_t ccur = 0;
        if (smem > ccur) {
            e = cudaFuncSetAttribute(k_attn_chunk<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            ccur = smem;
        }
        e = launch_pdl(k_attn_chunk<HD>, dim3(n_kv, nch_max, (nb + AC_TG - 1) / AC_TG), dim3(ATT_NT), smem, s, q,
                       (const float*)kc, (const float*)vc, n_head, n_kv, scale, st, nb, nsplit, part);
    } else {
        const size_t smem = attn_smem(HD, n_head / n_kv);
        static size_t cur = 0;
        if (smem > cur) {
            e = cudaFuncSetAttribute(k_attention<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            cur = smem;
        }
        e = launch_pdl(k_attention<HD>, dim3(n_kv, nsplit, nb), dim3(ATT_NT), smem, s, q, kc, vc, n_head, n_kv, scale,
                       st, nsplit, part, rf);
    }
    if (e != cudaSuccess || rf.cnt) return e;  // merged by the attention launch itself
    const size_t msmem = (size_t)n_head * HD * 4;
    static size_t mcur = 0;
    if (msmem > 48 * 1024 && msmem > mcur) {
        e = cudaFuncSetAttribute(k_attn_merge_prep<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem);
        if (e != cudaSuccess) return e;
        mcur = msmem;
    }
    return launch_pdl(k_attn_merge_prep<HD>, dim3(nb), dim3(MP_NT), msmem, s, part, n_head, nsplit, st, att, xf);
}
cudaError_t launch_attention(int hd, const float* q, float* kc, float* vc, int n_head, int n_kv, float scale,
                             const DecodeState* st, int nb, int nsplit, float* part, float* att, const XF& xf,
                             const RopeFuse& rf, int pos_host, cudaStream_t s) {
    if (n_head % n_kv || n_head / n_kv > ATT_MAXH * (ATT_NT / 32) || nsplit < 1 || nsplit > 128 ||
        (rf.qkv && nb != 1) || (rf.cnt && (nb != 1 || !rf.att)) || (n_head * hd) % 256)
        return cudaErrorInvalidValue;
    if (hd == 128) return attn_as<128>(q, kc, vc, n_head, n_kv, scale, st, nb, nsplit, part, att, xf, rf, pos_host, s);
    if (hd == 64) return attn_as<64>(q, kc, vc, n_head, n_kv, scale, st, nb, nsplit, part, att, xf, rf, pos_host, s);
    return cudaErrorInvalidValue;
}
cudaError_t launch_argmax(const float* lg, int n, float2* blk, int nblk, DecodeState* st, int advance, cudaStream_t s) {
    return launch_pdl(k_argmax, dim3(nblk), dim3(ARGMAX_NT), 0, s, lg, n, blk, st, advance);
}
cudaError_t launch_argmax_rows(const float* lg, int n, int ld, int rows, int* out, cudaStream_t s) {
    if (rows < 1) return cudaSuccess;
    return launch_pdl(k_argmax_rows, dim3(rows), dim3(ARGMAX_NT), 0, s, lg, n, ld, out);
}

cudaError_t launch_advance(DecodeState* st, int n, cudaStream_t s) {
    return launch_pdl(k_advance, dim3(1), dim3(1), 0, s, st, n);
}

}  // namespace eb
