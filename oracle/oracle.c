/* oracle/oracle.c -- TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's expert hot path.
 *
 * Used by tests/ as the parity checker and by bench.py as the "port" CPU baseline; never by the product.
 * Each function cites the reference lines (qwen3moe.cpp) whose behaviour it restates. The arithmetic
 * follows the reference's order where it decides rounding that parity depends on (routing: expf of
 * l - max, rank-order renormalisation, expert-ascending accumulation); inner dot products are plain
 * sequential fp32 sums.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- fp16 -> fp32, restating f16_slow (qwen3moe.cpp:56-63) ------------------------------------ */
float orc_f16(uint16_t h) {
    unsigned s = (h >> 15) & 1u, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    float v;
    if (e == 0) v = ldexpf((float)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = ldexpf((float)(m | 0x400u), (int)e - 25);
    return s ? -v : v;
}
static float rd16(const uint8_t* p) { return orc_f16((uint16_t)(p[0] | (p[1] << 8))); }

int orc_block_size(int type) {
    switch (type) {
        case ORC_F32: case ORC_F16: case ORC_Q8_0: return 32;
        case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K: return 256;
        default: return 0;
    }
}
int orc_block_bytes(int type) {
    switch (type) {
        case ORC_F32: return 128;
        case ORC_F16: return 64;
        case ORC_Q8_0: return 34;
        case ORC_Q4_K: return 144;
        case ORC_Q5_K: return 176;
        case ORC_Q6_K: return 210;
        default: return 0;
    }
}

/* 6-bit scale/min pair j (0..7) of a K-quant header, restating scale_min_k4 (qwen3moe.cpp:133-141). */
static void kq_scale_min(int j, const uint8_t* q, int* sc, int* mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* Q4_K super-block: d, dmin, 12 scale bytes, 128 nibble bytes (dq_q4_k, qwen3moe.cpp:142-158). */
static void dq_q4k(const uint8_t* b, float* y) {
    const float d = rd16(b), dmin = rd16(b + 2);
    const uint8_t* qs = b + 16;
    for (int c = 0; c < 4; c++) {
        int s0, m0, s1, m1;
        kq_scale_min(2 * c, b + 4, &s0, &m0);
        kq_scale_min(2 * c + 1, b + 4, &s1, &m1);
        const float d0 = d * s0, o0 = dmin * m0, d1 = d * s1, o1 = dmin * m1;
        for (int l = 0; l < 32; l++) {
            y[64 * c + l] = d0 * (qs[32 * c + l] & 0x0f) - o0;
            y[64 * c + 32 + l] = d1 * (qs[32 * c + l] >> 4) - o1;
        }
    }
}

/* Q5_K super-block: Q4_K plus one high bit per weight in qh[32] (dq_q5_k, qwen3moe.cpp:159-179). */
static void dq_q5k(const uint8_t* b, float* y) {
    const float d = rd16(b), dmin = rd16(b + 2);
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int c = 0; c < 4; c++) {
        int s0, m0, s1, m1;
        kq_scale_min(2 * c, b + 4, &s0, &m0);
        kq_scale_min(2 * c + 1, b + 4, &s1, &m1);
        const float d0 = d * s0, o0 = dmin * m0, d1 = d * s1, o1 = dmin * m1;
        for (int l = 0; l < 32; l++) {
            int lo = (qs[32 * c + l] & 0x0f) + (((qh[l] >> (2 * c)) & 1) ? 16 : 0);
            int hi = (qs[32 * c + l] >> 4) + (((qh[l] >> (2 * c + 1)) & 1) ? 16 : 0);
            y[64 * c + l] = d0 * lo - o0;
            y[64 * c + 32 + l] = d1 * hi - o1;
        }
    }
}

/* Q6_K super-block: 4-bit low parts ql[128], 2-bit high parts qh[64], int8 scales[16], fp16 d at 208
 * (dq_q6_k, qwen3moe.cpp:180-202). */
static void dq_q6k(const uint8_t* b, float* y) {
    const float d = rd16(b + 208);
    const int8_t* sc = (const int8_t*)(b + 192);
    for (int h = 0; h < 2; h++) {
        const uint8_t* ql = b + 64 * h;
        const uint8_t* qh = b + 128 + 32 * h;
        const int8_t* s = sc + 8 * h;
        float* o = y + 128 * h;
        for (int l = 0; l < 32; l++) {
            const int g = l / 16;
            int q1 = (int)((ql[l] & 0x0f) | ((qh[l] & 3) << 4)) - 32;
            int q2 = (int)((ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            o[l] = d * s[g] * q1;
            o[l + 32] = d * s[g + 2] * q2;
            o[l + 64] = d * s[g + 4] * q3;
            o[l + 96] = d * s[g + 6] * q4;
        }
    }
}

/* Q8_0 block: fp16 d + 32 int8 (dq_q8_0, qwen3moe.cpp:128-132). */
static void dq_q80(const uint8_t* b, float* y) {
    const float d = rd16(b);
    for (int i = 0; i < 32; i++) y[i] = d * (float)(int8_t)b[2 + i];
}

static void dq_block(int type, const uint8_t* b, float* y) {
    switch (type) {
        case ORC_F32: memcpy(y, b, 128); break;
        case ORC_F16: for (int i = 0; i < 32; i++) y[i] = rd16(b + 2 * i); break;
        case ORC_Q8_0: dq_q80(b, y); break;
        case ORC_Q4_K: dq_q4k(b, y); break;
        case ORC_Q5_K: dq_q5k(b, y); break;
        case ORC_Q6_K: dq_q6k(b, y); break;
        default: break;
    }
}

int orc_dequant_row(int type, const uint8_t* row, int64_t ne0, float* y) {
    const int bs = orc_block_size(type), bb = orc_block_bytes(type);
    if (!bs || ne0 % bs) return -1;
    for (int64_t b = 0; b < ne0 / bs; b++) dq_block(type, row + b * bb, y + b * bs);
    return 0;
}

/* matmul (qwen3moe.cpp:397-419): every row is dequantised one block at a time and dotted against all
 * nb tokens; rows are independent, so they are split across OpenMP threads. */
int orc_matmul(const uint8_t* w, int type, int64_t ne0, int64_t ne1, size_t row_bytes, const float* x, int nb,
               int ldx, float* out, int ldo) {
    const int bs = orc_block_size(type), bb = orc_block_bytes(type);
    if (!w || !x || !out || !bs || ne0 % bs || nb < 1 || ldx < ne0 || ldo < ne1) return -1;
    const int64_t nblk = ne0 / bs;
    int bad = 0;
#pragma omp parallel
    {
        float tmp[256];
        float* acc = (float*)malloc(sizeof(float) * (size_t)nb);
        if (!acc) {
#pragma omp atomic write
            bad = 1;
        }
#pragma omp for schedule(static)
        for (int64_t r = 0; r < ne1; r++) {
            if (!acc) continue;
            const uint8_t* wr = w + (size_t)r * row_bytes;
            for (int t = 0; t < nb; t++) acc[t] = 0.f;
            for (int64_t b = 0; b < nblk; b++) {
                dq_block(type, wr + b * bb, tmp);
                for (int t = 0; t < nb; t++) {
                    const float* xb = x + (size_t)t * ldx + b * bs;
                    float s = 0.f;
                    for (int i = 0; i < bs; i++) s += tmp[i] * xb[i];
                    acc[t] += s;
                }
            }
            for (int t = 0; t < nb; t++) out[(size_t)t * ldo + r] = acc[t];
        }
        free(acc);
    }
    return bad ? -2 : 0;
}

/* rmsnorm (qwen3moe.cpp:527-532). */
void orc_rmsnorm(const float* x, const float* w, float* out, int n, float eps) {
    float ss = 0.f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float sc = 1.0f / sqrtf(ss / n + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * sc * w[i];
}

/* Routing of one token (qwen3moe.cpp:1012-1022): r <- expf(l - max) (glibc expf, as the reference);
 * the top K under the strict order "larger r first, equal r -> lower index first" (the partial_sort
 * comparator at :1016), then w = r / (sum of the K chosen r in rank order). */
void orc_route_token(float* r, int E, int K, int* ids, float* w) {
    float mx = r[0];
    for (int e = 1; e < E; e++)
        if (r[e] > mx) mx = r[e];
    for (int e = 0; e < E; e++) r[e] = expf(r[e] - mx);
    unsigned char used[4096];
    memset(used, 0, (size_t)E);
    for (int i = 0; i < K; i++) {
        int best = -1;
        for (int e = 0; e < E; e++) {
            if (used[e]) continue;
            if (best < 0 || r[e] > r[best]) best = e; /* strictly larger; ties keep the lower index */
        }
        used[best] = 1;
        ids[i] = best;
    }
    float tot = 0.f;
    for (int i = 0; i < K; i++) tot += r[ids[i]];
    for (int i = 0; i < K; i++) w[i] = r[ids[i]] / tot;
}

/* MoE block (qwen3moe.cpp:1008-1069). Token lists per expert keep token order (:1020); experts are
 * processed in ascending id (:1025); each expert's rows are gathered (:1029), projected by gate and up,
 * combined with SiLU(g)*u (:1056-1059), projected by down (:1060) and added with the routing weight
 * into a zeroed per-token accumulator (:1024, :1062-1067), which is then added to x (:1069). */
int orc_moe_layer(int T, int D, int FF, int E, int K, const float* xn, const float* logits, const float* router_w,
                  const uint8_t* const* gate, const uint8_t* const* up, const uint8_t* const* down, int gt, int ut,
                  int dt, size_t grb, size_t urb, size_t drb, float* x, int* trace_ids, float* trace_w) {
    if (T < 1 || E < 1 || E > 4096 || K < 1 || K > E || !xn || !x || !gate || !up || !down) return -1;
    if (!logits && !router_w) return -1;
    int rc = 0;
    float* rl = (float*)malloc(sizeof(float) * (size_t)T * E);
    int* ids = (int*)malloc(sizeof(int) * (size_t)T * K);
    float* wts = (float*)malloc(sizeof(float) * (size_t)T * K);
    int* cnt = (int*)calloc((size_t)E + 1, sizeof(int));
    int* lst_tok = (int*)malloc(sizeof(int) * (size_t)T * K);
    float* lst_w = (float*)malloc(sizeof(float) * (size_t)T * K);
    float* tmp = (float*)calloc((size_t)T * D, sizeof(float));
    float* xs = (float*)malloc(sizeof(float) * (size_t)T * D);
    float* g = (float*)malloc(sizeof(float) * (size_t)T * FF);
    float* u = (float*)malloc(sizeof(float) * (size_t)T * FF);
    float* y = (float*)malloc(sizeof(float) * (size_t)T * D);
    if (!rl || !ids || !wts || !cnt || !lst_tok || !lst_w || !tmp || !xs || !g || !u || !y) { rc = -2; goto out; }

    if (logits) memcpy(rl, logits, sizeof(float) * (size_t)T * E);
    else if ((rc = orc_matmul((const uint8_t*)router_w, ORC_F32, D, E, (size_t)D * 4, xn, T, D, rl, E))) goto out;
    for (int t = 0; t < T; t++) orc_route_token(rl + (size_t)t * E, E, K, ids + (size_t)t * K, wts + (size_t)t * K);
    if (trace_ids) memcpy(trace_ids, ids, sizeof(int) * (size_t)T * K);
    if (trace_w) memcpy(trace_w, wts, sizeof(float) * (size_t)T * K);

    /* per-expert token lists in token order: counting sort by expert id (stable) */
    for (int i = 0; i < T * K; i++) cnt[ids[i] + 1]++;
    for (int e = 0; e < E; e++) cnt[e + 1] += cnt[e];
    {
        int* fill = (int*)malloc(sizeof(int) * (size_t)E);
        if (!fill) { rc = -2; goto out; }
        memcpy(fill, cnt, sizeof(int) * (size_t)E);
        for (int t = 0; t < T; t++)
            for (int k = 0; k < K; k++) {
                int e = ids[t * K + k], p = fill[e]++;
                lst_tok[p] = t;
                lst_w[p] = wts[t * K + k];
            }
        free(fill);
    }
    for (int e = 0; e < E; e++) {
        const int m = cnt[e + 1] - cnt[e];
        if (!m) continue;
        const int* tk = lst_tok + cnt[e];
        const float* tw = lst_w + cnt[e];
        for (int i = 0; i < m; i++) memcpy(xs + (size_t)i * D, xn + (size_t)tk[i] * D, sizeof(float) * D);
        if ((rc = orc_matmul(gate[e], gt, D, FF, grb, xs, m, D, g, FF))) goto out;
        if ((rc = orc_matmul(up[e], ut, D, FF, urb, xs, m, D, u, FF))) goto out;
        for (int i = 0; i < m * FF; i++) {
            const float gv = g[i];
            g[i] = gv / (1.0f + expf(-gv)) * u[i];
        }
        if ((rc = orc_matmul(down[e], dt, FF, D, drb, g, m, FF, y, D))) goto out;
        for (int i = 0; i < m; i++) {
            float* dst = tmp + (size_t)tk[i] * D;
            const float* src = y + (size_t)i * D;
            for (int d = 0; d < D; d++) dst[d] += tw[i] * src[d];
        }
    }
    for (size_t i = 0; i < (size_t)T * D; i++) x[i] += tmp[i];
out:
    free(rl); free(ids); free(wts); free(cnt); free(lst_tok); free(lst_w);
    free(tmp); free(xs); free(g); free(u); free(y);
    return rc;
}
