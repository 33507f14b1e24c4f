// oracle/ref_harness.cpp -- TEST INFRASTRUCTURE ONLY (parity checker and CPU baseline).
//
// Compiles the reference engine unmodified, from the file where it lies in the reference tree
// (qwen3moe.cpp + eahmmf.h; the include path is set by oracle/Makefile), the same way the reference's
// own suite does (tests/test_eahmmf.cpp:5-6: QWEN3MOE_NO_MAIN + #include "qwen3moe.cpp"), and exposes
// a small C ABI over it for ctypes. Only tests/, __graft_entry__.smoke() and bench.py's reference arm
// load the library built from this file; the product never links it.
//
// What is exposed:
//   eref_matmul        -> reference matmul()                              qwen3moe.cpp:397-419
//   eref_moe_layer     -> the MoE block of Engine::forward, restated around the reference matmul/expf
//                         and std::partial_sort exactly as written there   qwen3moe.cpp:1007-1069
//   eref_engine_*      -> Engine::load / forward / eval + routing trace   qwen3moe.cpp:859-1084
#define QWEN3MOE_NO_MAIN
#include "qwen3moe.cpp"

#include <memory>

namespace {

WeightView make_view(const uint8_t* w, int type, int64_t ne0, int64_t ne1, size_t row_bytes) {
    WeightView v;
    v.data = w;
    v.type = (uint32_t)type;
    v.ne0 = ne0;
    v.ne1 = ne1;
    v.row_bytes = row_bytes;
    v.bytes = row_bytes * (size_t)ne1;
    return v;
}

bool type_ok(int type) { return type >= 0 && type < 40 && g_types[type].dq != nullptr; }

// matmul() keeps a per-row accumulator of MAXB tokens (qwen3moe.cpp:409); longer inputs go in chunks,
// which does not change any per-token result (each token's accumulator is independent).
void matmul_chunked(const WeightView& W, const float* x, int nb, int ldx, float* out, int ldo) {
    for (int t0 = 0; t0 < nb; t0 += MAXB) {
        int n = std::min(MAXB, nb - t0);
        matmul(W, x + (size_t)t0 * ldx, n, ldx, out + (size_t)t0 * ldo, ldo);
    }
}

// One MoE block over nb <= MAXB tokens: qwen3moe.cpp:1008-1069 with the expert tensors passed in
// as per-expert component pointers instead of ExpertStore leases.
void moe_block(int nb, int D, int FF, int E, int K, const float* xn, const float* logits_in,
               const WeightView& router, const uint8_t* const* gate, const uint8_t* const* up,
               const uint8_t* const* down, int gt, int ut, int dt, size_t grb, size_t urb, size_t drb,
               float* x, int* trace_ids, float* trace_w) {
    std::vector<float> rl((size_t)nb * E), tmp((size_t)nb * D), xs((size_t)nb * D), gbuf((size_t)nb * FF),
        ubuf((size_t)nb * FF), ybuf((size_t)nb * D);
    if (logits_in) memcpy(rl.data(), logits_in, sizeof(float) * nb * E);
    else matmul(router, xn, nb, D, rl.data(), E);  // :1008
    std::vector<std::vector<std::pair<int, float>>> by_exp(E);
    std::vector<int> idx(E);
    for (int t = 0; t < nb; t++) {  // :1011-1023
        float* r = &rl[(size_t)t * E];
        float mx = *std::max_element(r, r + E), sum = 0;
        for (int e = 0; e < E; e++) { r[e] = expf(r[e] - mx); sum += r[e]; }
        std::iota(idx.begin(), idx.end(), 0);
        std::partial_sort(idx.begin(), idx.begin() + K, idx.end(),
                          [&](int a, int b) { return r[a] > r[b] || (r[a] == r[b] && a < b); });
        float tot = 0;
        for (int i = 0; i < K; i++) tot += r[idx[i]];
        for (int i = 0; i < K; i++) {
            by_exp[idx[i]].push_back({t, r[idx[i]] / tot});
            if (trace_ids) trace_ids[(size_t)t * K + i] = idx[i];
            if (trace_w) trace_w[(size_t)t * K + i] = r[idx[i]] / tot;
        }
    }
    memset(tmp.data(), 0, sizeof(float) * nb * D);  // :1024
    for (int e = 0; e < E; e++) {                    // :1025 expert-ascending
        auto& lst = by_exp[e];
        if (lst.empty()) continue;
        int m = (int)lst.size();
        for (int i = 0; i < m; i++) memcpy(&xs[(size_t)i * D], &xn[(size_t)lst[i].first * D], D * sizeof(float));
        WeightView g = make_view(gate[e], gt, D, FF, grb), u = make_view(up[e], ut, D, FF, urb),
                   dn = make_view(down[e], dt, FF, D, drb);
        matmul(g, xs.data(), m, D, gbuf.data(), FF);  // :1053-1054
        matmul(u, xs.data(), m, D, ubuf.data(), FF);
        for (int i = 0; i < m * FF; i++) {  // :1056-1059
            float gv = gbuf[i];
            gbuf[i] = gv / (1.0f + expf(-gv)) * ubuf[i];
        }
        matmul(dn, gbuf.data(), m, FF, ybuf.data(), D);  // :1060
        for (int i = 0; i < m; i++) {                      // :1062-1067
            float w = lst[i].second;
            float* dst = &tmp[(size_t)lst[i].first * D];
            const float* src = &ybuf[(size_t)i * D];
            for (int d = 0; d < D; d++) dst[d] += w * src[d];
        }
    }
    for (int i = 0; i < nb * D; i++) x[i] += tmp[i];  // :1069
}

}  // namespace

extern "C" {

// Initialise the dequant tables (init_types, qwen3moe.cpp:204-218) once; set the OpenMP thread count
// when n_threads > 0. Returns the thread count in use.
int eref_init(int n_threads) {
    static bool done = false;
    if (!done) {
        init_types();
        done = true;
    }
    if (n_threads > 0) omp_set_num_threads(n_threads);
    return omp_get_max_threads();
}

// out[t*ldo + r] = dot(row r, x[t*ldx ..]); any nb (chunked by MAXB). 0 on success.
int eref_matmul(const uint8_t* w, int type, int64_t ne0, int64_t ne1, size_t row_bytes, const float* x, int nb,
                int ldx, float* out, int ldo) {
    if (!w || !x || !out || nb < 1 || !type_ok(type) || ne0 % g_types[type].blck) return -1;
    matmul_chunked(make_view(w, type, ne0, ne1, row_bytes), x, nb, ldx, out, ldo);
    return 0;
}

// Whole MoE layer for T tokens, evaluated in MAXB-token blocks as Engine::eval would feed forward().
// xn: T*D normalised activations; logits: T*E router logits or NULL (then router_w, F32 [E*D], is used);
// x: T*D residual, updated in place; trace_ids/trace_w: T*K (optional).
int eref_moe_layer(int T, int D, int FF, int E, int K, const float* xn, const float* logits, const float* router_w,
                   const uint8_t* const* gate, const uint8_t* const* up, const uint8_t* const* down, int gt, int ut,
                   int dt, size_t grb, size_t urb, size_t drb, float* x, int* trace_ids, float* trace_w) {
    if (T < 1 || K < 1 || K > E || !xn || !x || !gate || !up || !down) return -1;
    if (!logits && !router_w) return -1;
    if (!type_ok(gt) || !type_ok(ut) || !type_ok(dt)) return -2;
    WeightView router = make_view((const uint8_t*)router_w, 0, D, E, (size_t)D * 4);
    for (int t0 = 0; t0 < T; t0 += MAXB) {
        int nb = std::min(MAXB, T - t0);
        moe_block(nb, D, FF, E, K, xn + (size_t)t0 * D, logits ? logits + (size_t)t0 * E : nullptr, router, gate,
                  up, down, gt, ut, dt, grb, urb, drb, x + (size_t)t0 * D,
                  trace_ids ? trace_ids + (size_t)t0 * K : nullptr, trace_w ? trace_w + (size_t)t0 * K : nullptr);
    }
    return 0;
}

// ---- whole engine -------------------------------------------------------------------------------
void* eref_engine_load(const char* path, int n_ctx) {
    eref_init(0);
    Engine* e = new Engine();
    e->load(path, n_ctx, false);  // dies (exit 1) on a malformed file, as the reference does
    return e;
}
void eref_engine_free(void* h) { delete (Engine*)h; }

// dims[0..10] = n_layer, D, n_head, n_kv, hd, n_expert, n_used, FF, n_vocab, n_ctx, tok_embd rows
int eref_engine_dims(void* h, int* dims) {
    Engine* e = (Engine*)h;
    int v[11] = {e->n_layer, e->D,  e->n_head,  e->n_kv,  e->hd, e->n_expert,
                 e->n_used,  e->FF, e->n_vocab, e->n_ctx, (int)e->tok_embd->ne[1]};
    memcpy(dims, v, sizeof v);
    return 0;
}

// Engine::eval (qwen3moe.cpp:1078-1084). logits (n_vocab) of the last token, or NULL.
int eref_engine_eval(void* h, const int* toks, int n, int p0, int n_batch, float* logits) {
    Engine* e = (Engine*)h;
    if (n < 1 || n_batch < 1 || n_batch > MAXB || p0 + n > e->n_ctx) return -1;
    std::vector<int> t(toks, toks + n);
    e->eval(t, p0, n_batch, logits);
    return 0;
}

void eref_engine_trace(void* h, int enable) {
    Engine* e = (Engine*)h;
    e->trace_routing = enable != 0;
    e->trace_ids.clear();
    e->trace_w.clear();
}
// Copies up to cap routing-trace entries (layer-major within each forward call); returns the count.
int eref_engine_trace_get(void* h, int* ids, float* w, int cap) {
    Engine* e = (Engine*)h;
    int n = (int)std::min<size_t>((size_t)cap, e->trace_ids.size());
    if (ids) memcpy(ids, e->trace_ids.data(), sizeof(int) * n);
    if (w) memcpy(w, e->trace_w.data(), sizeof(float) * n);
    return (int)e->trace_ids.size();
}

// Greedy generation with --temp 0 --repeat-penalty 1.0 semantics: prompt through eval(), then one
// token per forward(); argmax is std::max_element's first maximum (qwen3moe.cpp:1103).
// first_logits (n_vocab, optional) receives the logits after the prompt.
int eref_engine_greedy(void* h, const int* prompt, int n_prompt, int n_gen, int n_batch, int* out, float* first_logits) {
    Engine* e = (Engine*)h;
    if (n_prompt < 1 || n_prompt + n_gen > e->n_ctx || n_batch < 1 || n_batch > MAXB) return -1;
    std::vector<float> lg(e->n_vocab);
    std::vector<int> t(prompt, prompt + n_prompt);
    e->eval(t, 0, n_batch, lg.data());
    if (first_logits) memcpy(first_logits, lg.data(), sizeof(float) * e->n_vocab);
    int pos = n_prompt;
    for (int i = 0; i < n_gen; i++) {
        int tok = (int)(std::max_element(lg.begin(), lg.end()) - lg.begin());
        out[i] = tok;
        if (i + 1 < n_gen) e->forward(&tok, 1, pos++, lg.data());
    }
    return 0;
}

}  // extern "C"

// ---- the reference sampler (qwen3moe.cpp:1090-1130) ------------------------------------------------
namespace {
Sampler make_sampler(float temp, float top_p, float min_p, float rep, int top_k, int rep_n, uint64_t seed) {
    Sampler sp;
    sp.temp = temp;
    sp.top_p = top_p;
    sp.min_p = min_p;
    sp.rep = rep;
    sp.top_k = top_k;
    sp.rep_n = rep_n;
    sp.rng.seed(seed);  // as main() seeds it (qwen3moe.cpp:1231)
    return sp;
}
}  // namespace

extern "C" {
// Sampler::sample on one row of n logits (modified in place by the repetition penalty, as there), with
// the window hist[0 .. n_hist) and a fresh stream seeded with `seed`; returns the token.
int eref_sample(float* lg, int n, const int* hist, int n_hist, float temp, float top_p, float min_p, float rep,
                int top_k, int rep_n, uint64_t seed) {
    Sampler sp = make_sampler(temp, top_p, min_p, rep, top_k, rep_n, seed);
    std::vector<int> h(hist, hist + n_hist);
    return sp.sample(lg, n, h);
}

// The residency layer's checksum (eahmmf.h:64-76) of a host buffer.
uint64_t eref_hash64(const uint8_t* p, size_t n) { return eahmmf::hash64(p, n); }

// n draws of std::uniform_real_distribution<float>(0, 1) from std::mt19937_64 seeded with `seed`.
void eref_uniform(uint64_t seed, int n, float* out) {
    std::mt19937_64 g;
    g.seed(seed);
    for (int i = 0; i < n; i++) out[i] = std::uniform_real_distribution<float>(0.f, 1.f)(g);
}

// The generate loop (qwen3moe.cpp:1294-1310) without the tokenizer: the prompt through eval, then per
// step Sampler::sample over the logits with the generated tokens as history, and that token through a
// one-token eval; n_gen tokens out. The sampler's stream is seeded with `seed`.
int eref_engine_generate(void* h, const int* prompt, int n_prompt, int n_gen, int n_batch, float temp, float top_p,
                         float min_p, float rep, int top_k, int rep_n, uint64_t seed, int* out) {
    Engine* e = (Engine*)h;
    if (n_prompt < 1 || n_prompt + n_gen > e->n_ctx || n_batch < 1 || n_batch > MAXB) return -1;
    Sampler sp = make_sampler(temp, top_p, min_p, rep, top_k, rep_n, seed);
    std::vector<float> lg(e->n_vocab);
    std::vector<int> pending(prompt, prompt + n_prompt), hist;
    int n_past = 0;
    for (int step = 0; step < n_gen; step++) {
        e->eval(pending, n_past, n_batch, lg.data());
        n_past += (int)pending.size();
        const int tok = sp.sample(lg.data(), e->n_vocab, hist);
        hist.push_back(tok);
        out[step] = tok;
        pending = {tok};
    }
    return 0;
}
}  // extern "C"
