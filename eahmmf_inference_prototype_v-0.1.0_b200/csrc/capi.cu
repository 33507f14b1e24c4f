// capi.cu -- the extern "C" entry points declared in include/eahmmf_b200.h (groups 1 and 2).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/eahmmf_b200.h"
#include "common.cuh"
#include "kernels.cuh"

using namespace eb;

namespace {

bool legacy_type(int t) { return t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K; }

// Device scratch of the legacy entry points: grown on demand and kept, like the reference's static
// buffers (expert_cuda.cu:269-301). The entry points are documented single-threaded.
struct Scratch {
    float* p = nullptr;
    size_t cap = 0;
    bool ensure(size_t bytes) {
        if (bytes <= cap) return true;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        if (cudaMalloc(&p, bytes) != cudaSuccess) return false;
        cap = bytes;
        return true;
    }
};
Scratch g_x, g_o1, g_o2, g_xf;
cudaStream_t g_stream = nullptr;

bool legacy_stream() {
    if (g_stream) return true;
    return cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking) == cudaSuccess;
}
bool use_generic() {
    static const bool v = getenv("EAHMMF_OLD_KERNEL") != nullptr;  // the reference's switch (expert_cuda.cu:307)
    return v;
}

bool fragment_path(const QMat& W, const float* dx, int ldx) {
    return !use_generic() && gemv_mma_ok(W) && (reinterpret_cast<uintptr_t>(dx) & 15) == 0 && ldx % 4 == 0;
}
// Workspace of gemv_all: the activations of one pass in fragment form.
constexpr size_t gemv_ws_bytes(int K) { return xf_bytes(XPASS, K); }

// d_out[t*ldo + r] = W x d_x[t*ldx..] for t < nb, MT tokens per pass. The tensor-core path first puts
// the pass's activations in fragment form (ws, gemv_ws_bytes(K) bytes); other types and layouts take
// the per-row kernel.
cudaError_t gemv_all(const QMat& W, const float* dx, int nb, int ldx, float* dout, int ldo, int accumulate,
                     void* ws, cudaStream_t st) {
    const bool frag = ws && fragment_path(W, dx, ldx);
    const int per = frag ? XPASS : MT;
    for (int t0 = 0; t0 < nb; t0 += per) {
        const int m = nb - t0 < per ? nb - t0 : per;
        cudaError_t e;
        if (frag) {
            GemvXArgs a{};
            a.W = W;
            a.xf = xf_carve(ws, XPASS, W.K);
            a.m = m;
            a.Y = dout + (size_t)t0 * ldo;
            a.ldy = ldo;
            a.accumulate = accumulate;
            e = launch_prep_x(dx + (size_t)t0 * ldx, ldx, m, W.K, a.xf, st);
            if (e == cudaSuccess) e = launch_gemv_xf(a, st);
        } else {
            GemvArgs a{};
            a.W = W;
            a.X = dx + (size_t)t0 * ldx;
            a.ldx = ldx;
            a.m = m;
            a.Y = dout + (size_t)t0 * ldo;
            a.ldy = ldo;
            a.accumulate = accumulate;
            e = launch_gemv(a, st);
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

QMat qmat(const uint8_t* w, int type, int ne0, int ne1, size_t rb) { return QMat{w, type, ne0, ne1, rb}; }

bool shape_ok(int type, int ne0, size_t rb) {
    return ne0 > 0 && ne0 % block_elems(type) == 0 && rb == (size_t)(ne0 / block_elems(type)) * block_bytes(type);
}

}  // namespace

// ---------------------------------------------------------------------------------------------------
// 1. reference entry points
// ---------------------------------------------------------------------------------------------------
extern "C" bool eahmmf_cuda_matmul(const uint8_t* device_weights, int type, int ne0, int ne1, size_t row_bytes,
                                   const float* host_x, int nb, int ldx, float* host_out, int ldo) {
    if (!device_weights || !host_x || !host_out || ne0 <= 0 || ne1 <= 0 || nb <= 0 || ldx < ne0 || ldo < ne1 ||
        !legacy_type(type) || !shape_ok(type, ne0, row_bytes))
        return false;
    if (!legacy_stream() || !g_x.ensure((size_t)nb * ne0 * 4) || !g_o1.ensure((size_t)nb * ne1 * 4) ||
        !g_xf.ensure(gemv_ws_bytes(ne0)))
        return false;
    bool ok = cudaMemcpy2DAsync(g_x.p, (size_t)ne0 * 4, host_x, (size_t)ldx * 4, (size_t)ne0 * 4, nb,
                                cudaMemcpyHostToDevice, g_stream) == cudaSuccess;
    if (ok)
        ok = gemv_all(qmat(device_weights, type, ne0, ne1, row_bytes), g_x.p, nb, ne0, g_o1.p, ne1, 0, g_xf.p,
                      g_stream) == cudaSuccess;
    if (ok)
        ok = cudaMemcpy2DAsync(host_out, (size_t)ldo * 4, g_o1.p, (size_t)ne1 * 4, (size_t)ne1 * 4, nb,
                               cudaMemcpyDeviceToHost, g_stream) == cudaSuccess;
    // drain queued work even after an error, before the caller releases the lease or reuses scratch
    if (cudaStreamSynchronize(g_stream) != cudaSuccess) ok = false;
    return ok;
}

extern "C" bool eahmmf_cuda_matmul_pair(const uint8_t* gw, int gt, int gne0, int gne1, size_t grb, const uint8_t* uw,
                                        int ut, int une0, int une1, size_t urb, const float* host_x, int nb, int ldx,
                                        float* host_g, int ldg, float* host_u, int ldu) {
    if (!gw || !uw || !host_x || !host_g || !host_u || !legacy_type(gt) || !legacy_type(ut) || gne0 <= 0 ||
        gne1 <= 0 || une0 != gne0 || une1 != gne1 || nb <= 0 || ldx < gne0 || ldg < gne1 || ldu < une1 ||
        !shape_ok(gt, gne0, grb) || !shape_ok(ut, une0, urb))
        return false;
    if (!legacy_stream() || !g_x.ensure((size_t)nb * gne0 * 4) || !g_o1.ensure((size_t)nb * gne1 * 4) ||
        !g_o2.ensure((size_t)nb * une1 * 4) || !g_xf.ensure(gemv_ws_bytes(gne0)))
        return false;
    bool ok = cudaMemcpy2DAsync(g_x.p, (size_t)gne0 * 4, host_x, (size_t)ldx * 4, (size_t)gne0 * 4, nb,
                                cudaMemcpyHostToDevice, g_stream) == cudaSuccess;
    if (ok)
        ok = gemv_all(qmat(gw, gt, gne0, gne1, grb), g_x.p, nb, gne0, g_o1.p, gne1, 0, g_xf.p, g_stream) == cudaSuccess;
    if (ok)
        ok = gemv_all(qmat(uw, ut, une0, une1, urb), g_x.p, nb, une0, g_o2.p, une1, 0, g_xf.p, g_stream) == cudaSuccess;
    if (ok)
        ok = cudaMemcpy2DAsync(host_g, (size_t)ldg * 4, g_o1.p, (size_t)gne1 * 4, (size_t)gne1 * 4, nb,
                               cudaMemcpyDeviceToHost, g_stream) == cudaSuccess;
    if (ok)
        ok = cudaMemcpy2DAsync(host_u, (size_t)ldu * 4, g_o2.p, (size_t)une1 * 4, (size_t)une1 * 4, nb,
                               cudaMemcpyDeviceToHost, g_stream) == cudaSuccess;
    if (cudaStreamSynchronize(g_stream) != cudaSuccess) ok = false;
    return ok;
}

// ---------------------------------------------------------------------------------------------------
// 2. device-resident MoE block
// ---------------------------------------------------------------------------------------------------
namespace {
constexpr int CHUNK = MOE_TMAX;  // tokens per MoE block pass
size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }
struct WsLayout {
    size_t ids, wts, logits, offsets, active, slot_token, slot_w, token_slots, ngroups, groups, h, xf, y,
        total;
};
WsLayout ws_layout(const EahmmfMoeLayer* L, int T) {
    const int Tc = T < CHUNK ? T : CHUNK;
    const size_t K = (size_t)L->n_used, E = (size_t)L->n_expert, S = (size_t)Tc * K;
    WsLayout w;
    size_t o = 0;
    auto take = [&](size_t& at, size_t bytes) {
        at = o;
        o = a256(o + bytes);
    };
    take(w.ids, (size_t)T * K * 4);  // routing of every token of the call (kept for the engine's trace)
    take(w.wts, (size_t)T * K * 4);
    take(w.logits, L->d_router ? (size_t)Tc * E * 4 : 0);
    take(w.offsets, (E + 1) * 4);
    take(w.active, (E + 1) * 4);
    take(w.slot_token, S * 4);
    take(w.slot_w, S * 4);
    take(w.token_slots, S * 4);
    take(w.ngroups, 4);
    take(w.groups, S * sizeof(GroupRec));
    take(w.h, S * L->FF * 4);
    take(w.xf, xf_bytes(Tc, L->D));
    take(w.y, S * L->D * 4);
    w.total = o;
    return w;
}
// The block runs as grouped tensor-core GEMMs (gemm.cu) from 256 tokens per call when the slots average
// at least 16 per expert: every active expert's weights are dequantized once to f16 and each expert's
// slots are one dense contraction, instead of 64-token passes that each stream the routed experts again.
constexpr int GROUPED_MIN_T = 256;
constexpr int GROUPED_MIN_SLOTS_PER_EXPERT = 16;
struct GroupedLayout {
    size_t ids, wts, logits, offsets, active, ngroups, cnt, local, tiles_gu, tiles_dn, slot_token, slot_w,
        token_slots, wf, rs, bhi, bscale, tscale, h, y, total;
};
GroupedLayout grouped_layout(const EahmmfMoeLayer* L, int T) {
    const size_t K = (size_t)L->n_used, E = (size_t)L->n_expert, S = (size_t)T * K, D = L->D, FF = L->FF;
    GroupedLayout w;
    size_t o = 0;
    auto take = [&](size_t& at, size_t bytes) {
        at = o;
        o = a256(o + bytes);
    };
    take(w.ids, S * 4);  // same head as the 64-token layout: ids, then weights at the next 256 bytes
    take(w.wts, S * 4);
    take(w.logits, L->d_router ? (size_t)T * E * 4 : 0);
    take(w.offsets, (E + 1) * 4);
    take(w.active, (E + 1) * 4);
    take(w.ngroups, 4);
    take(w.cnt, E * 4);
    take(w.local, S * 4);
    take(w.tiles_gu, (E + 1) * 4);
    take(w.tiles_dn, (E + 1) * 4);
    take(w.slot_token, S * 4);
    take(w.slot_w, S * 4);
    take(w.token_slots, S * 4);
    take(w.wf, E * 3 * FF * D * 2);
    take(w.rs, E * (2 * FF + D) * 4);
    const size_t tiles = S / 128 + E + 1;  // bound on sum over experts of ceil(m_e / 128)
    const size_t kmax = D > FF ? D : FF;
    take(w.bhi, tiles * 128 * kmax * 2);
    take(w.bscale, S * 4);
    take(w.tscale, (size_t)T * 4);
    take(w.h, S * FF * 4);
    take(w.y, S * D * 4);
    w.total = o;
    return w;
}
bool grouped_ok(const EahmmfMoeLayer* L, int T) {
    return T >= GROUPED_MIN_T && (long long)T * L->n_used >= (long long)GROUPED_MIN_SLOTS_PER_EXPERT * L->n_expert &&
           L->D % DN_TILE_ROWS == 0 && L->FF % GU_TILE_ROWS == 0;
}

bool layer_ok(const EahmmfMoeLayer* L) {
    return L && L->n_expert > 0 && L->n_expert <= MAX_EXPERTS && L->n_used > 0 && L->n_used <= 32 &&
           L->n_used <= L->n_expert && L->D > 0 && L->D % 256 == 0 && L->FF > 0 && L->FF % 256 == 0 && L->d_gate &&
           L->d_up && L->d_down && is_kquant(L->gate_type) && is_kquant(L->up_type) && is_kquant(L->down_type) &&
           shape_ok(L->gate_type, L->D, L->gate_row_bytes) && shape_ok(L->up_type, L->D, L->up_row_bytes) &&
           shape_ok(L->down_type, L->FF, L->down_row_bytes) &&
           moe_smem_gateup(L->D, L->gate_row_bytes, L->up_row_bytes) <= 227 * 1024 &&
           moe_smem_down(L->FF, L->down_row_bytes) <= 227 * 1024;
}
}  // namespace

// ---- optional per-stage timing of eahmmf_cuda_moe_layer (events on the call's stream) --------------
namespace {
constexpr int PROF_STAGES = 4;  // router GEMV, routing + activation prep, gate/up (+ h prep), down/combine
struct StageTimer {
    bool on = false;
    cudaEvent_t ev[PROF_STAGES + 1] = {};
    double sum[PROF_STAGES] = {};
    int blocks = 0;
    bool ensure() {
        for (auto& e : ev)
            if (!e && cudaEventCreate(&e) != cudaSuccess) return false;
        return true;
    }
    void mark(int i, cudaStream_t st) {
        if (on && i <= PROF_STAGES) cudaEventRecord(ev[i], st);
    }
    // after a block's last mark: wait for it and add its stage durations
    bool collect() {
        if (!on) return true;
        if (cudaEventSynchronize(ev[PROF_STAGES]) != cudaSuccess) return false;
        for (int i = 0; i < PROF_STAGES; i++) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, ev[i], ev[i + 1]) != cudaSuccess) return false;
            sum[i] += ms * 1000.0;
        }
        blocks++;
        return true;
    }
    void reset() {
        for (double& v : sum) v = 0;
        blocks = 0;
    }
} g_prof;
}  // namespace

extern "C" int eahmmf_cuda_moe_profile(int enable) {
    if (enable && !g_prof.ensure()) return ST_CUDA;
    g_prof.on = enable != 0;
    g_prof.reset();
    return ST_OK;
}

extern "C" int eahmmf_cuda_moe_profile_read(float* us, int cap) {
    if (!g_prof.on || !us || cap < PROF_STAGES || g_prof.blocks == 0) return ST_BAD_ARG;
    for (int i = 0; i < PROF_STAGES; i++) us[i] = (float)(g_prof.sum[i] / g_prof.blocks);
    g_prof.reset();
    return ST_OK;
}

extern "C" size_t eahmmf_cuda_moe_workspace_bytes(const EahmmfMoeLayer* L, int T) {
    if (!layer_ok(L) || T < 1) return 0;
    return grouped_ok(L, T) ? grouped_layout(L, T).total : ws_layout(L, T).total;
}

namespace {
// The MoE block for a ragged batch of T >= GROUPED_MIN_T tokens as grouped tensor-core GEMMs.
int moe_grouped(const EahmmfMoeLayer* L, int T, const float* d_xn, const float* d_logits, float* d_x, uint8_t* ws,
                cudaStream_t st, int* d_status, const int* given) {
    const GroupedLayout w = grouped_layout(L, T);
    const int K = L->n_used, E = L->n_expert, S = T * K;
    MoeArgs a{};
    a.gate = L->d_gate;
    a.up = L->d_up;
    a.down = L->d_down;
    a.gate_type = L->gate_type;
    a.up_type = L->up_type;
    a.down_type = L->down_type;
    a.gate_rb = L->gate_row_bytes;
    a.up_rb = L->up_row_bytes;
    a.down_rb = L->down_row_bytes;
    a.n_expert = E;
    a.n_used = K;
    a.D = L->D;
    a.FF = L->FF;
    a.T = T;
    a.xn = d_xn;
    a.x = d_x;
    a.rw.ids = reinterpret_cast<int*>(ws + w.ids);
    a.rw.wts = reinterpret_cast<float*>(ws + w.wts);
    a.rw.offsets = reinterpret_cast<int*>(ws + w.offsets);
    a.rw.active = reinterpret_cast<int*>(ws + w.active);
    a.rw.ngroups = reinterpret_cast<int*>(ws + w.ngroups);
    a.rw.slot_token = reinterpret_cast<int*>(ws + w.slot_token);
    a.rw.slot_w = reinterpret_cast<float*>(ws + w.slot_w);
    a.rw.token_slots = reinterpret_cast<int*>(ws + w.token_slots);
    a.y = reinterpret_cast<float*>(ws + w.y);
    a.status = d_status;
    a.given = given;
    int* cnt = reinterpret_cast<int*>(ws + w.cnt);
    int* local = reinterpret_cast<int*>(ws + w.local);
    int* tiles_gu = reinterpret_cast<int*>(ws + w.tiles_gu);
    int* tiles_dn = reinterpret_cast<int*>(ws + w.tiles_dn);
    GroupedArgs g{};
    g.w[0] = L->d_gate;
    g.w[1] = L->d_up;
    g.w[2] = L->d_down;
    g.type[0] = L->gate_type;
    g.type[1] = L->up_type;
    g.type[2] = L->down_type;
    g.rb[0] = L->gate_row_bytes;
    g.rb[1] = L->up_row_bytes;
    g.rb[2] = L->down_row_bytes;
    g.E = E;
    g.D = L->D;
    g.FF = L->FF;
    g.offsets = a.rw.offsets;
    g.slot_token = a.rw.slot_token;
    g.T = T;
    g.tiles_gu = tiles_gu;
    g.tiles_dn = tiles_dn;
    g.wf = reinterpret_cast<__half*>(ws + w.wf);
    g.w_expert = (size_t)3 * L->FF * L->D;
    g.w_off[0] = 0;
    g.w_off[1] = (size_t)L->FF * L->D;
    g.w_off[2] = (size_t)2 * L->FF * L->D;
    g.rs = reinterpret_cast<float*>(ws + w.rs);
    g.xn = d_xn;
    g.h = reinterpret_cast<float*>(ws + w.h);
    g.bhi = reinterpret_cast<__half*>(ws + w.bhi);
    g.bscale = reinterpret_cast<float*>(ws + w.bscale);
    g.tscale = reinterpret_cast<float*>(ws + w.tscale);
    g.y = a.y;
    g.xh = reinterpret_cast<__half*>(ws + w.y);  // T D f16 <= S D fp32; consumed before y is written
    g.status = d_status;
    g_prof.mark(0, st);
    if (d_logits || given) {
        a.logits = d_logits;
    } else {
        float* lg = reinterpret_cast<float*>(ws + w.logits);
        if (launch_f32_gemv(L->d_router, L->D, E, d_xn, L->D, T, lg, E, st) != cudaSuccess) return ST_CUDA;
        a.logits = lg;
    }
    g_prof.mark(1, st);
    if (cudaMemsetAsync(cnt, 0, (size_t)E * 4, st) != cudaSuccess || launch_route_big(a, cnt, local, st) != cudaSuccess ||
        launch_plan_big(a, cnt, tiles_gu, tiles_dn, st) != cudaSuccess || launch_scatter_big(a, local, st) != cudaSuccess ||
        launch_grouped_dequant(g, st) != cudaSuccess)
        return ST_CUDA;
    const int slot_tiles = (S + 127) / 128 + E;  // bound on sum over experts of ceil(m_e / 128)
    if (launch_pack_tokens(g, slot_tiles, st) != cudaSuccess) return ST_CUDA;
    g_prof.mark(2, st);
    // stage timer: [2] the two GEMMs with the h repack between them, [3] the combine
    if (launch_grouped_gemm(g, 0, (L->FF / GU_TILE_ROWS) * slot_tiles, st) != cudaSuccess ||
        launch_pack_slots(g, slot_tiles, st) != cudaSuccess ||
        launch_grouped_gemm(g, 1, (L->D / DN_TILE_ROWS) * slot_tiles, st) != cudaSuccess)
        return ST_CUDA;
    g_prof.mark(3, st);
    if (launch_moe_combine(a, st) != cudaSuccess) return ST_CUDA;
    g_prof.mark(4, st);
    if (!g_prof.collect()) return ST_CUDA;
    return ST_OK;
}
}  // namespace

namespace {
// The MoE block (eahmmf_cuda_moe_layer) with an optional deferred combine (engine use: when `defer` is
// set and the call runs as one 64-token pass, the combine is not launched and defer receives what it
// needs), or, with `given`, on assigned experts instead of a routing of logits (eahmmf_cuda_moe_experts).
int moe_run(const EahmmfMoeLayer* L, int T, const float* d_xn, const float* d_logits, float* d_x, void* d_workspace,
            size_t workspace_bytes, void* stream, int* d_status, MoeDeferred* defer, const float* norm_w, float eps,
            const int* given, const MoeHook* hook = nullptr) {
    // norm_w: d_xn is the un-normalised residual and the RMSNorm is applied inside the router launch
    // (only for the fused small-batch path: T <= FUSED_ROUTE_TMAX, router matrix present)
    if (norm_w && (T > FUSED_ROUTE_TMAX || d_logits || given || !L || !L->d_router)) return ST_BAD_ARG;
    if (!layer_ok(L)) return (L && !(is_kquant(L->gate_type) && is_kquant(L->up_type) && is_kquant(L->down_type)))
                                  ? ST_BAD_TYPE
                                  : ST_BAD_ARG;
    if (T < 1 || !d_xn || !d_x || !d_workspace || (!d_logits && !given && !L->d_router)) return ST_BAD_ARG;
    if (given && (L->n_used != 1 || defer)) return ST_BAD_ARG;
    if (reinterpret_cast<uintptr_t>(d_xn) & 15 || reinterpret_cast<uintptr_t>(d_x) & 7 ||
        reinterpret_cast<uintptr_t>(d_workspace) & 255)
        return ST_BAD_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(d_workspace);
    // assigned-expert calls (the expert-parallel receiver) pass their whole fixed-capacity buffer, most
    // of it padding rows at larger rank counts: they take the grouped path only at four times the slot
    // density, so that the f16 copy of every local expert is not made for a few real rows
    if (grouped_ok(L, T) &&
        (!given || (long long)T * L->n_used >= 4LL * GROUPED_MIN_SLOTS_PER_EXPERT * L->n_expert)) {
        if (workspace_bytes < grouped_layout(L, T).total) return ST_CAPACITY;
        return moe_grouped(L, T, d_xn, d_logits, d_x, ws, st, d_status, given);
    }
    const WsLayout w = ws_layout(L, T);
    if (workspace_bytes < w.total) return ST_CAPACITY;
    const int K = L->n_used, E = L->n_expert;
    for (int t0 = 0; t0 < T; t0 += CHUNK) {
        const int tc = T - t0 < CHUNK ? T - t0 : CHUNK;
        MoeArgs a{};
        a.gate = L->d_gate;
        a.up = L->d_up;
        a.down = L->d_down;
        a.gate_type = L->gate_type;
        a.up_type = L->up_type;
        a.down_type = L->down_type;
        a.gate_rb = L->gate_row_bytes;
        a.up_rb = L->up_row_bytes;
        a.down_rb = L->down_row_bytes;
        a.n_expert = E;
        a.n_used = K;
        a.D = L->D;
        a.FF = L->FF;
        a.T = tc;
        a.xn = d_xn + (size_t)t0 * L->D;
        a.x = d_x + (size_t)t0 * L->D;
        a.h = reinterpret_cast<float*>(ws + w.h);
        a.rw.ids = reinterpret_cast<int*>(ws + w.ids) + (size_t)t0 * K;
        a.rw.wts = reinterpret_cast<float*>(ws + w.wts) + (size_t)t0 * K;
        a.rw.offsets = reinterpret_cast<int*>(ws + w.offsets);
        a.rw.active = reinterpret_cast<int*>(ws + w.active);
        a.rw.slot_token = reinterpret_cast<int*>(ws + w.slot_token);
        a.rw.slot_w = reinterpret_cast<float*>(ws + w.slot_w);
        a.rw.token_slots = reinterpret_cast<int*>(ws + w.token_slots);
        a.rw.ngroups = reinterpret_cast<int*>(ws + w.ngroups);
        a.rw.groups = reinterpret_cast<GroupRec*>(ws + w.groups);
        a.xf = xf_carve(ws + w.xf, tc, L->D);
        a.y = reinterpret_cast<float*>(ws + w.y);
        a.status = d_status;
        // up to FUSED_ROUTE_TMAX tokens: the XF prep rides on the router launch (or a prep launch) and the
        // gate/up kernel routes by itself; larger blocks go through k_moe_route
        a.fused_route = tc <= FUSED_ROUTE_TMAX && !given ? 1 : 0;
        // larger chunks: up to GW of an expert's slots per weight pass, where those kernels' plans fit
        a.gsz = a.fused_route ? MU
                              : moe_chunk_group_size(L->D, L->FF, L->gate_row_bytes, L->up_row_bytes, L->down_row_bytes);
        a.given = given ? given + (size_t)t0 * K : nullptr;
        g_prof.mark(0, st);
        if (given) {
            a.logits = nullptr;  // k_moe_route takes the assigned experts and preps the tokens' XF
        } else if (d_logits) {
            a.logits = d_logits + (size_t)t0 * E;
            if (a.fused_route && launch_prep_x(a.xn, L->D, tc, L->D, a.xf, st) != cudaSuccess) return ST_CUDA;
        } else {
            float* lg = reinterpret_cast<float*>(ws + w.logits);
            const cudaError_t e = a.fused_route
                                      ? launch_router_prep(L->d_router, L->D, E, a.xn, L->D, tc, lg, E, a.xf, norm_w, eps, st)
                                      : launch_f32_gemv(L->d_router, L->D, E, a.xn, L->D, tc, lg, E, st);
            if (e != cudaSuccess) return ST_CUDA;
            a.logits = lg;
        }
        if (hook && hook->fn) {
            const int rc = hook->fn(hook->ctx, a.logits, tc, E, st);
            if (rc != ST_OK) return rc;
        }
        g_prof.mark(1, st);
        if (!a.fused_route && launch_moe_route(a, st) != cudaSuccess) return ST_CUDA;
        g_prof.mark(2, st);
        if (launch_moe_gateup(a, st) != cudaSuccess) return ST_CUDA;
        g_prof.mark(3, st);
        const bool deferred = defer && T <= CHUNK;
        if (launch_moe_down(a, st, !deferred) != cudaSuccess) return ST_CUDA;
        if (deferred) {
            defer->token_slots = a.rw.token_slots;
            defer->slot_w = a.rw.slot_w;
            defer->y = a.y;
            defer->K = K;
        }
        g_prof.mark(4, st);
        if (!g_prof.collect()) return ST_CUDA;
    }
    return ST_OK;
}
}  // namespace

namespace eb {
int moe_layer_run(const EahmmfMoeLayer* L, int T, const float* d_xn, const float* d_logits, float* d_x,
                  void* d_workspace, size_t workspace_bytes, void* stream, int* d_status, MoeDeferred* defer,
                  const float* norm_w, float eps, const MoeHook* hook = nullptr) {
    return moe_run(L, T, d_xn, d_logits, d_x, d_workspace, workspace_bytes, stream, d_status, defer, norm_w, eps,
                   nullptr, hook);
}
}  // namespace eb

namespace {
// The layer as the assigned-expert entry sees it: one expert per row, no router.
EahmmfMoeLayer experts_view(const EahmmfMoeLayer* L) {
    EahmmfMoeLayer v = *L;
    v.n_used = 1;
    v.d_router = nullptr;
    return v;
}
}  // namespace

extern "C" size_t eahmmf_cuda_moe_experts_workspace_bytes(const EahmmfMoeLayer* L, int R) {
    if (!L) return 0;
    const EahmmfMoeLayer v = experts_view(L);
    return eahmmf_cuda_moe_workspace_bytes(&v, R);
}

extern "C" int eahmmf_cuda_moe_experts(const EahmmfMoeLayer* L, int R, const float* d_rows, const int* d_eid,
                                       float* d_y, void* d_workspace, size_t workspace_bytes, void* stream,
                                       int* d_status) {
    if (!L || !d_eid) return ST_BAD_ARG;
    const EahmmfMoeLayer v = experts_view(L);
    return moe_run(&v, R, d_rows, nullptr, d_y, d_workspace, workspace_bytes, stream, d_status, nullptr, nullptr, 0.f,
                   d_eid);
}

extern "C" int eahmmf_cuda_moe_layer(const EahmmfMoeLayer* L, int T, const float* d_xn, const float* d_logits,
                                     float* d_x, void* d_workspace, size_t workspace_bytes, void* stream,
                                     int* d_status) {
    return moe_layer_run(L, T, d_xn, d_logits, d_x, d_workspace, workspace_bytes, stream, d_status, nullptr, nullptr,
                         0.f);
}

extern "C" int eahmmf_cuda_route_topk(const float* d_logits, int T, int E, int K, int* d_ids, float* d_w, void* stream,
                                      int* d_status) {
    if (!d_logits || !d_ids || !d_w || T < 1 || E < 1 || E > MAX_EXPERTS || K < 1 || K > 32 || K > E) return ST_BAD_ARG;
    MoeArgs a{};
    a.logits = d_logits;
    a.T = T;
    a.n_expert = E;
    a.n_used = K;
    a.rw.ids = d_ids;
    a.rw.wts = d_w;
    a.status = d_status;
    return launch_route_big(a, nullptr, nullptr, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? ST_OK
                                                                                                      : ST_CUDA;
}

extern "C" int eahmmf_cuda_moe_combine(int T, int K, int D, const int* d_token_slots, const float* d_slot_w,
                                       const float* d_y, float* d_x, void* stream) {
    if (T < 1 || K < 1 || K > 32 || D < 2 || D % 2 || !d_token_slots || !d_slot_w || !d_y || !d_x) return ST_BAD_ARG;
    if ((reinterpret_cast<uintptr_t>(d_y) | reinterpret_cast<uintptr_t>(d_x)) & 7) return ST_BAD_ARG;
    MoeArgs a{};
    a.T = T;
    a.n_used = K;
    a.D = D;
    a.rw.token_slots = const_cast<int*>(d_token_slots);
    a.rw.slot_w = const_cast<float*>(d_slot_w);
    a.y = const_cast<float*>(d_y);
    a.x = d_x;
    return launch_moe_combine(a, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? ST_OK : ST_CUDA;
}

extern "C" size_t eahmmf_cuda_gemv_workspace_bytes(int ne0) { return ne0 > 0 ? gemv_ws_bytes(ne0) : 0; }

extern "C" int eahmmf_cuda_gemv(const uint8_t* d_w, int type, int ne0, int ne1, size_t row_bytes, const float* d_x,
                                int nb, int ldx, float* d_out, int ldo, int accumulate, void* d_workspace,
                                size_t workspace_bytes, void* stream) {
    if (!type_supported(type)) return ST_BAD_TYPE;
    if (!d_w || !d_x || !d_out || ne1 <= 0 || nb <= 0 || ldx < ne0 || ldo < ne1 || !shape_ok(type, ne0, row_bytes))
        return ST_BAD_ARG;
    if (d_workspace && workspace_bytes < gemv_ws_bytes(ne0)) return ST_CAPACITY;
    return gemv_all(qmat(d_w, type, ne0, ne1, row_bytes), d_x, nb, ldx, d_out, ldo, accumulate, d_workspace,
                    reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
               ? ST_OK
               : ST_CUDA;
}

// ---- eahmmf_cuda_gemv_static: the same GEMV with its workspace in a fixed device array -------------
// For callers that may not allocate device memory on this path. The fragment-form activations of one
// pass live in a file-scope __device__ array sized for ne0 <= EAHMMF_GEMV_STATIC_MAX_NE0; larger
// rows are refused with EAHMMF_ST_CAPACITY. Every byte a pass reads is written by that pass's prep
// kernel first, so the array needs no clearing. One array per device: calls that overlap on one
// device (several streams or threads) race on it.
namespace {
constexpr size_t STATIC_WS_BYTES = 224 * 1024;
static_assert(EAHMMF_GEMV_STATIC_MAX_NE0 % 256 == 0, "row length must be whole super-blocks");
__device__ __align__(256) uint8_t g_static_ws[STATIC_WS_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_static_mu;
void* g_static_ptr[MAX_DEVICES] = {};

// Address of this device's copy of g_static_ws, looked up once per device with that device current.
void* static_ws(int* err) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) {
        *err = ST_CUDA;
        return nullptr;
    }
    std::lock_guard<std::mutex> g(g_static_mu);
    if (!g_static_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_ws) != cudaSuccess || !p) {
            *err = ST_CUDA;
            return nullptr;
        }
        g_static_ptr[dev] = p;
    }
    return g_static_ptr[dev];
}
}  // namespace

extern "C" int eahmmf_cuda_gemv_static(const uint8_t* d_w, int type, int ne0, int ne1, size_t row_bytes,
                                       const float* d_x, int nb, int ldx, float* d_out, int ldo, int accumulate,
                                       void* stream) {
    static_assert(gemv_ws_bytes(EAHMMF_GEMV_STATIC_MAX_NE0) <= STATIC_WS_BYTES, "static workspace too small");
    if (!type_supported(type)) return ST_BAD_TYPE;
    if (!d_w || !d_x || !d_out || ne1 <= 0 || nb <= 0 || ldx < ne0 || ldo < ne1 || !shape_ok(type, ne0, row_bytes))
        return ST_BAD_ARG;
    if (ne0 > EAHMMF_GEMV_STATIC_MAX_NE0 || gemv_ws_bytes(ne0) > STATIC_WS_BYTES) return ST_CAPACITY;
    int err = ST_OK;
    void* ws = static_ws(&err);
    if (!ws) return err;
    return gemv_all(qmat(d_w, type, ne0, ne1, row_bytes), d_x, nb, ldx, d_out, ldo, accumulate, ws,
                    reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
               ? ST_OK
               : ST_CUDA;
}

extern "C" const char* eahmmf_b200_version(void) { return "eahmmf-b200 0.1.0 (sm_100a)"; }
extern "C" int eahmmf_b200_sm_count(void) { return sm_count(); }
