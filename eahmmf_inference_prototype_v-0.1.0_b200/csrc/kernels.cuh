// kernels.cuh -- launch-side declarations of the sm_100a kernels (implemented in kernels.cu) and the
// parameter blocks they take. Host code (capi.cu, engine.cu) only sees these.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace eb {

constexpr int MT = 8;               // tokens per pass of the per-row kernel
constexpr int XPASS = 4;            // tokens per pass of the tensor-core GEMV
constexpr int MOE_TMAX = 64;        // tokens per MoE block call (the engine's MAXB, qwen3moe.cpp:39)
constexpr int MU = 2;               // slots per MoE work group (one MMA column set)
constexpr int GW = 8;               // slots per work group of the many-token MoE path (four column sets)
constexpr int ROUTE_NT = 512;       // threads of the routing / prep kernel
constexpr int COMB_NT = 256;        // threads of a combine block
constexpr int MAX_EXPERTS = 512;

// A quantized matrix: rows of row_bytes bytes, ne0 = K elements per row.
struct QMat {
    const uint8_t* w;
    int type;
    int K;
    int rows;
    size_t row_bytes;
};

// Dense GEMV: Y[t*ldy + r] (=|+=) dot(row r, X[t*ldx ..]) for t < m (m <= MT).
struct GemvArgs {
    QMat W;
    const float* X;
    int ldx;
    int m;
    float* Y;
    int ldy;
    int accumulate;
    int generic;  // force the per-element kernel (the reference's EAHMMF_OLD_KERNEL switch)
    int* status;
};

// One work group of the MoE block: up to MU consecutive slots of one expert (written by k_moe_route).
struct __align__(16) GroupRec {
    const uint8_t* w[3];  // the expert's gate, up and down matrices
    int e;                // expert
    int s0;               // first slot
    int mc;               // slots in the group (1..MU)
    int tok[MU];          // token of each slot
    int pad[16 - 6 - 3 - MU];
};
static_assert(sizeof(GroupRec) == 64, "GroupRec is one 64-byte record");

// Routing/permutation workspace of one MoE call (all device pointers, sized for T tokens).
struct RouteWs {
    int* ids;          // [T*K] routed expert ids, rank order (bit-exact with the CPU path)
    float* wts;        // [T*K] renormalised routing weights
    int* offsets;      // [E+1] exclusive prefix of per-expert slot counts
    int* active;       // [E+1] active[0] = number of experts with slots; active[1..] their ids ascending
    int* slot_token;   // [T*K] token of each slot (slots grouped by expert ascending, tokens ascending)
    float* slot_w;     // [T*K] routing weight of each slot
    int* token_slots;  // [T*K] slots of token t, ascending (= expert-ascending)
    int* ngroups;      // [1] number of work groups
    GroupRec* groups;  // [T*K] work groups, expert ascending
};

struct MoeArgs {
    // experts: per-expert component pointers, gate/up [FF x D], down [D x FF]
    const uint8_t* const* gate;  // device arrays of n_expert device pointers
    const uint8_t* const* up;
    const uint8_t* const* down;
    int gate_type, up_type, down_type;
    size_t gate_rb, up_rb, down_rb;
    int n_expert, n_used, D, FF;
    int T;
    const float* xn;      // [T*D] normalised activations (expert input)
    XF xf;                // xn in fragment form (rows = tokens)
    const float* logits;  // [T*E] router logits
    float* x;             // [T*D] residual, += weighted expert outputs
    float* h;             // [T*K*FF] SiLU(gate)*up per slot
    float* y;             // [T*K*D] expert outputs per slot (down projection, before the combine)
    RouteWs rw;
    int* status;
    int gsz;          // slots per work group: MU (small batches, routed in the gate/up kernel) or GW
    int fused_route;  // T <= FUSED_ROUTE_TMAX: k_moe_gateup routes itself (no k_moe_route launch); the
                      // XF of the tokens must already be in xf
    const int* given; // optional [T*K] expert of every (token, k) slot, taken as routed with weight 1
                      // instead of a top-k of the logits (unused then; entries < 0 are absent slots,
                      // K must be 1); needs fused_route = 0
};
constexpr int FUSED_ROUTE_TMAX = 8;

// Dense GEMV on activations already in fragment form: Y[t*ldy + r] (=|+=) row r . x_t, t < m <= XPASS.
struct GemvXArgs {
    QMat W;
    XF xf;
    int m;
    float* Y;
    int ldy;
    int accumulate;
    int* status;
    // Prologue (one token, m == 1): instead of copying the token's XF row from xf, every block forms it in
    // shared memory from a fp32 row: pro = GEMV_PRO_ROW: prow itself; pro = GEMV_PRO_NORM: the RMSNorm
    // (weight pnw, epsilon peps) of the residual row prow plus its pending MoE combine (py, pslots: pK
    // slots of the token in ascending expert order, pw: the slots' weights; py null: none).
    int pro;
    const float* prow;
    const float* py;
    const int* pslots;
    const float* pw;
    int pK;
    const float* pnw;
    float peps;
    // Epilogue (accumulate, m == 1): each output row first takes the token's pending MoE combine, as the
    // norm kernel would have added it: Y = (Y + sum_k w_k ey[slot_k]) + value (ey rows of W.rows floats).
    // pslots / eslots null: slot k is k (the slot map of a single-token MoE call).
    const float* ey;
    const int* eslots;
    const float* ew;
    int eK;
};
constexpr int GEMV_PRO_XF = 0, GEMV_PRO_ROW = 1, GEMV_PRO_NORM = 2;

// Grouped tensor-core path of the MoE block (gemm.cu) for ragged batches.
// Output rows of one grouped tensor-core tile (x 128 slots): a gate/up tile holds 128 FF rows (their gate and
// up rows, 256 accumulator columns), a down tile 256 D rows.
constexpr int GU_TILE_ROWS = 128, DN_TILE_ROWS = 256;

struct GroupedArgs {
    const uint8_t* const* w[3];  // per-expert component pointer tables: gate, up, down
    int type[3];
    size_t rb[3];
    int E, D, FF;
    const int* offsets;     // [E+1] slot offsets per expert
    const int* slot_token;  // [S] token of each slot
    int T;                  // tokens of the call
    const int* tiles_gu;    // [E+1] prefix of gate/up tiles per expert (FF/GU_TILE_ROWS x ceil(m_e/128))
    const int* tiles_dn;    // [E+1] prefix of down tiles per expert (D/DN_TILE_ROWS x ceil(m_e/128))
    __half* wf;             // f16 weights, per expert: gate [FF x D], up [FF x D], down [D x FF]
    size_t w_expert;        // elements per expert (3 FF D)
    size_t w_off[3];        // element offsets of gate, up, down within an expert
    float* rs;              // per expert 2 FF + D row scales (powers of two)
    const float* xn;        // [T x D] expert input rows
    float* h;               // [S x FF] SiLU(g) * u per slot
    __half* bhi;            // activations of the GEMM in progress, f16 of row / bscale, tile-major by
                            //   (expert, 128-slot tile): tiles x 128 x K
    float* bscale;          // [S] per-slot scale of the packed rows
    float* tscale;          // [T] per-token scale of the xn rows
    __half* xh;             // [T x D] f16 of each xn row / tscale (held in the y space, which is dead until
                            //   the down GEMM writes y)
    float* y;               // [S x D] down outputs per slot
    int* status;
};

// A caller's step between the router launch of a MoE pass (the logits of its T tokens complete on the
// stream) and the expert kernels, e.g. to make the routed experts resident first. Nonzero stops the pass.
struct MoeHook {
    int (*fn)(void* ctx, const float* d_logits, int T, int E, cudaStream_t st);
    void* ctx;
};

// The combine inputs of a MoE pass whose combine the caller performs itself.
struct MoeDeferred {
    const int* token_slots = nullptr;  // [T*K] slots of each token, ascending expert order
    const float* slot_w = nullptr;     // routing weight of each slot
    const float* y = nullptr;          // [slots x D] expert outputs
    int K = 0;
};

int sm_count();
bool gemv_mma_ok(const QMat& W);                 // tensor-core path available for this matrix
// bytes of an XF block of `rows` rows: digits (3 bytes per element), per row the per-16 sums and the
// scale (K/16 + 4 floats), per row the group sums (16 + K/8 bytes)
constexpr size_t xf_bytes(int rows, int K) {
    return (size_t)rows * K * 3 + (size_t)rows * (K / 16 + XF_SUM_PAD) * 4 + (size_t)rows * xf_gs_bytes(K) + 256;
}
XF xf_carve(void* base, int rows, int K);        // XF views over such a block
cudaError_t launch_prep_x(const float* X, int ldx, int rows, int K, const XF& out, cudaStream_t st);
cudaError_t launch_gemv_xf(const GemvXArgs& a, cudaStream_t st);
// Dense K-quant GEMM over 1..64 tokens in fragment form (a.m tokens, one launch): the same per-token
// arithmetic and summation order as launch_gemv_xf, the weight tiles read once.
bool gemm_xf_ok(const QMat& W);
cudaError_t launch_gemm_xf(const GemvXArgs& a, cudaStream_t st);
cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t st);  // per-row kernel (any type)
// MoE block (moe.cu): routing + grouping + activation prep, then gate/up, then down, then the combine;
// the last three are launched with programmatic stream serialization.
cudaError_t launch_moe_route(const MoeArgs& a, cudaStream_t st);
cudaError_t launch_moe_gateup(const MoeArgs& a, cudaStream_t st);
// combine = false leaves y, token_slots and slot_w for the caller to combine (engine: fused into the next
// RMSNorm)
cudaError_t launch_moe_down(const MoeArgs& a, cudaStream_t st, bool combine = true);
size_t moe_smem_gateup(int D, size_t rbg, size_t rbu);
// Slots per work group of the chunked (non-fused) MoE path: GW where the wide groups' shared-memory plans
// fit (the Qwen3-30B shapes), MU otherwise (wider layers such as D 4096 / FF 1536).
int moe_chunk_group_size(int D, int FF, size_t rbg, size_t rbu, size_t rbd);
size_t moe_smem_down(int FF, size_t rbd);
cudaError_t launch_grouped_dequant(const GroupedArgs& g, cudaStream_t st);
cudaError_t launch_pack_tokens(const GroupedArgs& g, int slot_tiles, cudaStream_t st);  // xn rows of the slots
cudaError_t launch_pack_slots(const GroupedArgs& g, int slot_tiles, cudaStream_t st);  // the slots' h rows
cudaError_t launch_grouped_gemm(const GroupedArgs& g, int mode, int max_tiles, cudaStream_t st);  // 0 gate/up, 1 down
// routing of a ragged batch of any size (moe.cu): per-token top-k with expert counts (cnt zeroed by the
// caller), then offsets / tile prefixes / active list, then the slot maps
cudaError_t launch_route_big(const MoeArgs& a, int* cnt, int* local, cudaStream_t st);
cudaError_t launch_plan_big(const MoeArgs& a, const int* cnt, int* tiles_gu, int* tiles_dn, cudaStream_t st);
cudaError_t launch_scatter_big(const MoeArgs& a, const int* local, cudaStream_t st);
cudaError_t launch_moe_combine(const MoeArgs& a, cudaStream_t st);
cudaError_t launch_f32_gemv(const float* W, int K, int rows, const float* X, int ldx, int m, float* Y, int ldy,
                            cudaStream_t st);
// the router GEMV plus, in m extra blocks, the m token rows of X in fragment form (xf); with norm_w the
// rows are RMSNorm-ed first (X is then the residual, normalised on the fly)
cudaError_t launch_router_prep(const float* W, int K, int rows, const float* X, int ldx, int m, float* Y, int ldy,
                               const XF& xf, const float* norm_w, float eps, cudaStream_t st);

}  // namespace eb
