/* eahmmf_b200.h -- C ABI of the B200 (sm_100a) expert hot path, libeahmmf_b200.so.
 *
 * Four groups of entry points:
 *
 *  1. The reference's own CUDA entry points, same names, signatures and conventions, so the unmodified
 *     engine (qwen3moe.cpp built with -DEAHMMF_CUDA -DEAHMMF_CUDA_COMPUTE) links against this library
 *     instead of expert_cuda.o. Weights are device pointers (WeightView.dev), activations and outputs
 *     are HOST pointers, the result is ready on return, `false` means bad arguments, an unsupported
 *     type or a CUDA error (the caller then falls back to its CPU kernel). Single-threaded caller.
 *
 *  2. Device-resident entry points for the whole MoE block: routing, grouping, gate/up/SiLU and
 *     down/combine run on the GPU with no host round trip. They never allocate: the caller passes a
 *     workspace of eahmmf_cuda_moe_workspace_bytes(). Return 0 on success or EAHMMF_ST_* bits.
 *
 *  3. The device backend used by eahmmf::B200Device (include/eahmmf_b200_device.hpp): allocation,
 *     pinned-staged asynchronous copies on a side stream, free-memory queries.
 *
 *  4. A device-resident engine: a whole qwen3moe GGUF model in HBM, forward / eval / greedy decode
 *     with the MoE block of group 2 and the attention path on the GPU.
 *
 * ggml type ids accepted: 0 F32, 1 F16, 8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K (the expert kernels take the
 * K-quants 12/13/14). Weight buffers must stay readable up to the next 16-byte boundary after their last
 * row (bulk copies are 16-byte granular); every ExpertStore footprint and cudaMalloc block is.
 */
#ifndef EAHMMF_B200_H
#define EAHMMF_B200_H
#include <stddef.h>
#include <stdint.h>
#ifndef __cplusplus
#include <stdbool.h>
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status bits (device status word and return values of group 2/3). */
#define EAHMMF_ST_OK 0
#define EAHMMF_ST_BAD_ARG 1
#define EAHMMF_ST_BAD_TYPE 2
#define EAHMMF_ST_CUDA 4
#define EAHMMF_ST_WAIT_TIMEOUT 8
#define EAHMMF_ST_BAD_INDEX 16
#define EAHMMF_ST_CAPACITY 32

/* ---- 1. reference entry points --------------------------------------------------------------- */

/* out[t*ldo + r] = dot(dequant(row r of device_weights), host_x[t*ldx ..]) for r < ne1, t < nb.
 * Replaces eahmmf_cuda_matmul, expert_cuda.cu:251-261 (declared by the engine at qwen3moe.cpp:422,
 * called from gpu_matmul, qwen3moe.cpp:471-474, and matmul_shadow, qwen3moe.cpp:444). Gaps between
 * rows of host_out (ldo > ne1) are left untouched. */
bool eahmmf_cuda_matmul(const uint8_t* device_weights, int type, int ne0, int ne1, size_t row_bytes,
                        const float* host_x, int nb, int ldx, float* host_out, int ldo);

/* Gate and up projections of the same activations: one host->device copy, one synchronisation.
 * Replaces eahmmf_cuda_matmul_pair, expert_cuda.cu:344-348 (called from gpu_matmul_pair,
 * qwen3moe.cpp:476-491, in the MoE block at qwen3moe.cpp:1037). */
bool eahmmf_cuda_matmul_pair(const uint8_t* gw, int gt, int gne0, int gne1, size_t grb, const uint8_t* uw, int ut,
                             int une0, int une1, size_t urb, const float* host_x, int nb, int ldx, float* host_g,
                             int ldg, float* host_u, int ldu);

/* ---- 2. device-resident MoE block ------------------------------------------------------------- */

/* One MoE layer's experts: per-expert component pointers, as ExpertStore leases expose them
 * (WeightView.dev of ExpertViews.gate/up/down, eahmmf.h:54-62, :737-742). gate/up are [FF rows x D],
 * down is [D rows x FF]. */
typedef struct EahmmfMoeLayer {
    int n_expert; /* experts in the layer (<= 512) */
    int n_used;   /* experts per token, k (<= 32) */
    int D;        /* hidden size (multiple of 256) */
    int FF;       /* expert intermediate size (multiple of 256) */
    int gate_type, up_type, down_type; /* 12 Q4_K, 13 Q5_K or 14 Q6_K */
    size_t gate_row_bytes, up_row_bytes, down_row_bytes;
    const uint8_t* const* d_gate; /* device array of n_expert device pointers */
    const uint8_t* const* d_up;
    const uint8_t* const* d_down;
    const float* d_router; /* F32 [n_expert x D] router matrix; NULL when logits are passed in */
} EahmmfMoeLayer;

/* Bytes of workspace eahmmf_cuda_moe_layer needs for T tokens (S = T x n_used slots). The workspace
 * starts with the routing result of the last call: int32 ids[S], then float weights[S] (rank order).
 * Below 256 tokens (or below 16 slots per expert on average) the call runs in passes of at most 64
 * tokens: about 8 S + min(T, 64) x n_used x (FF + D) x 4 bytes (6.3 MB at the Qwen3-30B-A3B shape).
 * From 256 tokens with >= 16 slots per expert it takes the grouped tensor-core path, whose workspace
 * holds an f16 copy of every expert of the layer, n_expert x 3 x FF x D x 2 bytes (1.21 GB at the
 * 30B shape, 4.83 GB at the 235B-A22B shape), plus S x (FF + D + 7) x 4 bytes of per-slot rows and
 * indices and (S / 128 + n_expert + 1) x 128 x max(D, FF) x 2 bytes of packed activations (3.27 GB in
 * all for 16,193 tokens at the 30B shape). */
size_t eahmmf_cuda_moe_workspace_bytes(const EahmmfMoeLayer* L, int T);

/* The MoE block of Engine::forward (qwen3moe.cpp:1008-1069) for T tokens, on `stream` (cudaStream_t,
 * NULL = default stream), asynchronous:
 *   logits = d_logits ? d_logits : d_xn x router^T;  softmax numerators exp(l - max);  top-k with the
 *   reference's comparator;  weights renormalised over the k;  per active expert (ascending id) the
 *   gate/up projections, SiLU(g)*u, the down projection, and the weighted sum added to d_x.
 * d_xn: [T x D] expert input (post-norm, 16-byte aligned); d_x: [T x D] residual (8-byte aligned),
 * updated in place. Tokens are taken in blocks of 64, as the engine's forward() is fed at most
 * MAXB = 64 tokens (qwen3moe.cpp:39, :933); per-token results do not depend on the blocking.
 * d_status (optional) receives EAHMMF_ST_* bits raised inside kernels. */
int eahmmf_cuda_moe_layer(const EahmmfMoeLayer* L, int T, const float* d_xn, const float* d_logits, float* d_x,
                          void* d_workspace, size_t workspace_bytes, void* stream, int* d_status);

/* The routing step alone (qwen3moe.cpp:1011-1023): per token, softmax numerators, top-k by
 * (r desc, index asc), weights renormalised over the k, ids bit-exact with the CPU path. d_logits
 * [T x E], d_ids / d_w [T x K] in rank order. Used by the expert-parallel layer to dispatch tokens. */
int eahmmf_cuda_route_topk(const float* d_logits, int T, int E, int K, int* d_ids, float* d_w, void* stream,
                           int* d_status);

/* The weighted combine alone (qwen3moe.cpp:1024, :1062-1069): d_x[t] += sum over k of
 * d_slot_w[s] * d_y[s] for the K slots s = d_token_slots[t*K + k], which must be listed in ascending
 * expert order (the reference's summation order). d_y [slots x D]; d_x [T x D]; D even, 8-byte aligned. */
int eahmmf_cuda_moe_combine(int T, int K, int D, const int* d_token_slots, const float* d_slot_w, const float* d_y,
                            float* d_x, void* stream);

/* The expert application alone, on assigned experts (the expert-parallel receiver; no counterpart in the
 * reference, whose MoE block routes and applies in one process, qwen3moe.cpp:1025-1067): for every row r
 * with d_eid[r] >= 0, d_y[r] += down(SiLU(gate x) * (up x)) of expert d_eid[r] over x = d_rows[r], the
 * same per-row arithmetic as eahmmf_cuda_moe_layer's (no routing, weight 1; zero d_y first to get the
 * expert output itself). Rows with d_eid[r] < 0 are absent: in no product, d_y[r] untouched.
 * The router matrix and n_used of L are ignored. Workspace: eahmmf_cuda_moe_experts_workspace_bytes(L, R). */
size_t eahmmf_cuda_moe_experts_workspace_bytes(const EahmmfMoeLayer* L, int R);
int eahmmf_cuda_moe_experts(const EahmmfMoeLayer* L, int R, const float* d_rows, const int* d_eid, float* d_y,
                            void* d_workspace, size_t workspace_bytes, void* stream, int* d_status);

/* Expert-parallel exchange buffers (no counterpart in the reference). A dispatch buffer is `world`
 * blocks of `cap` rows, block d bound for rank d; a row is EAHMMF_EP_HDR floats of header (word 0: the
 * destination's local expert id as int bits; word 1 of a block's first row: the block's valid-row count)
 * and the D floats of the token's expert input. The caller exchanges whole blocks (equal splits of
 * cap * (D + EAHMMF_EP_HDR) floats, e.g. NCCL all-to-all), so no split size has to reach the host.
 *  - ep_pack: slot s = t*K + k of this rank's routing (d_ids/d_w [T x K], rank order, global expert ids
 *    < E_loc * world) goes to rank d_ids[s] / E_loc, at the next row of that block in slot order.
 *    d_token_pos[t*K + j] receives the position (d * cap + row) of token t's j-th slot by ascending
 *    expert id, d_pos_w[position] its weight: eahmmf_cuda_moe_combine over the returned rows with these
 *    gives the reference's expert-ascending sum. Needs cap >= T*K (else EAHMMF_ST_CAPACITY).
 *  - ep_unpack (receiver): the valid rows of the received blocks, compacted to the front of d_rows
 *    [world*cap x D] in ascending local-expert order (within an expert in (source, row) order; in
 *    (source, row) order alone when world*cap > 4096), their experts in d_eid (-1 and zero rows after
 *    them), and d_src = the received position of each compact row (-1 after). d_y (optional) is
 *    zeroed. Rows of one expert together let eahmmf_cuda_moe_experts read its weights once.
 *  - ep_return: d_ret[d_src[j]] = d_y[j] for the valid compact rows, d_ret being the return buffer
 *    (world blocks of cap D-float rows) that travels back by the inverse exchange. */
#define EAHMMF_EP_HDR 4
int eahmmf_cuda_ep_pack(const int* d_ids, const float* d_w, const float* d_xn, int T, int K, int D, int E_loc,
                        int world, int cap, float* d_send, int* d_token_pos, float* d_pos_w, void* stream,
                        int* d_status);
int eahmmf_cuda_ep_unpack(const float* d_recv, int D, int world, int cap, float* d_rows, int* d_eid, int* d_src,
                          float* d_y, void* stream);
int eahmmf_cuda_ep_return(const float* d_y, const int* d_src, int D, int world, int cap, float* d_ret, void* stream);

/* Stage timing of eahmmf_cuda_moe_layer: when enabled, each call records CUDA events on its stream
 * around its four stages (router GEMV, routing + activation prep, gate/up, down + combine) of every
 * 64-token block (on the grouped tensor-core path: router GEMV, routing + dequantization + activation
 * packing, the two GEMMs with the h repack between them, combine) and waits for them; eahmmf_cuda_moe_profile_read returns the mean stage durations (us)
 * over the blocks since the last read (or enable) and restarts the average. The events serialise the
 * stages (each kernel timed on its own) and the wait makes each call synchronous. Off by default;
 * single-threaded use. */
int eahmmf_cuda_moe_profile(int enable);
int eahmmf_cuda_moe_profile_read(float* us, int cap);

/* Dense quantized GEMV on device buffers: d_out[t*ldo + r] (=, or += when accumulate) dot(row r, d_x[t*ldx..]),
 * the reference's matmul (qwen3moe.cpp:397-419) with device activations. K-quant rows run on the tensor
 * cores once the activations are in fragment form, which needs eahmmf_cuda_gemv_workspace_bytes(ne0)
 * bytes of workspace (256-byte aligned); without a workspace every type takes the per-row kernel. */
size_t eahmmf_cuda_gemv_workspace_bytes(int ne0);
int eahmmf_cuda_gemv(const uint8_t* d_w, int type, int ne0, int ne1, size_t row_bytes, const float* d_x, int nb,
                     int ldx, float* d_out, int ldo, int accumulate, void* d_workspace, size_t workspace_bytes,
                     void* stream);

/* eahmmf_cuda_gemv without a caller workspace and without any allocation: no counterpart in the
 * reference (its expert_cuda.cu grows cudaMalloc'd static buffers on demand). The fragment-form
 * activations go to a fixed __device__ array of 224 KiB, enough for rows of up to
 * EAHMMF_GEMV_STATIC_MAX_NE0 elements; a longer ne0 returns EAHMMF_ST_CAPACITY before anything is
 * launched. Results are identical to eahmmf_cuda_gemv's.
 *   - The first call on each device, with that device current, looks up the array's address
 *     (cudaGetSymbolAddress) and keeps it; make that first call before any stream capture begins.
 *   - There is one array per device: calls that overlap on the same device (several streams or
 *     host threads) race on it and must be serialised by the caller. */
#define EAHMMF_GEMV_STATIC_MAX_NE0 16384
int eahmmf_cuda_gemv_static(const uint8_t* d_w, int type, int ne0, int ne1, size_t row_bytes, const float* d_x,
                            int nb, int ldx, float* d_out, int ldo, int accumulate, void* stream);

/* ---- token sampler ---------------------------------------------------------------------------- */

/* Parameters of the reference's Sampler (qwen3moe.cpp:1090-1094; CLI defaults temp 0.7, top_p 0.8,
 * min_p 0, rep 1.05, top_k 20, rep_n 64). */
typedef struct EahmmfSamplerParams {
    float temp, top_p, min_p, rep;
    int top_k, rep_n;
} EahmmfSamplerParams;

/* Sampler::sample (qwen3moe.cpp:1095-1130) on the device for one logits row of n entries:
 *   the repetition penalty over the last rep_n entries of d_hist (each occurrence divides a positive
 *   logit by rep, multiplies another by it; d_logits is modified in place, as the reference's are);
 *   temp <= 0: the first maximum; else the top_k largest logits in (value desc, index asc) order,
 *   p_i = exp((l_i - max) / temp) normalised by their sequential sum, the min-p and top-p cuts, and the
 *   first i whose running sum reaches r = u * (sum of the kept p), u being the caller's draw of the
 *   reference's std::uniform_real_distribution<float> from its std::mt19937_64 (eahmmf_rng_uniform).
 * The token goes to *d_token. Takes 1 <= top_k <= 256 when temp > 0 (else EAHMMF_ST_BAD_ARG) and
 * n <= 262144. Workspace: eahmmf_cuda_sample_workspace_bytes(n) bytes, 16-byte aligned. Asynchronous. */
size_t eahmmf_cuda_sample_workspace_bytes(int n);
int eahmmf_cuda_sample(float* d_logits, int n, const int* d_hist, int n_hist, const EahmmfSamplerParams* p, float u,
                       int* d_token, void* d_workspace, size_t workspace_bytes, void* stream);

/* The reference sampler's random stream: std::mt19937_64 seeded as Sampler::rng.seed(seed)
 * (qwen3moe.cpp:1231), and one draw of std::uniform_real_distribution<float>(0, 1) -- the canonical
 * value the reference's uniform_real_distribution(0, total) scales by total. */
typedef struct EahmmfRng EahmmfRng;
EahmmfRng* eahmmf_rng_create(uint64_t seed);
float eahmmf_rng_uniform(EahmmfRng* r);
void eahmmf_rng_free(EahmmfRng* r);

/* ---- 3. device backend (eahmmf::B200Device) --------------------------------------------------- */

typedef struct EahmmfDev EahmmfDev;
/* Binds the calling thread's current device; staging_bytes of pinned host memory (two halves) stage
 * pageable sources so host->device copies run as DMA on a non-blocking side stream. */
EahmmfDev* eahmmf_dev_create(size_t staging_bytes);
void eahmmf_dev_destroy(EahmmfDev* d);
void* eahmmf_dev_alloc(EahmmfDev* d, size_t bytes);        /* NULL on failure (DeviceBackend::alloc) */
void eahmmf_dev_release(EahmmfDev* d, void* p, size_t bytes);
bool eahmmf_dev_h2d(EahmmfDev* d, void* dst, const void* src, size_t n); /* enqueued; valid after sync */
bool eahmmf_dev_d2h(EahmmfDev* d, void* dst, const void* src, size_t n); /* complete on return */
bool eahmmf_dev_sync(EahmmfDev* d);
size_t eahmmf_dev_total_memory(EahmmfDev* d);
size_t eahmmf_dev_free_memory(EahmmfDev* d);
void* eahmmf_dev_stream(EahmmfDev* d); /* the side stream (cudaStream_t) */
/* Test hook: the next n calls of the given kind fail before any CUDA call is made
 * (kind 0 alloc, 1 h2d, 2 d2h). */
void eahmmf_dev_inject_fault(EahmmfDev* d, int kind, int n);

/* ---- 4. device-resident engine (qwen3moe forward pass) ----------------------------------------- */

/* A whole qwen3moe GGUF model in HBM: Engine::load / forward / eval (qwen3moe.cpp:858-1084) with every
 * step on the GPU: embedding, RMSNorm, fused q|k|v GEMV, QK-norm + NeoX RoPE, KV cache (fp32, n_ctx
 * positions), causal GQA attention, o-projection, the MoE block of group 2, output GEMV, argmax. One
 * decode step is a captured CUDA graph; the next token and position stay on the device. Token ids and
 * logits cross the host boundary only at the calls below. Single-threaded use per engine. */
typedef struct EahmmfEngine EahmmfEngine;

/* Loads the GGUF (qwen3moe architecture, head size 64 or 128, D and FF multiples of 256, expert
 * types Q4_K/Q5_K/Q6_K) into device memory; n_ctx is capped by the model's context_length as in
 * Engine::load (qwen3moe.cpp:879). NULL on failure, with a message in err (if given). */
EahmmfEngine* eahmmf_engine_load(const char* gguf_path, int n_ctx, char* err, size_t err_cap);
void eahmmf_engine_free(EahmmfEngine* e);
/* Expert residency beyond HBM (the reference's reason to exist: eahmmf.h's RAM/VRAM tiers, with the
 * asynchronous prefetch its README lists as not implemented): the model loads with only the non-expert
 * tensors in HBM; expert bytes stay in the mapped GGUF (registered with the driver for DMA) and a device
 * cache of expert_vram_bytes holds whole experts (at least one layer's worth). Each MoE pass reads back
 * its routing, makes every routed expert resident (a hit waits for a fill in flight; a miss evicts the
 * least recently used expert the pass does not need), uploads the layer's pointer table and starts, on a
 * second stream, the fills of the experts the next layer routed at its last pass, which overlap this
 * layer's expert kernels. Results are those of the fully resident engine (the same kernels over the same
 * bytes). Decode steps run without the captured graph (the host acts inside each step). */
EahmmfEngine* eahmmf_engine_load_budget(const char* gguf_path, int n_ctx, size_t expert_vram_bytes, char* err,
                                        size_t err_cap);
/* Cache counters: [0] slots (experts), [1] hits, [2] misses, [3] prefetch fills, [4] hits on prefetched
 * experts, [5] evictions, [6] bytes copied host -> device, [7] 1 when fills are DMA from the registered
 * mapping. All zero for a fully resident engine. */
#define EAHMMF_CACHE_STATS 8
int eahmmf_engine_cache_stats(EahmmfEngine* e, uint64_t* v, int cap);
/* dims[0..10] = n_layer, D, n_head, n_kv, hd, n_expert, n_used, FF, n_vocab, n_ctx, embedding rows */
int eahmmf_engine_dims(EahmmfEngine* e, int* dims);
/* Engine::eval (qwen3moe.cpp:1078-1084): n tokens from position p0 in forward passes of n_batch
 * (<= 64) tokens; logits (n_vocab floats, host, optional) of the last token. */
int eahmmf_engine_eval(EahmmfEngine* e, const int* toks, int n, int p0, int n_batch, float* logits);
/* Greedy generation (temperature 0, repeat penalty 1.0; std::max_element's first maximum,
 * qwen3moe.cpp:1103): the prompt from position 0, then n_gen tokens, out[0] being the argmax of the
 * prompt's logits. first_logits (optional) receives those logits. */
int eahmmf_engine_greedy(EahmmfEngine* e, const int* prompt, int n_prompt, int n_gen, int n_batch, int* out,
                         float* first_logits);
/* Token selection of the engine's generation: p NULL = the first maximum (the default; greedy); else the
 * reference's sampler with these parameters (eahmmf_cuda_sample's contract, on the device inside every
 * decode step) and its random stream seeded with `seed` (one draw per generated token, continuing across
 * generations as the reference's Sampler::rng does). Replaces the captured decode step. */
int eahmmf_engine_sampler(EahmmfEngine* e, const EahmmfSamplerParams* p, uint64_t seed);
/* The reference's generate loop (qwen3moe.cpp:1294-1310) with the engine's selection: the prompt from
 * position 0, then n_gen tokens, out[0] chosen from the prompt's logits; the history the repetition
 * penalty reads is the tokens generated by this call (hist, :1285, :1301). eahmmf_engine_greedy is this
 * with the first-maximum selection and returns EAHMMF_ST_BAD_ARG while a sampler is configured. */
int eahmmf_engine_generate(EahmmfEngine* e, const int* prompt, int n_prompt, int n_gen, int n_batch, int* out);
/* Continues generation for n_steps tokens from the engine's current state (after eval or greedy):
 * each step feeds the last argmax token. device_ms (optional) = device time of the steps (CUDA events
 * on the engine's stream); out (optional) receives the tokens. */
int eahmmf_engine_decode(EahmmfEngine* e, int n_steps, int* out, float* device_ms);
/* One greedy decode step driven from the host, as the reference's generate loop feeds one token per
 * eval call (qwen3moe.cpp:1294-1310; greedy = first maximum, :1103): `token` (>= 0) is copied in as the
 * step's input (negative: the engine's own last argmax), one forward pass at the engine's position (the
 * captured graph), and the argmax is copied back to *next; synchronous. Returns the kernels' status bits
 * (EAHMMF_ST_BAD_ARG when the context is full). */
int eahmmf_engine_step(EahmmfEngine* e, int token, int* next);
/* Several sequences at once (no counterpart in the reference, whose Engine holds one sequence,
 * qwen3moe.cpp:791, :910-913): the engine keeps n_slots sequences, each with its own KV cache of n_ctx
 * positions, and a step runs one token of each of up to 64 sequences as one forward pass (the dense and
 * expert projections batched over the rows, attention per row over its own sequence's cache).
 *  - set_slots: caches for n_slots sequences, zeroed (the single-sequence calls above use slot 0);
 *  - prefill_slot: a new sequence in `slot`: the prompt from position 0 (passes of n_batch), the first
 *    maximum of its logits into *first;
 *  - step_slots: one greedy step: row i feeds toks[i] to sequence slots[i] at position pos[i] (its next
 *    free position; distinct slots) and receives the first maximum of that row's logits in next[i].
 * Per-row results are those of the single-sequence calls (the same kernels' per-token arithmetic). */
int eahmmf_engine_set_slots(EahmmfEngine* e, int n_slots);
int eahmmf_engine_prefill_slot(EahmmfEngine* e, int slot, const int* prompt, int n, int n_batch, int* first);
int eahmmf_engine_step_slots(EahmmfEngine* e, int n, const int* slots, const int* pos, const int* toks, int* next);
/* The residency layer's --verify contract (Config::verify, eahmmf.h:203-214: every copy checksummed
 * against its GGUF source with hash64, eahmmf.h:64-76, :940, :1014) for the engine's HBM copy: the hash64
 * of every expert component (layers x experts x gate/up/down) computed on the device in one launch, the
 * source's on the host from the GGUF file as it is now; *n_bad counts the components that differ.
 * Synchronous; allocates a small table for the launch. */
int eahmmf_engine_verify(EahmmfEngine* e, int* n_checked, int* n_bad);
/* Routing trace (Engine::trace_routing, qwen3moe.cpp:1021): when enabled, every forward pass appends
 * each layer's top-k ids and weights, layer-major; trace_get copies up to cap entries and returns the
 * total. Tracing runs decode steps without the graph. */
void eahmmf_engine_trace(EahmmfEngine* e, int enable);
int eahmmf_engine_trace_get(EahmmfEngine* e, int* ids, float* w, int cap);
/* Kernel launches in one captured decode step (nodes of its CUDA graph); 0 before the first capture. */
int eahmmf_engine_graph_nodes(EahmmfEngine* e);
/* Per-operation timing of decode steps: when enabled, steps run without the graph and record CUDA
 * events between the operations of the pass; profile_read returns the mean device time per step (us)
 * of each class, summed over layers: [0] embedding + rotary table, [1] attention RMSNorm, [2] q|k|v
 * GEMV, [3] QK-norm + RoPE + KV append, [4] attention, [5] o-projection, [6] FFN RMSNorm, [7] MoE block,
 * [8] output RMSNorm + GEMV, [9] argmax, and restarts the average. Returns the number of classes. */
#define EAHMMF_ENGINE_PROFILE_CLASSES 10
int eahmmf_engine_profile(EahmmfEngine* e, int enable);
int eahmmf_engine_profile_read(EahmmfEngine* e, float* us, int cap);

/* hash64 (eahmmf.h:64-76) of n device byte ranges d_ptrs[i] .. + d_sizes[i] (device arrays) into
 * d_out[i], one warp per range; and the same on the host. */
int eahmmf_cuda_hash64(const uint8_t* const* d_ptrs, const size_t* d_sizes, int n, uint64_t* d_out, void* stream);
uint64_t eahmmf_hash64(const uint8_t* p, size_t n);

/* ---- misc ------------------------------------------------------------------------------------ */
const char* eahmmf_b200_version(void);
int eahmmf_b200_sm_count(void);

#ifdef __cplusplus
}
#endif
#endif
