// decode.cuh -- launch-side declarations of the forward-pass kernels outside the expert block
// (decode.cu) and the device-resident decode state they share.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace eb {

constexpr int ATT_CH = 64;       // context positions per attention chunk
constexpr int ATT_NT = 256;      // threads of an attention block (8 warps)
constexpr int ATT_MAXH = 2;      // q heads per warp: GQA groups of up to 16 heads per kv head
constexpr int ARGMAX_NT = 1024;  // threads of an argmax block

// Device-resident state of a generation: the position of the next forward pass, the token it feeds
// (written by the argmax), and the output history. Kernels read `pos` at run time, so a captured
// decode step replays unchanged.
struct DecodeState {
    int pos;      // position of the first token of the next forward pass
    int token;    // next input token (argmax of the last logits)
    int ticket;   // argmax block counter (reset by the last block)
    int n_out;    // tokens recorded so far
    int cap_out;  // capacity of out
    int slot_rows;     // cache rows per sequence slot (multi-sequence steps)
    int* out;          // [cap_out] generated tokens
    const int* tpos;   // multi-sequence step: [nb] position of each token row (null: pos + t)
    const int* tslot;  // multi-sequence step: [nb] sequence slot of each row, whose cache rows start at
                       // slot * slot_rows of the layer's cache (null: the cache passed in, row = position)
};
// Position of token row t of a forward pass, and the first cache row of its sequence.
__device__ __forceinline__ int tok_pos(const DecodeState* st, int t) { return st->tpos ? st->tpos[t] : st->pos + t; }
__device__ __forceinline__ size_t tok_base(const DecodeState* st, int t) {
    return st->tslot ? (size_t)st->tslot[t] * (size_t)st->slot_rows : 0;
}

// Arguments of k_norm_prep: rows t0 .. t0 + rows - 1 of x (row length n, stride ldx); when y is set,
// first x[t] += sum_k slot_w[s] y[s] over s = token_slots[t*K + k]; then RMSNorm with w, eps; the
// normalised rows (XF row r = t - t0) go to xf and, when xn is set, to xn[r * n].
struct NormPrepArgs {
    float* x;
    int ldx, n, t0;
    const float* w;
    float eps;
    const float* y;
    const int* token_slots;
    const float* slot_w;
    int K;
    XF xf;
    float* xn;
};
cudaError_t launch_norm_prep(const NormPrepArgs& a, int rows, cudaStream_t s);
cudaError_t launch_embed(const uint8_t* W, int type, size_t rb, int D, int n_rows, const int* toks, int nb, float* x,
                         int* status, cudaStream_t s);
cudaError_t launch_rmsnorm(const float* x, int ldx, const float* w, float* out, int ldo, int rows, int n, float eps,
                           cudaStream_t s);
cudaError_t launch_rope_table(const DecodeState* st, const float* inv_freq, int half, int nb, float2* cs,
                              cudaStream_t s);
cudaError_t launch_qk_rope_kv(int hd, const float* qkv, int n_head, int n_kv, const float* qn, const float* kn,
                              float eps, const float2* cs, const DecodeState* st, int nb, float* q_out, float* kc,
                              float* vc, cudaStream_t s);
size_t attn_smem(int hd, int grp);
// Single-token steps: when qkv is set the attention kernel does the q/k head norms, the rotation and the
// KV append itself (k_qk_rope_kv is not launched); q is then unused.
struct RopeFuse {
    const float* qkv;  // [QD + 2 KD] q|k|v row of the step's token, or null
    const float* qn;
    const float* kn;
    float eps;
    const float2* cs;  // the token's HD/2 cos/sin pairs
    // merge fused into the attention launch (single-token steps): the last split block of each kv head
    // merges its q heads into att; cnt: n_kv zeroed counters (reset by that block). Null: k_attn_merge_prep
    // merges and puts the rows in fragment form.
    int* cnt;
    float* att;
};
// Attention of nb token rows (split partials in part: nb * n_head * nsplit * (hd + 2) floats, nsplit
// <= 128), then the merge of each row into att (fp32, [nb x n_head hd]) and into xf (fragment form, the
// o-projection's activations); with rf.cnt (one row) the attention launch merges into rf.att itself and
// leaves the fragment form to the o-projection's prologue. pos_host: state->pos when the host knows it
// (a prompt pass), else -1; a prompt pass at a known position whose chunks fit the splits runs the
// chunk-shared kernel (k_attn_chunk), with the same records.
cudaError_t launch_attention(int hd, const float* q, float* kc, float* vc, int n_head, int n_kv, float scale,
                             const DecodeState* st, int nb, int nsplit, float* part, float* att, const XF& xf,
                             const RopeFuse& rf, int pos_host, cudaStream_t s);
// blk: nblk float2 of scratch
cudaError_t launch_argmax(const float* lg, int n, float2* blk, int nblk, DecodeState* st, int advance, cudaStream_t s);
cudaError_t launch_advance(DecodeState* st, int n, cudaStream_t s);
// First maximum of each of `rows` logits rows (n entries each, stride ld) into out[row].
cudaError_t launch_argmax_rows(const float* lg, int n, int ld, int rows, int* out, cudaStream_t s);

}  // namespace eb
