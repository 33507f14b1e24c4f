/* oracle/oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference's CPU algorithm for the MoE expert hot path. It is the parity
 * checker for the CUDA library and the "port" CPU baseline; the product never links it. Every function
 * names the reference lines (qwen3moe.cpp) it restates. Pinned by tests/test_oracle_golden.py against
 * the reference compiled from its own sources (oracle/_ref), against gguf-py's independent dequantizer,
 * and -- through the reference engine -- against the reference's golden vectors (baseline/logits.txt,
 * baseline/gen_greedy.bin).
 */
#ifndef EAHMMF_ORACLE_H
#define EAHMMF_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids used on the path (qwen3moe.cpp:204-218). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q5_K = 13, ORC_Q6_K = 14 };

float orc_f16(uint16_t h);                                  /* f16_slow, qwen3moe.cpp:56-63 */
int orc_block_size(int type);                               /* elements per block, 0 if unsupported */
int orc_block_bytes(int type);                              /* bytes per block, 0 if unsupported */
int orc_dequant_row(int type, const uint8_t* row, int64_t ne0, float* y); /* dq_*, :78-202 */

/* out[t*ldo + r] = dot(dequant(row r), x[t*ldx ..]), r < ne1, t < nb  (matmul, :397-419). 0 = ok. */
int orc_matmul(const uint8_t* w, int type, int64_t ne0, int64_t ne1, size_t row_bytes, const float* x, int nb,
               int ldx, float* out, int ldo);

/* rmsnorm, :527-532 (one row). */
void orc_rmsnorm(const float* x, const float* w, float* out, int n, float eps);

/* Router softmax + top-k + renormalisation for one token, :1011-1023. r (E floats) is overwritten
 * with expf(l - max) exactly as the reference does; ids/w receive the K choices in rank order. */
void orc_route_token(float* r, int E, int K, int* ids, float* w);

/* Whole MoE layer for T tokens (:1008-1069): routing from logits (T*E) or, when logits == NULL, from
 * router_w (F32 E*D) applied to xn; experts visited in ascending id; x (T*D) += weighted expert sum.
 * trace_ids/trace_w (T*K, optional) receive the routing. 0 = ok. */
int orc_moe_layer(int T, int D, int FF, int E, int K, const float* xn, const float* logits, const float* router_w,
                  const uint8_t* const* gate, const uint8_t* const* up, const uint8_t* const* down, int gt, int ut,
                  int dt, size_t grb, size_t urb, size_t drb, float* x, int* trace_ids, float* trace_w);

#ifdef __cplusplus
}
#endif
#endif
