// sample.cuh -- launch-side declarations of the token sampler (sample.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/eahmmf_b200.h"
#include "decode.cuh"

namespace eb {

constexpr int SAMPLE_BLK = 4096;      // logits per candidate block
constexpr int SAMPLE_KMAX = 256;      // candidates kept per block: the largest top_k the sampler takes
constexpr int SAMPLE_FIN_MAX = 16384; // candidates the finishing block sorts (n <= 64 * SAMPLE_BLK)

struct SampleArgs {
    float* logits;  // [n], penalised in place
    int n;
    EahmmfSamplerParams p;
    // stateless call: the window of generated tokens, this call's uniform draw, the output
    const int* hist;
    int n_hist;
    float u;
    int* token;
    // engine step (st set): hist = st->out[0 .. n_out), u = u_arr[st->n_out]; the token goes to st as the
    // argmax kernel writes it (token, out[n_out], n_out + 1, pos + advance)
    DecodeState* st;
    const float* u_arr;
    int advance;
    uint64_t* cand;  // sample_ws_bytes(n) of scratch
};

size_t sample_ws_bytes(int n);
bool sample_ok(const EahmmfSamplerParams& p, int n);
cudaError_t launch_sample(const SampleArgs& a, cudaStream_t st);

}  // namespace eb
