// sample.cu -- the reference's token sampler on the GPU (Sampler::sample, qwen3moe.cpp:1090-1130):
// repetition penalty over the last rep_n generated tokens, then either the first maximum (temp <= 0) or
// top-k by value, softmax numerators at temperature `temp` relative to the maximum, normalisation,
// min-p and top-p cuts, and the inverse-CDF pick of a uniform draw r in [0, total). Three launches:
//
//   k_sample_penalty   one block: each distinct token of the window is divided (positive logit) or
//                      multiplied (otherwise) by `rep` once per occurrence, as the reference's loop does
//                      one occurrence at a time; the logits are modified in place, as the reference's are;
//   k_sample_cand      blocks of SAMPLE_BLK logits: 64-bit keys (orderable value bits << 32 | ~index)
//                      sorted descending in shared memory (bitonic), the block's first SAMPLE_KMAX kept;
//   k_sample_finish    one block: the candidates sorted the same way -- the global order by (value desc,
//                      index asc) -- and one thread runs the reference's arithmetic over the first
//                      top_k in its order: fp32 differences and divisions, the sums taken sequentially in
//                      rank order, r = u * total with u the canonical draw of the reference's
//                      std::uniform_real_distribution<float> (drawn on the host from the same
//                      std::mt19937_64 stream, eahmmf_rng_*).
//
// Numerics: the softmax numerators are the correctly rounded float of exp((double)x) -- glibc's expf,
// which the reference calls, agrees except within a few thousandths of an ulp of a rounding boundary.
// Equal logits are ordered by lower index (std::partial_sort leaves their order unspecified). NaN logits
// rank last.
#include <cstdint>
#include <random>

#include "../../include/eahmmf_b200.h"
#include "common.cuh"
#include "decode.cuh"
#include "sample.cuh"

namespace eb {
namespace {

constexpr int PEN_NT = 256;
constexpr int CAND_NT = 1024;
constexpr int FIN_NT = 1024;

__device__ __forceinline__ uint32_t okey(float f) {  // larger float -> larger key; NaN -> 0
    const uint32_t b = __float_as_uint(f);
    if (f != f) return 0u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float kval(uint64_t k) {
    const uint32_t u = (uint32_t)(k >> 32);
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}
__device__ __forceinline__ int kidx(uint64_t k) { return (int)~(uint32_t)k; }

// Descending bitonic sort of n (a power of two) keys in shared memory by the whole block.
__device__ void bitonic_desc(uint64_t* s, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
                const int lo = 2 * i - (i & (j - 1));  // first index of the pair whose partner is lo + j
                const int hi = lo + j;
                const bool desc = (lo & k) == 0;
                const uint64_t a = s[lo], b = s[hi];
                if (desc ? a < b : a > b) {
                    s[lo] = b;
                    s[hi] = a;
                }
            }
            __syncthreads();
        }
    }
}

// The generated-token window and this call's draw, from the arguments or from the engine's state.
struct Src {
    const int* hist;
    int n_hist;
    float u;
};
__device__ __forceinline__ Src source(const SampleArgs& a) {
    Src s{a.hist, a.n_hist, a.u};
    if (a.st) {
        const int n = a.st->n_out;
        s.hist = a.st->out;
        s.n_hist = n < a.st->cap_out ? n : a.st->cap_out;
        s.u = a.u_arr ? a.u_arr[n] : 0.f;
    }
    return s;
}

__global__ void __launch_bounds__(PEN_NT) k_sample_penalty(SampleArgs a) {
    pdl_wait();  // the logits come from the previous grid
    pdl_trigger();
    if (a.p.rep == 1.0f || a.p.rep_n <= 0) return;
    const Src s = source(a);
    const int from = s.n_hist > a.p.rep_n ? s.n_hist - a.p.rep_n : 0, w = s.n_hist - from;
    for (int i = threadIdx.x; i < w; i += PEN_NT) {
        const int t = s.hist[from + i];
        bool first = true;
        int m = 0;
        for (int j = 0; j < w; j++) {
            const int v = s.hist[from + j];
            if (v == t) {
                m++;
                if (j < i) first = false;
            }
        }
        if (!first || t < 0 || t >= a.n) continue;
        float x = a.logits[t];
        for (int r = 0; r < m; r++) x = x > 0.f ? __fdiv_rn(x, a.p.rep) : __fmul_rn(x, a.p.rep);
        a.logits[t] = x;
    }
}

__global__ void __launch_bounds__(CAND_NT) k_sample_cand(SampleArgs a) {
    __shared__ uint64_t s[SAMPLE_BLK];
    pdl_wait();  // the penalised logits
    pdl_trigger();
    const int base = blockIdx.x * SAMPLE_BLK;
    for (int i = threadIdx.x; i < SAMPLE_BLK; i += CAND_NT) {
        const int e = base + i;
        s[i] = e < a.n ? ((uint64_t)okey(a.logits[e]) << 32) | (uint32_t)~(uint32_t)e : 0ull;
    }
    __syncthreads();
    bitonic_desc(s, SAMPLE_BLK);
    for (int i = threadIdx.x; i < SAMPLE_KMAX; i += CAND_NT) a.cand[(size_t)blockIdx.x * SAMPLE_KMAX + i] = s[i];
}

__global__ void __launch_bounds__(FIN_NT) k_sample_finish(SampleArgs a, int ncand, int npow2) {
    extern __shared__ __align__(16) uint64_t s[];
    __shared__ float p[SAMPLE_KMAX];
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < npow2; i += FIN_NT) s[i] = i < ncand ? a.cand[i] : 0ull;
    __syncthreads();
    bitonic_desc(s, npow2);
    if (threadIdx.x != 0) return;
    const Src src = source(a);
    const EahmmfSamplerParams& P = a.p;
    int tok;
    if (P.temp <= 0.f) {
        tok = s[0] ? kidx(s[0]) : 0;  // every logit NaN: std::max_element returns the first
    } else {
        const int keep = P.top_k < a.n ? P.top_k : a.n;
        const float mx = kval(s[0]);
        float sum = 0.f;
        for (int i = 0; i < keep; i++) {
            p[i] = (float)exp((double)__fdiv_rn(__fsub_rn(kval(s[i]), mx), P.temp));
            sum = __fadd_rn(sum, p[i]);
        }
        for (int i = 0; i < keep; i++) p[i] = __fdiv_rn(p[i], sum);
        int cut = keep;
        if (P.min_p > 0.f) {
            const float lim = __fmul_rn(P.min_p, p[0]);
            cut = 0;
            while (cut < keep && p[cut] >= lim) cut++;
        }
        if (P.top_p < 1.0f) {
            float cum = 0.f;
            int k = 0;
            while (k < cut) {
                cum = __fadd_rn(cum, p[k++]);
                if (cum >= P.top_p) break;
            }
            cut = k;
        }
        float tot = 0.f;
        for (int i = 0; i < cut; i++) tot = __fadd_rn(tot, p[i]);
        const float r = __fadd_rn(__fmul_rn(src.u, __fsub_rn(tot, 0.f)), 0.f);  // uniform(0, tot): u (b - a) + a
        tok = cut > 0 ? kidx(s[cut - 1]) : kidx(s[0]);
        float acc = 0.f;
        for (int i = 0; i < cut; i++) {
            acc = __fadd_rn(acc, p[i]);
            if (r <= acc) {
                tok = kidx(s[i]);
                break;
            }
        }
    }
    if (a.st) {
        DecodeState* st = a.st;
        st->token = tok;
        if (st->n_out < st->cap_out) st->out[st->n_out] = tok;
        st->n_out++;
        if (a.advance) st->pos += 1;
    } else {
        *a.token = tok;
    }
}

}  // namespace

size_t sample_ws_bytes(int n) { return (size_t)((n + SAMPLE_BLK - 1) / SAMPLE_BLK) * SAMPLE_KMAX * 8; }

bool sample_ok(const EahmmfSamplerParams& p, int n) {
    if (n < 1 || (n + SAMPLE_BLK - 1) / SAMPLE_BLK * SAMPLE_KMAX > SAMPLE_FIN_MAX) return false;
    if (p.temp > 0.f && (p.top_k < 1 || p.top_k > SAMPLE_KMAX)) return false;
    return !(p.rep != p.rep) && p.rep != 0.f;
}

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t st) {
    const int nblk = (a.n + SAMPLE_BLK - 1) / SAMPLE_BLK, ncand = nblk * SAMPLE_KMAX;
    int np2 = 1;
    while (np2 < ncand) np2 <<= 1;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(k_sample_finish, cudaFuncAttributeMaxDynamicSharedMemorySize, SAMPLE_FIN_MAX * 8) !=
            cudaSuccess)
            return cudaErrorInvalidValue;
        attr = true;
    }
    cudaError_t e = launch_pdl(k_sample_penalty, dim3(1), dim3(PEN_NT), 0, st, a);
    if (e == cudaSuccess) e = launch_pdl(k_sample_cand, dim3(nblk), dim3(CAND_NT), 0, st, a);
    if (e == cudaSuccess) e = launch_pdl(k_sample_finish, dim3(1), dim3(FIN_NT), (size_t)np2 * 8, st, a, ncand, np2);
    return e;
}

}  // namespace eb

using namespace eb;

// ---- C ABI -------------------------------------------------------------------------------------------
struct EahmmfRng {
    std::mt19937_64 g;
};

extern "C" EahmmfRng* eahmmf_rng_create(uint64_t seed) {
    EahmmfRng* r = new EahmmfRng();
    r->g.seed(seed);
    return r;
}
extern "C" void eahmmf_rng_free(EahmmfRng* r) { delete r; }
extern "C" float eahmmf_rng_uniform(EahmmfRng* r) {
    return r ? std::uniform_real_distribution<float>(0.f, 1.f)(r->g) : 0.f;
}

extern "C" size_t eahmmf_cuda_sample_workspace_bytes(int n) { return n > 0 ? sample_ws_bytes(n) : 0; }

extern "C" int eahmmf_cuda_sample(float* d_logits, int n, const int* d_hist, int n_hist,
                                  const EahmmfSamplerParams* p, float u, int* d_token, void* d_workspace,
                                  size_t workspace_bytes, void* stream) {
    if (!d_logits || !p || !d_token || !d_workspace || n_hist < 0 || (n_hist > 0 && !d_hist) || !sample_ok(*p, n))
        return ST_BAD_ARG;
    if (workspace_bytes < sample_ws_bytes(n) || (reinterpret_cast<uintptr_t>(d_workspace) & 15)) return ST_CAPACITY;
    SampleArgs a{};
    a.logits = d_logits;
    a.n = n;
    a.p = *p;
    a.hist = d_hist;
    a.n_hist = n_hist;
    a.u = u;
    a.token = d_token;
    a.cand = static_cast<uint64_t*>(d_workspace);
    return launch_sample(a, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? ST_OK : ST_CUDA;
}
