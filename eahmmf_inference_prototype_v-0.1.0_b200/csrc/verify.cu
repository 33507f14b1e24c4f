// verify.cu -- the residency layer's checksum (hash64, eahmmf.h:64-76) computed on the device, so that a
// copy staged into HBM can be checked against its GGUF source without reading it back to the host (the
// reference checks each migration by a d2h copy and a host hash, eahmmf.h:1014).
//
// hash64 is a sequential chain over the 8-byte little-endian words of a range, then its tail bytes:
//   h = 1469598103934665603;  per word w: h ^= w; h *= 1099511628211; h ^= h >> 29;
//   per tail byte b: h ^= b; h *= 1099511628211.
// One range is one chain, so a warp takes a range: its lanes load 32 consecutive words (one coalesced
// 256-byte read, issued PREFETCH chunks ahead of use) and lane 0 folds them in order, receiving each by
// shuffle. Ranges are independent, so the grid covers all of a model's expert components at once.
#include <cstdint>

#include "../../include/eahmmf_b200.h"
#include "common.cuh"

namespace eb {
namespace {

constexpr uint64_t H_SEED = 1469598103934665603ull, H_MUL = 1099511628211ull;
constexpr int HASH_NT = 256;
constexpr int PREFETCH = 4;  // 256-byte chunks in flight per warp

__device__ __forceinline__ uint64_t load_word(const uint8_t* p, bool aligned) {
    if (aligned) return __ldg(reinterpret_cast<const unsigned long long*>(p));
    uint64_t w = 0;
#pragma unroll
    for (int b = 0; b < 8; b++) w |= (uint64_t)__ldg(p + b) << (8 * b);
    return w;
}

__global__ void __launch_bounds__(HASH_NT) k_hash64(const uint8_t* const* __restrict__ ptrs,
                                                    const size_t* __restrict__ sizes, int n,
                                                    unsigned long long* __restrict__ out) {
    const int warp = blockIdx.x * (HASH_NT / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (warp >= n) return;
    const uint8_t* p = ptrs[warp];
    const size_t bytes = sizes[warp], words = bytes / 8;
    const bool aligned = (reinterpret_cast<uintptr_t>(p) & 7) == 0;
    const size_t chunks = (words + 31) / 32;
    uint64_t h = H_SEED;
    uint64_t buf[PREFETCH];
#pragma unroll
    for (int c = 0; c < PREFETCH; c++) {
        const size_t i = (size_t)c * 32 + lane;
        buf[c] = (size_t)c < chunks && i < words ? load_word(p + 8 * i, aligned) : 0ull;
    }
    for (size_t c0 = 0; c0 < chunks; c0 += PREFETCH) {
#pragma unroll
        for (int q = 0; q < PREFETCH; q++) {  // static register indices: buf[q] holds chunk c0 + q
            const size_t c = c0 + q;
            if (c >= chunks) break;  // the same for every lane
            const uint64_t cur = buf[q];
            const size_t nc = c + PREFETCH, i = nc * 32 + lane;
            buf[q] = nc < chunks && i < words ? load_word(p + 8 * i, aligned) : 0ull;
            const int m = (int)min((size_t)32, words - c * 32);
            for (int j = 0; j < m; j++) {
                const uint64_t w = __shfl_sync(0xffffffffu, cur, j);
                h ^= w;
                h *= H_MUL;
                h ^= h >> 29;
            }
        }
    }
    if (lane == 0) {
        for (size_t i = words * 8; i < bytes; i++) {
            h ^= p[i];
            h *= H_MUL;
        }
        out[warp] = h;
    }
}

}  // namespace

cudaError_t launch_hash64(const uint8_t* const* d_ptrs, const size_t* d_sizes, int n, uint64_t* d_out,
                          cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int per = HASH_NT / 32;
    k_hash64<<<(n + per - 1) / per, HASH_NT, 0, st>>>(d_ptrs, d_sizes, n,
                                                       reinterpret_cast<unsigned long long*>(d_out));
    return cudaGetLastError();
}

// The same chain on the host, for the sources (a restatement of eahmmf.h:64-76).
uint64_t host_hash64(const uint8_t* p, size_t n) {
    uint64_t h = H_SEED;
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        uint64_t w;
        __builtin_memcpy(&w, p + i, 8);
        h ^= w;
        h *= H_MUL;
        h ^= h >> 29;
    }
    for (; i < n; i++) {
        h ^= p[i];
        h *= H_MUL;
    }
    return h;
}

}  // namespace eb

extern "C" int eahmmf_cuda_hash64(const uint8_t* const* d_ptrs, const size_t* d_sizes, int n, uint64_t* d_out,
                                  void* stream) {
    if (n < 0 || (n > 0 && (!d_ptrs || !d_sizes || !d_out))) return eb::ST_BAD_ARG;
    return eb::launch_hash64(d_ptrs, d_sizes, n, d_out, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
               ? eb::ST_OK
               : eb::ST_CUDA;
}

extern "C" uint64_t eahmmf_hash64(const uint8_t* p, size_t n) { return p || !n ? eb::host_hash64(p, n) : 0; }
