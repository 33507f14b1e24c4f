// common.cuh -- shared definitions of the sm_100a expert hot path: ggml type ids, status codes and the
// TMA-bulk / mbarrier helpers.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace eb {

// ggml type ids handled on the path (the reference's table: qwen3moe.cpp:204-218).
constexpr int T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14;

__host__ __device__ constexpr int block_elems(int t) { return (t == T_Q4_K || t == T_Q5_K || t == T_Q6_K) ? 256 : 32; }
__host__ __device__ constexpr int block_bytes(int t) {
    return t == T_Q4_K ? 144 : t == T_Q5_K ? 176 : t == T_Q6_K ? 210 : t == T_Q8_0 ? 34 : t == T_F16 ? 64 : t == T_F32 ? 128 : 0;
}
__host__ __device__ constexpr bool is_kquant(int t) { return t == T_Q4_K || t == T_Q5_K || t == T_Q6_K; }
__host__ __device__ constexpr bool type_supported(int t) {
    return t == T_F32 || t == T_F16 || t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K;
}

// Status bits written by kernels into a device status word (atomicOr) and returned by the C ABI.
enum : int {
    ST_OK = 0,
    ST_BAD_ARG = 1 << 0,       // host-side argument validation failed
    ST_BAD_TYPE = 1 << 1,      // unsupported ggml type
    ST_CUDA = 1 << 2,          // a CUDA runtime call failed
    ST_WAIT_TIMEOUT = 1 << 3,  // a bounded mbarrier wait gave up (copy never completed)
    ST_BAD_INDEX = 1 << 4,     // an expert id / token index out of range reached a kernel
    ST_CAPACITY = 1 << 5,      // a size exceeded the workspace the caller provided
};

// Activations in fragment form ("XF", layout in kq.cuh), rows of K elements:
//   frag   rows x K*3 bytes: three int8 digits per element in MMA B-fragment order
//   sum    rows x (K/16 + 4) floats: the per-16 sums of the row, then the row scale s and three zeros
//          (the dense GEMV's minimum terms)
//   gs     rows x (16 + K/8) bytes: the row scale s (float, then 12 zero bytes), then per super-block
//          32 bytes: the eight 32-element group sums of the row divided by s, as f16 high parts
//          (16 bytes) and f16 residues (16 bytes) -- the B operand of the expert kernels' minimum-term
//          MMA; divided by s they are bounded by 32 * 127 and fit f16
struct XF {
    const uint2* frag;
    const float* sum;
    const uint8_t* gs;
    int nseg;  // K / 16
};
constexpr int XF_SUM_PAD = 4;  // floats after a row's segment sums (scale + padding to 16 bytes)
__host__ __device__ constexpr int xf_gs_bytes(int K) { return 16 + K / 8; }

// Programmatic dependent launch. A kernel launched with launch_pdl may start while its predecessor on
// the stream is still running; it must call pdl_wait() before touching anything the predecessor
// writes (and every kernel of a chain calls it, so completion is transitive). pdl_trigger() lets the
// successor launch early; every kernel calls it right after its own pdl_wait(), so at most one kernel
// waits ahead of the running one (successors launched further ahead would hold SM resources that the
// running kernel's remaining blocks need).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, const Args&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

// Sum of squares of a row of K floats (K % 4 == 0, 16-byte aligned) by the first 128 threads of a block
// (blockDim.x >= 128, a multiple of 32; every thread calls it), in one fixed order: every RMSNorm uses
// it, so the result does not depend on which kernel (or how many tokens per pass) computed it. red4: 4
// floats of shared memory.
__device__ __forceinline__ float row_sumsq128(const float* __restrict__ x, int K, float* red4) {
    float ss = 0.f;
    if (threadIdx.x < 128) {  // larger blocks: threads 128.. add nothing, so the order stays the same
        for (int i = threadIdx.x; i < K / 4; i += 128) {
            const float4 v = reinterpret_cast<const float4*>(x)[i];
            ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0 && threadIdx.x < 128) red4[threadIdx.x >> 5] = ss;
    __syncthreads();
    return (red4[0] + red4[1]) + (red4[2] + red4[3]);
}

// Exact 2^e for -126 <= e <= 127.
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }

// ---------------------------------------------------------------------------------------------
// TMA bulk copies and mbarriers (single-CTA clusters).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// try_wait with a suspend-time hint: the waiting thread sleeps in hardware until the phase completes
// (or the hint expires) instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: gives up after WAIT_LIMIT_NS of wall time (a bulk copy lands in microseconds), so a
// copy that never completes ends the kernel with ST_WAIT_TIMEOUT instead of hanging the GPU.
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) return false;
    }
}
// 1-D bulk copy global -> shared, completion counted on bar. dst, src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float f16_to_f32(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }

// x / (1 + exp(-x)) * u, the SiLU-gated product of qwen3moe.cpp:1056-1059 (IEEE division).
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdiv_rn(g, 1.0f + expf(-g)) * u; }

}  // namespace eb
