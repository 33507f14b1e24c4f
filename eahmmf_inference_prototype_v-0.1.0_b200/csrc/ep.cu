// ep.cu -- the expert-parallel exchange around the MoE block: packing of a rank's
// routed slots for the dispatch all-to-all, compaction of the rows a rank receives, and the rows that go
// back. The collectives themselves are the caller's (NCCL all-to-all with equal splits over NVLink): the
// buffers have a fixed capacity per (source, destination) pair, so no split size ever has to reach the
// host and a layer runs without a host synchronisation.
//
// Layout of a dispatch buffer: world blocks of `cap` rows, block d going to rank d. A row is EP_HDR
// floats of header followed by the D floats of the token's expert input (xn). Header word 0 is the
// destination's local expert id, word 1 of the block's first row the number of valid rows in the block
// (valid rows are the block's first rows, slots in ascending (token, k) order, so the exchange is
// deterministic). The return buffer has the same blocks with plain D-float rows.
//
// The reference has no expert parallelism; its MoE block is the single-process loop of
// qwen3moe.cpp:1008-1069, whose per-token results these kernels leave unchanged (every slot's output
// depends only on its own row, and the combine keeps the expert-ascending order).
#include <cstdint>

#include "../../include/eahmmf_b200.h"
#include "common.cuh"

namespace eb {
namespace {

constexpr int PLAN_NT = 1024;
constexpr int EP_MAX_WORLD = 64;
static_assert(EAHMMF_EP_HDR == 4, "row header of four floats keeps rows 16-byte aligned");

__device__ __forceinline__ void set_status(int* st, int bits) {
    if (st) atomicOr(st, bits);
}

// One block: positions of every slot, stable in slot order within each destination block.
//   token_pos[t*K + j] = dest*cap + i of token t's j-th slot by ascending expert id (the combine order)
//   pos_w[dest*cap + i] = the slot's routing weight;  send header word 0 = the local expert id
// and, after the last chunk, header word 1 of each block's first row = the block's count.
__global__ void __launch_bounds__(PLAN_NT) k_ep_plan(const int* __restrict__ ids, const float* __restrict__ w, int T,
                                                     int K, int D, int E_loc, int world, int cap,
                                                     float* __restrict__ send, int* __restrict__ token_pos,
                                                     float* __restrict__ pos_w, int* status) {
    __shared__ int wcnt[EP_MAX_WORLD][PLAN_NT / 32];
    __shared__ int run[EP_MAX_WORLD];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, S = T * K, row = D + EAHMMF_EP_HDR;
    if (tid < world) run[tid] = 0;
    // every position entry starts in range, so that an id the loop rejects (status raised) leaves no
    // position outside the buffers for the gather and the combine
    for (int s = tid; s < S; s += PLAN_NT) token_pos[s] = 0;
    __syncthreads();
    for (int base = 0; base < S; base += PLAN_NT) {
        const int s = base + tid;
        int e = -1, dest = -1;
        if (s < S) {
            e = __ldg(ids + s);
            if (e < 0 || e >= E_loc * world) {
                set_status(status, ST_BAD_INDEX);
                e = -1;
            } else {
                dest = e / E_loc;
            }
        }
        // per destination: the slot's rank among this chunk's slots of the same destination
        int my_rank = 0;
        for (int d = 0; d < world; d++) {
            const unsigned m = __ballot_sync(0xffffffffu, dest == d);
            if (dest == d) my_rank = __popc(m & ((1u << lane) - 1u));
            if (lane == 0) wcnt[d][warp] = __popc(m);
        }
        __syncthreads();
        if (dest >= 0) {
            int before = run[dest];
            for (int v = 0; v < warp; v++) before += wcnt[dest][v];
            const int i = before + my_rank;
            if (i >= cap) {
                set_status(status, ST_CAPACITY);
            } else {
                const int pos = dest * cap + i;
                const int t = s / K;
                int rank = 0;  // the slot's place among the token's k slots by expert id
                for (int j = 0; j < K; j++) rank += __ldg(ids + (size_t)t * K + j) < e;
                token_pos[(size_t)t * K + rank] = pos;
                pos_w[pos] = __ldg(w + s);
                send[(size_t)pos * row] = __int_as_float(e - dest * E_loc);
            }
        }
        __syncthreads();
        if (tid < world) {
            int tot = 0;
            for (int v = 0; v < PLAN_NT / 32; v++) tot += wcnt[tid][v];
            run[tid] += tot;
        }
        __syncthreads();
    }
    if (tid < world) send[(size_t)tid * cap * row + 1] = __int_as_float(min(run[tid], cap));
}

// One block per slot: the token's row into the slot's position (all of a token's slots carry its row).
__global__ void __launch_bounds__(256) k_ep_gather(const float* __restrict__ xn, int K, int D,
                                                   const int* __restrict__ token_pos, float* __restrict__ send) {
    const int s = blockIdx.x, t = s / K, row = D + EAHMMF_EP_HDR;
    const int pos = token_pos[s];
    const float4* src = reinterpret_cast<const float4*>(xn + (size_t)t * D);
    float4* dst = reinterpret_cast<float4*>(send + (size_t)pos * row + EAHMMF_EP_HDR);
    for (int i = threadIdx.x; i < D / 4; i += blockDim.x) dst[i] = __ldg(src + i);
}

// Counts of the source blocks and their prefix (thread 0 of every unpack block computes them).
__device__ __forceinline__ void block_counts(const float* recv, int world, int cap, int row, int* cnt, int* pre,
                                             int* total) {
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int q = 0; q < world; q++) {
            int c = __float_as_int(recv[(size_t)q * cap * row + 1]);
            c = c < 0 ? 0 : c > cap ? cap : c;
            cnt[q] = c;
            pre[q] = acc;
            acc += c;
        }
        *total = acc;
    }
    __syncthreads();
}

// One block: the order of the received rows. Every position's key is (local expert, position) for a valid
// row and a value above all of them otherwise; a bitonic sort of the keys in shared memory gives the
// compact order, valid rows first by ascending expert and, within an expert, by (src, i). Rows of one
// expert then sit together, so the expert kernels, which take their rows in 64-row chunks, read each
// expert's weights about once instead of once per chunk it appears in.
constexpr int ORDER_MAX = 4096;  // positions (world * cap) the sort takes; more use the (src, i) order
constexpr int ORDER_NT = 1024;
__global__ void __launch_bounds__(ORDER_NT) k_ep_order(const float* __restrict__ recv, int D, int world, int cap,
                                                       int* __restrict__ eid, int* __restrict__ src_of) {
    __shared__ int cnt[EP_MAX_WORLD], pre[EP_MAX_WORLD], total;
    __shared__ uint32_t key[ORDER_MAX];
    const int R = world * cap, row = D + EAHMMF_EP_HDR, tid = threadIdx.x;
    block_counts(recv, world, cap, row, cnt, pre, &total);
    int n2 = 1;
    while (n2 < R) n2 <<= 1;
    for (int b = tid; b < n2; b += ORDER_NT) {
        uint32_t k = 0xffffffffu;  // padding
        if (b < R) {
            const int src = b / cap, i = b - src * cap;
            if (i < cnt[src]) {
                const int e = __float_as_int(recv[(size_t)b * row]);
                k = ((uint32_t)min(max(e, 0), 0x7ffe) << 16) | (uint32_t)b;  // out-of-range ids: after the others
            } else {
                k = (0x7fffu << 16) | (uint32_t)b;
            }
        }
        key[b] = k;
    }
    __syncthreads();
    for (int size = 2; size <= n2; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < n2; i += ORDER_NT) {
                const int p = i ^ stride;
                if (p > i) {
                    const uint32_t a = key[i], c = key[p];
                    if ((a > c) == ((i & size) == 0)) {
                        key[i] = c;
                        key[p] = a;
                    }
                }
            }
            __syncthreads();
        }
    for (int j = tid; j < R; j += ORDER_NT) {
        const uint32_t k = key[j];
        const int b = (int)(k & 0xffffu);
        const bool valid = (k >> 16) != 0x7fffu;
        eid[j] = valid ? __float_as_int(recv[(size_t)b * row]) : -1;
        src_of[j] = valid ? b : -1;
    }
}
// One block per compact row j (after k_ep_order): the received row src_of[j], or zeros.
__global__ void __launch_bounds__(256) k_ep_fill(const float* __restrict__ recv, int D, const int* __restrict__ src_of,
                                                 float* __restrict__ rows, float* __restrict__ y) {
    const int j = blockIdx.x, b = src_of[j], row = D + EAHMMF_EP_HDR;
    float4* dst = reinterpret_cast<float4*>(rows + (size_t)j * D);
    if (b >= 0) {
        const float4* s4 = reinterpret_cast<const float4*>(recv + (size_t)b * row + EAHMMF_EP_HDR);
        for (int c = threadIdx.x; c < D / 4; c += blockDim.x) dst[c] = s4[c];
    } else {
        for (int c = threadIdx.x; c < D / 4; c += blockDim.x) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (y) {
        float4* y4 = reinterpret_cast<float4*>(y + (size_t)j * D);
        for (int c = threadIdx.x; c < D / 4; c += blockDim.x) y4[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// More positions than the sort takes: one block per received row position (src, i): valid rows are
// compacted in (src, i) order to the front
// of rows / eid / src_of; the other positions become zero rows with expert -1 at the back. y (optional)
// is zeroed for the expert application that adds into it.
__global__ void __launch_bounds__(256) k_ep_unpack(const float* __restrict__ recv, int D, int world, int cap,
                                                   float* __restrict__ rows, int* __restrict__ eid,
                                                   int* __restrict__ src_of, float* __restrict__ y) {
    __shared__ int cnt[EP_MAX_WORLD], pre[EP_MAX_WORLD], total;
    const int b = blockIdx.x, src = b / cap, i = b % cap, row = D + EAHMMF_EP_HDR;
    block_counts(recv, world, cap, row, cnt, pre, &total);
    const bool valid = i < cnt[src];
    // invalid positions: after the valid rows, in (src, i) order (src * cap - pre[src] invalid rows
    // precede block src)
    const int j = valid ? pre[src] + i : total + (src * cap - pre[src]) + (i - cnt[src]);
    float4* dst = reinterpret_cast<float4*>(rows + (size_t)j * D);
    if (valid) {
        const float4* s4 = reinterpret_cast<const float4*>(recv + (size_t)b * row + EAHMMF_EP_HDR);
        for (int c = threadIdx.x; c < D / 4; c += blockDim.x) dst[c] = s4[c];
    } else {
        for (int c = threadIdx.x; c < D / 4; c += blockDim.x) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (y) {
        float4* y4 = reinterpret_cast<float4*>(y + (size_t)j * D);
        for (int c = threadIdx.x; c < D / 4; c += blockDim.x) y4[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (threadIdx.x == 0) {
        eid[j] = valid ? __float_as_int(recv[(size_t)b * row]) : -1;
        src_of[j] = valid ? b : -1;
    }
}

// One block per compact row: valid rows' outputs back to the position they came from.
__global__ void __launch_bounds__(256) k_ep_return(const float* __restrict__ y, const int* __restrict__ src_of, int D,
                                                   float* __restrict__ ret) {
    const int j = blockIdx.x;
    const int b = src_of[j];
    if (b < 0) return;
    const float4* s4 = reinterpret_cast<const float4*>(y + (size_t)j * D);
    float4* d4 = reinterpret_cast<float4*>(ret + (size_t)b * D);
    for (int c = threadIdx.x; c < D / 4; c += blockDim.x) d4[c] = s4[c];
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace eb

using namespace eb;

extern "C" int eahmmf_cuda_ep_pack(const int* d_ids, const float* d_w, const float* d_xn, int T, int K, int D,
                                   int E_loc, int world, int cap, float* d_send, int* d_token_pos, float* d_pos_w,
                                   void* stream, int* d_status) {
    if (!d_send || !d_token_pos || !d_pos_w || T < 0 || (T > 0 && (!d_ids || !d_w || !d_xn || !al16(d_xn))) ||
        K < 1 || K > 32 || D < 4 || D % 4 || E_loc < 1 || world < 1 || world > EP_MAX_WORLD || cap < 1 ||
        !al16(d_send))
        return ST_BAD_ARG;
    if ((long long)T * K > cap) return ST_CAPACITY;  // a block could overflow
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    k_ep_plan<<<1, PLAN_NT, 0, st>>>(d_ids, d_w, T, K, D, E_loc, world, cap, d_send, d_token_pos, d_pos_w, d_status);
    if (T > 0) k_ep_gather<<<T * K, 256, 0, st>>>(d_xn, K, D, d_token_pos, d_send);
    return cudaGetLastError() == cudaSuccess ? ST_OK : ST_CUDA;
}

extern "C" int eahmmf_cuda_ep_unpack(const float* d_recv, int D, int world, int cap, float* d_rows, int* d_eid,
                                     int* d_src, float* d_y, void* stream) {
    if (!d_recv || !d_rows || !d_eid || !d_src || D < 4 || D % 4 || world < 1 || world > EP_MAX_WORLD || cap < 1 ||
        !al16(d_recv) || !al16(d_rows) || (d_y && !al16(d_y)))
        return ST_BAD_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (world * cap <= ORDER_MAX) {
        k_ep_order<<<1, ORDER_NT, 0, st>>>(d_recv, D, world, cap, d_eid, d_src);
        k_ep_fill<<<world * cap, 256, 0, st>>>(d_recv, D, d_src, d_rows, d_y);
    } else {
        k_ep_unpack<<<world * cap, 256, 0, st>>>(d_recv, D, world, cap, d_rows, d_eid, d_src, d_y);
    }
    return cudaGetLastError() == cudaSuccess ? ST_OK : ST_CUDA;
}

extern "C" int eahmmf_cuda_ep_return(const float* d_y, const int* d_src, int D, int world, int cap, float* d_ret,
                                     void* stream) {
    if (!d_y || !d_src || !d_ret || D < 4 || D % 4 || world < 1 || world > EP_MAX_WORLD || cap < 1 || !al16(d_y) ||
        !al16(d_ret))
        return ST_BAD_ARG;
    k_ep_return<<<world * cap, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(d_y, d_src, D, d_ret);
    return cudaGetLastError() == cudaSuccess ? ST_OK : ST_CUDA;
}
