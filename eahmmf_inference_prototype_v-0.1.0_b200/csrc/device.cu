// device.cu -- device backend behind eahmmf::B200Device (include/eahmmf_b200_device.hpp), group 3 of
// include/eahmmf_b200.h.
//
// The reference's CudaDevice (eahmmf.h:153-197) copies from pageable host memory on a blocking stream,
// so each cudaMemcpyAsync degenerates into a staged synchronous copy. Here host->device copies from
// pageable memory go through two pinned staging halves on a non-blocking side stream: while the DMA
// engine drains one half, the CPU fills the other; an event per half guards reuse. Sources that are
// already pinned are copied directly. Results are valid for kernels only after sync(), the same
// contract the store relies on (eahmmf.h:95, :1012).
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/eahmmf_b200.h"

struct EahmmfDev {
    int device = 0;
    cudaStream_t st = nullptr;
    uint8_t* stage[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool ev_live[2] = {false, false};
    size_t half = 0;
    int cur = 0;
    size_t total = 0;
    int fail[3] = {0, 0, 0};
    std::mutex mu;
};

namespace {
bool take(int& n) {
    if (n > 0) {
        n--;
        return true;
    }
    return false;
}
bool is_pinned(const void* p) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeHost;
}
}  // namespace

extern "C" EahmmfDev* eahmmf_dev_create(size_t staging_bytes) {
    EahmmfDev* d = new EahmmfDev();
    cudaGetDevice(&d->device);
    if (staging_bytes < (1u << 20)) staging_bytes = 1u << 20;
    d->half = (staging_bytes / 2 + 4095) & ~(size_t)4095;
    bool ok = cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking) == cudaSuccess;
    for (int i = 0; ok && i < 2; i++) {
        ok = cudaHostAlloc((void**)&d->stage[i], d->half, cudaHostAllocDefault) == cudaSuccess &&
             cudaEventCreateWithFlags(&d->ev[i], cudaEventDisableTiming) == cudaSuccess;
    }
    size_t fr = 0, tot = 0;
    if (ok) ok = cudaMemGetInfo(&fr, &tot) == cudaSuccess;
    d->total = fr;  // like the reference: capacity = free memory when the backend is created
    if (!ok) {
        eahmmf_dev_destroy(d);
        return nullptr;
    }
    return d;
}

extern "C" void eahmmf_dev_destroy(EahmmfDev* d) {
    if (!d) return;
    if (d->st) cudaStreamSynchronize(d->st);
    for (int i = 0; i < 2; i++) {
        if (d->ev[i]) cudaEventDestroy(d->ev[i]);
        if (d->stage[i]) cudaFreeHost(d->stage[i]);
    }
    if (d->st) cudaStreamDestroy(d->st);
    delete d;
}

extern "C" void* eahmmf_dev_alloc(EahmmfDev* d, size_t bytes) {
    std::lock_guard<std::mutex> g(d->mu);
    if (take(d->fail[0])) return nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

extern "C" void eahmmf_dev_release(EahmmfDev* d, void* p, size_t) {
    if (!p) return;
    std::lock_guard<std::mutex> g(d->mu);
    cudaStreamSynchronize(d->st);  // no staged copy may still target p
    cudaFree(p);
}

extern "C" bool eahmmf_dev_h2d(EahmmfDev* d, void* dst, const void* src, size_t n) {
    std::lock_guard<std::mutex> g(d->mu);
    if (take(d->fail[1])) return false;
    if (n == 0) return true;
    if (is_pinned(src)) return cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, d->st) == cudaSuccess;
    const uint8_t* s = static_cast<const uint8_t*>(src);
    uint8_t* o = static_cast<uint8_t*>(dst);
    for (size_t done = 0; done < n;) {
        const size_t c = n - done < d->half ? n - done : d->half;
        const int h = d->cur;
        if (d->ev_live[h] && cudaEventSynchronize(d->ev[h]) != cudaSuccess) return false;
        memcpy(d->stage[h], s + done, c);
        if (cudaMemcpyAsync(o + done, d->stage[h], c, cudaMemcpyHostToDevice, d->st) != cudaSuccess) return false;
        if (cudaEventRecord(d->ev[h], d->st) != cudaSuccess) return false;
        d->ev_live[h] = true;
        d->cur ^= 1;
        done += c;
    }
    return true;
}

extern "C" bool eahmmf_dev_d2h(EahmmfDev* d, void* dst, const void* src, size_t n) {
    std::lock_guard<std::mutex> g(d->mu);
    if (take(d->fail[2])) return false;
    return cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, d->st) == cudaSuccess &&
           cudaStreamSynchronize(d->st) == cudaSuccess;
}

extern "C" bool eahmmf_dev_sync(EahmmfDev* d) {
    std::lock_guard<std::mutex> g(d->mu);
    return cudaStreamSynchronize(d->st) == cudaSuccess;
}

extern "C" size_t eahmmf_dev_total_memory(EahmmfDev* d) { return d->total; }

extern "C" size_t eahmmf_dev_free_memory(EahmmfDev* d) {
    size_t fr = 0, tot = 0;
    return cudaMemGetInfo(&fr, &tot) == cudaSuccess ? fr : 0;
}

extern "C" void* eahmmf_dev_stream(EahmmfDev* d) { return d->st; }

extern "C" void eahmmf_dev_inject_fault(EahmmfDev* d, int kind, int n) {
    std::lock_guard<std::mutex> g(d->mu);
    if (kind >= 0 && kind < 3) d->fail[kind] = n;
}
