// eahmmf_b200_device.hpp -- C++ adapters that plug libeahmmf_b200 into the reference engine's own types.
//
// Include after the engine's eahmmf.h (it needs eahmmf::DeviceBackend, ExpertStore, ExpertLease and
// WeightView) and link libeahmmf_b200.so. Header-only; everything below calls the C ABI of
// eahmmf_b200.h, so no CUDA headers are needed here.
//
//   eahmmf::B200Device   replaces eahmmf::CudaDevice (eahmmf.h:153-197). Same DeviceBackend contract
//                        (eahmmf.h:88-100): alloc returns nullptr on failure, h2d is enqueued and valid
//                        for kernels after sync(), d2h is complete on return, cpu_readable() is false,
//                        total_memory() is the free memory when the backend is created. Differences:
//                        copies run on a non-blocking side stream, and pageable sources are staged
//                        through two pinned halves so the copy is DMA rather than a synchronous
//                        staged copy.
//   eahmmf::B200LayerTable
//                        long-lived leases on every expert of one layer and the device pointer tables
//                        eahmmf_cuda_moe_layer consumes (gate/up/down WeightView.dev, eahmmf.h:737-742).
//                        Built once the layer is VRAM-resident; the leases keep the bytes in place.
#ifndef EAHMMF_B200_DEVICE_HPP
#define EAHMMF_B200_DEVICE_HPP

#include <cstdint>
#include <vector>

#include "eahmmf_b200.h"

namespace eahmmf {

struct B200Device : DeviceBackend {
    EahmmfDev* d = nullptr;
    explicit B200Device(size_t staging_bytes = size_t(64) << 20) : d(eahmmf_dev_create(staging_bytes)) {}
    ~B200Device() override { eahmmf_dev_destroy(d); }
    B200Device(const B200Device&) = delete;
    B200Device& operator=(const B200Device&) = delete;

    bool ok() const { return d != nullptr; }
    const char* name() const override { return "cuda"; }  // the name the engine logs and tests expect
    void* alloc(size_t n) override { return d ? eahmmf_dev_alloc(d, n) : nullptr; }
    void release(void* p, size_t n) override {
        if (d) eahmmf_dev_release(d, p, n);
    }
    bool h2d(void* dst, const void* src, size_t n) override { return d && eahmmf_dev_h2d(d, dst, src, n); }
    bool d2h(void* dst, const void* src, size_t n) override { return d && eahmmf_dev_d2h(d, dst, src, n); }
    bool sync() override { return d && eahmmf_dev_sync(d); }
    bool cpu_readable() const override { return false; }
    size_t total_memory() const override { return d ? eahmmf_dev_total_memory(d) : 0; }
    size_t free_memory() const override { return d ? eahmmf_dev_free_memory(d) : 0; }
    void* stream() const { return d ? eahmmf_dev_stream(d) : nullptr; }  // cudaStream_t
};

// The expert table of one layer for eahmmf_cuda_moe_layer. build() acquires a lease on every expert
// (the store must serve them from VRAM: WeightView.dev set for all three components) and uploads three
// device arrays of per-expert component pointers through the backend. Returns false, holding nothing,
// if any expert is not VRAM-resident or an upload fails; the engine then keeps its per-expert path.
struct B200LayerTable {
    std::vector<ExpertLease> leases;
    EahmmfMoeLayer desc{};
    DeviceBackend* dev = nullptr;
    void* tables = nullptr;
    size_t table_bytes = 0;

    bool build(ExpertStore& store, DeviceBackend& backend, int layer, int n_expert, int n_used,
               const float* d_router /* F32 [E x D] on the device, or nullptr */) {
        clear();
        std::vector<uint64_t> ptr(3 * (size_t)n_expert);
        for (int e = 0; e < n_expert; e++) {
            ExpertLease l = store.acquire_lease(layer, e);
            if (!l) return clear(), false;
            const ExpertViews& v = l.views();
            const WeightView* c[3] = {&v.gate, &v.up, &v.down};
            for (int k = 0; k < 3; k++) {
                if (!c[k]->dev) return clear(), false;
                ptr[(size_t)k * n_expert + e] = reinterpret_cast<uint64_t>(c[k]->dev);
            }
            if (e == 0) {
                desc.n_expert = n_expert;
                desc.n_used = n_used;
                desc.D = (int)v.gate.ne0;
                desc.FF = (int)v.gate.ne1;
                desc.gate_type = (int)v.gate.type;
                desc.up_type = (int)v.up.type;
                desc.down_type = (int)v.down.type;
                desc.gate_row_bytes = v.gate.row_bytes;
                desc.up_row_bytes = v.up.row_bytes;
                desc.down_row_bytes = v.down.row_bytes;
            }
            leases.push_back(std::move(l));
        }
        table_bytes = ptr.size() * sizeof(uint64_t);
        tables = backend.alloc(table_bytes);
        if (!tables || !backend.h2d(tables, ptr.data(), table_bytes) || !backend.sync()) {
            if (tables) backend.release(tables, table_bytes);
            tables = nullptr;
            return clear(), false;
        }
        dev = &backend;
        const uint8_t* const* t = static_cast<const uint8_t* const*>(tables);
        desc.d_gate = t;
        desc.d_up = t + n_expert;
        desc.d_down = t + 2 * (size_t)n_expert;
        desc.d_router = d_router;
        return true;
    }
    void clear() {
        if (tables && dev) dev->release(tables, table_bytes);
        tables = nullptr;
        dev = nullptr;
        leases.clear();  // releases the pins (ExpertLease destructor)
        desc = EahmmfMoeLayer{};
    }
    ~B200LayerTable() { clear(); }
};

}  // namespace eahmmf

#endif
