// oracle/b200_store_check.cpp -- TEST INFRASTRUCTURE: the reference engine with eahmmf::B200Device.
//
// Built by oracle/Makefile (target `storecheck`) from the reference engine compiled unmodified (through
// ref_harness.cpp) plus include/eahmmf_b200_device.hpp, linked against libeahmmf_b200.so. It checks the
// two C++ adapters against the engine's own types on a GPU:
//   1. The engine's ExpertStore runs on B200Device (exec tier VRAM, --verify checksums, gpu_compute),
//      the expert bytes read back through the backend equal the GGUF source, and the engine's decode
//      (every expert matmul through eahmmf_cuda_matmul_pair) prints logits and greedy ids.
//   2. B200LayerTable builds each layer's device pointer tables from leases, and
//      eahmmf_cuda_moe_layer on those tables matches the reference MoE block (moe_block, the restatement
//      of qwen3moe.cpp:1008-1069 around the reference matmul) on seeded inputs.
//
// Usage: b200_store_check <model.gguf> <comma-separated prompt ids> <n_gen> <T>
// Prints `key value...` lines; tests/test_gpu_store.py parses them.
#include "ref_harness.cpp"

#include <cuda_runtime.h>

#include <random>
#include <sstream>

#include "../include/eahmmf_b200_device.hpp"

namespace {

double rel_l2(const std::vector<float>& a, const std::vector<float>& b) {
    double n = 0, d = 0;
    for (size_t i = 0; i < a.size(); i++) {
        n += ((double)a[i] - b[i]) * ((double)a[i] - b[i]);
        d += (double)b[i] * b[i];
    }
    return std::sqrt(n / std::max(d, 1e-30));
}

// Host address of expert e's component c inside the mapped GGUF (experts are stacked along ne2).
const uint8_t* host_component(Engine& E, int l, int c, int e) {
    const Tensor* t = c == 0 ? E.layers[l].gate : c == 1 ? E.layers[l].up : E.layers[l].down;
    return E.g.map + t->file_off + (size_t)e * t->row_bytes * (size_t)t->ne[1];
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: %s model.gguf ids n_gen T\n", argv[0]);
        return 2;
    }
    std::vector<int> prompt;
    {
        std::stringstream ss(argv[2]);
        std::string tok;
        while (std::getline(ss, tok, ',')) prompt.push_back(atoi(tok.c_str()));
    }
    const int n_gen = atoi(argv[3]), T = atoi(argv[4]);
    eref_init(4);
    Engine E;
    E.load(argv[1], 256, false);

    auto* dev = new eahmmf::B200Device();
    if (!dev->ok()) {
        printf("backend_create 0\n");
        return 1;
    }
    printf("backend_name %s\nn_expert %d\n", dev->name(), E.n_expert);
    eahmmf::Config cfg;
    cfg.exec_tier = eahmmf::Residency::VRAM;
    cfg.verify = true;  // every migration checksummed against the GGUF source through d2h
    cfg.gpu_compute = true;
    cfg.log_acquires = false;
    if (!E.init_experts(cfg, std::unique_ptr<eahmmf::DeviceBackend>(dev))) return 1;
#ifdef EAHMMF_CUDA_COMPUTE
    g_cuda_compute = 1;
#endif

    // 1. decode through the store (the engine acquires each routed expert from VRAM)
    std::vector<int> out(n_gen);
    std::vector<float> first(E.n_vocab);
    if (eref_engine_greedy(&E, prompt.data(), (int)prompt.size(), n_gen, 32, out.data(), first.data())) return 1;
    printf("logits");
    for (int i = 0; i < E.n_vocab; i++) printf(" %.9g", first[i]);
    printf("\ngreedy");
    for (int t : out) printf(" %d", t);
    printf("\nstore_pinned_after_decode %llu\n", (unsigned long long)E.store->stats().pinned_now);

    // 2. layer tables from leases, the MoE layer on the device against the reference block
    std::mt19937 rng(1234);
    std::normal_distribution<float> nd(0.f, 1.f);
    int all_ok = 1;
    for (int l = 0; l < E.n_layer; l++) {
        eahmmf::B200LayerTable tab;
        const bool built = tab.build(*E.store, *E.dev, l, E.n_expert, E.n_used, nullptr);
        printf("layer %d table %d pinned %llu\n", l, (int)built, (unsigned long long)E.store->stats().pinned_now);
        if (!built) {
            all_ok = 0;
            continue;
        }
        // device copies equal the source bytes (read back through the backend)
        int bytes_equal = 1;
        for (int e = 0; e < E.n_expert; e++) {
            const eahmmf::ExpertViews& v = tab.leases[e].views();
            const eahmmf::WeightView* c[3] = {&v.gate, &v.up, &v.down};
            for (int k = 0; k < 3; k++) {
                std::vector<uint8_t> h(c[k]->bytes);
                if (!E.dev->d2h(h.data(), c[k]->dev, h.size()) ||
                    memcmp(h.data(), host_component(E, l, k, e), h.size()) != 0)
                    bytes_equal = 0;
            }
        }
        std::vector<float> xn((size_t)T * E.D), lg((size_t)T * E.n_expert), x0((size_t)T * E.D);
        for (auto& v : xn) v = nd(rng);
        for (auto& v : lg) v = nd(rng);
        for (auto& v : x0) v = nd(rng);
        std::vector<float> want = x0, got((size_t)T * E.D);
        std::vector<const uint8_t*> hg(E.n_expert), hu(E.n_expert), hd(E.n_expert);
        for (int e = 0; e < E.n_expert; e++) {
            hg[e] = host_component(E, l, 0, e);
            hu[e] = host_component(E, l, 1, e);
            hd[e] = host_component(E, l, 2, e);
        }
        const EahmmfMoeLayer& L = tab.desc;
        std::vector<int> want_ids((size_t)T * E.n_used);
        eref_moe_layer(T, E.D, E.FF, E.n_expert, E.n_used, xn.data(), lg.data(), nullptr, hg.data(), hu.data(),
                       hd.data(), L.gate_type, L.up_type, L.down_type, L.gate_row_bytes, L.up_row_bytes,
                       L.down_row_bytes, want.data(), want_ids.data(), nullptr);
        float *d_xn = nullptr, *d_lg = nullptr, *d_x = nullptr;
        void* d_ws = nullptr;
        const size_t wsb = eahmmf_cuda_moe_workspace_bytes(&L, T);
        int st = -1;
        if (cudaMalloc(&d_xn, xn.size() * 4) == cudaSuccess && cudaMalloc(&d_lg, lg.size() * 4) == cudaSuccess &&
            cudaMalloc(&d_x, x0.size() * 4) == cudaSuccess && cudaMalloc(&d_ws, wsb) == cudaSuccess &&
            cudaMemcpy(d_xn, xn.data(), xn.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
            cudaMemcpy(d_lg, lg.data(), lg.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
            cudaMemcpy(d_x, x0.data(), x0.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess) {
            st = eahmmf_cuda_moe_layer(&L, T, d_xn, d_lg, d_x, d_ws, wsb, nullptr, nullptr);
            if (cudaMemcpy(got.data(), d_x, got.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) st = -2;
        }
        std::vector<int> got_ids((size_t)T * E.n_used);
        if (st == 0 && cudaMemcpy(got_ids.data(), d_ws, got_ids.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
            st = -3;
        cudaFree(d_xn);
        cudaFree(d_lg);
        cudaFree(d_x);
        cudaFree(d_ws);
        // contribution of the layer (x - x0) against the reference's
        std::vector<float> dg(got.size()), dw(want.size());
        for (size_t i = 0; i < got.size(); i++) {
            dg[i] = got[i] - x0[i];
            dw[i] = want[i] - x0[i];
        }
        printf("layer %d bytes_equal %d status %d ids_equal %d rel_l2 %.3e\n", l, bytes_equal, st,
               (int)(got_ids == want_ids), rel_l2(dg, dw));
        tab.clear();
        printf("layer %d released pinned %llu\n", l, (unsigned long long)E.store->stats().pinned_now);
    }
    printf("done %d\n", all_ok);
    return 0;
}
