// engine.cu -- a device-resident qwen3moe forward pass (group 4 of include/eahmmf_b200.h): the whole
// model of a GGUF file in HBM, Engine::forward / eval / greedy generation (qwen3moe.cpp:929-1084, the
// harness-level greedy loop with --temp 0 --repeat-penalty 1.0) with every step on the GPU.
//
// Per layer and forward pass (nb tokens): RMSNorm -> fused q|k|v GEMV (one K-quant matrix, rows of
// q, k and v concatenated at load) -> per-head RMSNorm + NeoX RoPE + KV append -> split-context GQA
// attention -> o-projection GEMV accumulated into the residual -> RMSNorm -> MoE block
// (eahmmf_cuda_moe_layer: router GEMV, top-k, grouping, gate/up/SiLU, down, combine). After the last
// layer: RMSNorm of the last row -> output GEMV -> first-maximum argmax, which writes the next token and
// advances the position on the device. One decode step is captured once as a CUDA graph and replayed
// per token; nothing returns to the host between tokens.
//
// Numerics follow the reference's fp32 formulas (RMSNorm 1/sqrtf(mean + eps), RoPE angles in double
// rounded to float, softmax attention with 1/sqrt(hd) scaling); summation orders differ (tree and
// tensor-core reductions), so logits agree to fp32 rounding and greedy tokens agree exactly unless two
// logits tie within that rounding.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/eahmmf_b200.h"
#include "common.cuh"
#include "decode.cuh"
#include "kernels.cuh"
#include "sample.cuh"

namespace eb {
int moe_layer_run(const EahmmfMoeLayer* L, int T, const float* d_xn, const float* d_logits, float* d_x,
                  void* d_workspace, size_t workspace_bytes, void* stream, int* d_status, MoeDeferred* defer,
                  const float* norm_w, float eps, const MoeHook* hook = nullptr);
cudaError_t launch_hash64(const uint8_t* const* d_ptrs, const size_t* d_sizes, int n, uint64_t* d_out,
                          cudaStream_t st);
uint64_t host_hash64(const uint8_t* p, size_t n);
}
using namespace eb;

namespace {

// ---- GGUF v2/v3 reader (the container layout GGUF::load parses, qwen3moe.cpp:285-347) -------------
struct GgufValue {
    uint32_t type = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
};
struct GgufTensor {
    int nd = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    int type = -1;
    uint64_t off = 0;
    size_t row_bytes = 0, bytes = 0;
    uint64_t file_off = 0;
};
struct Gguf {
    const uint8_t* map = nullptr;
    size_t size = 0;
    uint64_t data_start = 0;
    std::map<std::string, GgufValue> kv;
    std::map<std::string, GgufTensor> tensors;
    std::string err;

    ~Gguf() {
        if (map) munmap(const_cast<uint8_t*>(map), size);
    }
    struct Rd {
        const uint8_t *p, *end;
        bool ok = true;
        bool need(size_t n) {
            if (!ok || (size_t)(end - p) < n) ok = false;
            return ok;
        }
        template <typename V>
        V get() {
            V v{};
            if (need(sizeof(V))) {
                memcpy(&v, p, sizeof(V));
                p += sizeof(V);
            }
            return v;
        }
        std::string str() {
            const uint64_t n = get<uint64_t>();
            if (!need(n)) return std::string();
            std::string s(reinterpret_cast<const char*>(p), (size_t)n);
            p += n;
            return s;
        }
    };
    static bool scalar(Rd& r, uint32_t t, GgufValue& v) {
        v.type = t;
        switch (t) {
            case 0: v.i = r.get<uint8_t>(); break;
            case 1: v.i = r.get<int8_t>(); break;
            case 2: v.i = r.get<uint16_t>(); break;
            case 3: v.i = r.get<int16_t>(); break;
            case 4: v.i = r.get<uint32_t>(); break;
            case 5: v.i = r.get<int32_t>(); break;
            case 6: v.f = r.get<float>(); v.i = (int64_t)v.f; break;
            case 7: v.i = r.get<uint8_t>(); break;
            case 8: v.s = r.str(); break;
            case 10: v.i = (int64_t)r.get<uint64_t>(); break;
            case 11: v.i = r.get<int64_t>(); break;
            case 12: v.f = r.get<double>(); v.i = (int64_t)v.f; break;
            default: return false;
        }
        if (t != 6 && t != 12) v.f = (double)v.i;
        return r.ok;
    }
    bool open(const char* path) {
        const int fd = ::open(path, O_RDONLY);
        if (fd < 0) return fail("cannot open file");
        struct stat st;
        if (fstat(fd, &st) != 0) {
            ::close(fd);
            return fail("cannot stat file");
        }
        size = (size_t)st.st_size;
        void* m = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
        ::close(fd);
        if (m == MAP_FAILED) {
            map = nullptr;
            return fail("mmap failed");
        }
        map = static_cast<const uint8_t*>(m);
        Rd r{map, map + size};
        if (size < 4 || memcmp(map, "GGUF", 4) != 0) return fail("not a GGUF file");
        r.p += 4;
        const uint32_t ver = r.get<uint32_t>();
        if (ver < 2 || ver > 3) return fail("unsupported GGUF version");
        const uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
        for (uint64_t i = 0; i < nkv && r.ok; i++) {
            const std::string key = r.str();
            const uint32_t t = r.get<uint32_t>();
            GgufValue v;
            if (t == 9) {  // array: skipped except for its length (tokenizer tables are not needed here)
                const uint32_t et = r.get<uint32_t>();
                const uint64_t n = r.get<uint64_t>();
                if (et == 9) return fail("nested arrays unsupported");
                for (uint64_t k = 0; k < n && r.ok; k++) {
                    GgufValue e;
                    if (!scalar(r, et, e)) return fail("bad array element");
                }
                v.type = 9;
                v.i = (int64_t)n;
            } else if (!scalar(r, t, v)) {
                return fail("bad metadata value");
            }
            kv[key] = v;
        }
        std::vector<std::pair<std::string, GgufTensor>> ts;
        for (uint64_t i = 0; i < nt && r.ok; i++) {
            GgufTensor t;
            const std::string name = r.str();
            t.nd = (int)r.get<uint32_t>();
            if (t.nd < 1 || t.nd > 4) return fail("bad tensor dims");
            for (int d = 0; d < t.nd; d++) t.ne[d] = (int64_t)r.get<uint64_t>();
            t.type = (int)r.get<uint32_t>();
            t.off = r.get<uint64_t>();
            ts.emplace_back(name, t);
        }
        if (!r.ok) return fail("truncated header");
        uint64_t align = 32;
        auto it = kv.find("general.alignment");
        if (it != kv.end() && it->second.i > 0) align = (uint64_t)it->second.i;
        const uint64_t pos = (uint64_t)(r.p - map);
        data_start = (pos + align - 1) / align * align;
        for (auto& nt_ : ts) {
            GgufTensor& t = nt_.second;
            if (!type_supported(t.type)) return fail("unsupported tensor type");
            if (t.ne[0] % block_elems(t.type)) return fail("row length not a whole number of blocks");
            t.row_bytes = (size_t)(t.ne[0] / block_elems(t.type)) * block_bytes(t.type);
            t.bytes = t.row_bytes * (size_t)(t.ne[1] * t.ne[2] * t.ne[3]);
            t.file_off = data_start + t.off;
            if (t.file_off + t.bytes > size) return fail("tensor out of file bounds");
            tensors[nt_.first] = t;
        }
        return true;
    }
    bool fail(const char* m) {
        err = m;
        return false;
    }
    const GgufTensor* tensor(const std::string& n) const {
        auto it = tensors.find(n);
        return it == tensors.end() ? nullptr : &it->second;
    }
    int64_t geti(const std::string& k, int64_t def, bool* missing = nullptr) const {
        auto it = kv.find(k);
        if (it == kv.end()) {
            if (missing) *missing = true;
            return def;
        }
        return it->second.i;
    }
    double getf(const std::string& k, double def) const {
        auto it = kv.find(k);
        return it == kv.end() ? def : it->second.f;
    }
    std::string gets(const std::string& k) const {
        auto it = kv.find(k);
        return it == kv.end() ? std::string() : it->second.s;
    }
};

float host_f16(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t b;
    if (e == 0) {
        if (m == 0) {
            b = s;
        } else {  // subnormal: renormalise
            int ee = -1;
            uint32_t mm = m;
            do {
                ee++;
                mm <<= 1;
            } while (!(mm & 1024));
            b = s | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 1023) << 13);
        }
    } else if (e == 31) {
        b = s | 0x7f800000u | (m << 13);
    } else {
        b = s | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &b, 4);
    return f;
}

constexpr int MAXB = 64;  // tokens per forward pass (qwen3moe.cpp:39)

}  // namespace

struct EahmmfEngine {
    int n_layer = 0, D = 0, n_head = 0, n_kv = 0, hd = 0, QD = 0, KD = 0, n_expert = 0, n_used = 0, FF = 0,
        n_vocab = 0, n_ctx = 0, n_embd_rows = 0;
    float eps = 1e-6f, rope_base = 1e6f;
    cudaStream_t st = nullptr;
    uint8_t* weights = nullptr;  // the GGUF data section, as in the file
    struct Layer {
        float *attn_norm, *ffn_norm, *q_norm, *k_norm;
        const uint8_t* wq[3];  // q, k, v (or the fused q|k|v matrix in wq[0] when fused)
        int qkv_type[3];
        size_t qkv_rb[3];
        bool fused;
        const uint8_t* wo;
        int wo_type;
        size_t wo_rb;
        EahmmfMoeLayer moe;
    };
    std::vector<Layer> layers;
    // every expert component in HBM with its place in the file (the residency layer's TensorSlice)
    struct Slice {
        const uint8_t* dev;
        uint64_t file_off;
        size_t bytes;
    };
    std::vector<Slice> slices;
    std::string path;
    // Oversubscribed mode (expert_budget > 0): the experts stay in the mapped file (pinned for DMA) and a
    // device cache of `slots` expert footprints holds the resident ones (see ExpertCache).
    struct ExpertCache {
        std::unique_ptr<Gguf> file;     // the mapping the host copies come from
        bool pinned = false;            // fills are DMA copies: from the registered mapping or a pinned copy
        const uint8_t* host = nullptr;  // the bytes fills copy from (file offsets)
        uint8_t* host_copy = nullptr;   // pinned copy of the file when the mapping cannot be registered
        size_t comp[3] = {0, 0, 0};     // bytes of one expert's gate, up, down
        size_t off[3] = {0, 0, 0};      // their offsets inside a slot
        size_t foot = 0;                // slot bytes
        int slots = 0;
        uint8_t* dev = nullptr;         // [slots x foot]
        std::vector<uint64_t> src[3];   // [layer * E + expert] file offset of each component
        std::vector<int> slot_of;       // [layer * E + expert] -> slot or -1
        std::vector<int> owner;         // [slot] -> layer * E + expert or -1
        std::vector<uint64_t> last_use, pin;  // per slot: LRU tick, epoch of the pass that needs it
        std::vector<cudaEvent_t> ready; // per slot: its last fill completed
        std::vector<std::vector<int>> last_set;  // [layer] experts routed at the layer's last pass
        uint64_t tick = 0, epoch = 0;
        cudaStream_t side = nullptr;    // fills (host -> device copies)
        uint64_t* h_tab = nullptr;      // pinned mirror of every layer's 3 x E pointer table
        int* d_ids = nullptr;           // [MAXB * K] routing of the pass
        float* d_w = nullptr;
        int* h_ids = nullptr;           // pinned
        uint64_t hits = 0, misses = 0, prefetched = 0, prefetch_hits = 0, bytes = 0, evictions = 0;
        std::vector<uint8_t> from_prefetch;  // [slot] filled by a prefetch and not used since
    };
    std::unique_ptr<ExpertCache> cache;
    int cur_layer = 0;
    const uint8_t* embd = nullptr;
    int embd_type = 0;
    size_t embd_rb = 0;
    const uint8_t* out_w = nullptr;
    int out_type = 0;
    size_t out_rb = 0;
    std::vector<void*> allocs;  // every cudaMalloc of the engine (freed in the destructor)
    float *out_norm = nullptr, *inv_freq = nullptr, *kc = nullptr, *vc = nullptr;
    float *x = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr, *logits = nullptr;
    float* attn_part = nullptr;
    float2 *rope_cs = nullptr, *amax_blk = nullptr;
    int amax_nblk = 0;
    void *moe_ws = nullptr, *gemv_ws = nullptr;
    void* xf_rows = nullptr;  // [MAXB rows of D] normalised activations in fragment form
    void* xf_att = nullptr;   // [MAXB rows of QD] attention outputs in fragment form
    size_t moe_ws_bytes = 0, gemv_ws_bytes = 0;
    int* toks = nullptr;       // device token staging [MAXB]
    int pos_host = -1;         // state->pos during an eval pass (set by eval_dev), -1 otherwise
    int hpos = 0;              // host copy of state->pos after the work enqueued so far
    int* h_toks = nullptr;     // pinned [MAXB]
    int* status = nullptr;     // device status word
    int* att_cnt = nullptr;    // [n_kv] split counters of the attention launch's fused merge (self-resetting)
    DecodeState* state = nullptr;
    DecodeState* h_state = nullptr;  // pinned mirror for reads
    int* out = nullptr;
    int cap_out = 0;
    cudaGraphExec_t step_graph = nullptr;
    // token selection: the first maximum (greedy), or the reference's sampler with its random stream
    bool sampling = false;
    EahmmfSamplerParams sparams{};
    EahmmfRng* rng = nullptr;
    float* u_dev = nullptr;   // [n_ctx + 1] uniform draw of each generated index (device)
    float* u_host = nullptr;  // pinned staging of the same
    void* samp_ws = nullptr;
    int hn_out = 0;           // host copy of state->n_out after the work enqueued so far
    // multi-sequence decode: n_slots sequences, each with n_ctx cache rows per layer; single-sequence
    // passes (eval, greedy, decode) run on slot `slot_cur`, a multi-sequence step on bstate's rows
    int n_slots = 1, slot_cur = 0;
    DecodeState* bstate = nullptr;  // the multi-sequence step's state (tpos / tslot set)
    DecodeState* fst = nullptr;     // the state of the forward pass in progress
    int* d_tpos = nullptr;          // [MAXB] positions of a multi-sequence step's rows
    int* d_tslot = nullptr;         // [MAXB] their slots
    int* d_btok = nullptr;          // [MAXB] their input tokens, then their argmax
    int* h_b = nullptr;             // pinned staging [3 * MAXB]
    float* logits_b = nullptr;      // [MAXB x n_vocab] logits of every row of a multi-sequence step
    int graph_nodes = 0;
    bool trace = false;
    std::vector<int> trace_ids;
    std::vector<float> trace_w;
    std::vector<int> h_ids;
    std::vector<float> h_w;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    std::string err;
    // per-operation profile of eager decode steps
    static constexpr int NPROF = EAHMMF_ENGINE_PROFILE_CLASSES;
    bool prof = false;
    std::vector<cudaEvent_t> pev;  // pool, reused per step
    std::vector<int> pcls;         // class of the operation that ends at each recorded event
    int pn = 0;
    double psum[NPROF] = {};
    int psteps = 0;

    ~EahmmfEngine() {
        if (st) cudaStreamSynchronize(st);
        if (cache) {
            ExpertCache& C = *cache;
            if (C.side) cudaStreamSynchronize(C.side);
            for (cudaEvent_t ev : C.ready)
                if (ev) cudaEventDestroy(ev);
            if (C.side) cudaStreamDestroy(C.side);
            if (C.h_tab) cudaFreeHost(C.h_tab);
            if (C.h_ids) cudaFreeHost(C.h_ids);
            if (C.host_copy) cudaFreeHost(C.host_copy);
            else if (C.pinned && C.file) cudaHostUnregister(const_cast<uint8_t*>(C.file->map));
            cache.reset();  // unmaps the file
        }
        for (cudaEvent_t v : pev) cudaEventDestroy(v);
        if (step_graph) cudaGraphExecDestroy(step_graph);
        if (u_host) cudaFreeHost(u_host);
        if (rng) eahmmf_rng_free(rng);
        for (void* p : allocs) cudaFree(p);
        if (h_toks) cudaFreeHost(h_toks);
        if (h_b) cudaFreeHost(h_b);
        for (int i = 0; i < 2; i++) {
            if (up_stage[i]) cudaFreeHost(up_stage[i]);
            if (up_ev[i]) cudaEventDestroy(up_ev[i]);
        }
        if (h_state) cudaFreeHost(h_state);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        if (st) cudaStreamDestroy(st);
    }
    template <typename T>
    bool dalloc(T*& p, size_t bytes) {
        void* v = nullptr;
        if (cudaMalloc(&v, bytes < 256 ? 256 : bytes) != cudaSuccess) return false;
        allocs.push_back(v);
        p = static_cast<T*>(v);
        return true;
    }
    bool fail(const std::string& m) {
        err = m;
        return false;
    }

    // F32 copy of a small F32/F16 tensor (norm weights, router), converted on the host.
    bool f32_tensor(const Gguf& g, const GgufTensor* t, size_t n, float*& dst) {
        if (!t || (size_t)(t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]) != n) return false;
        std::vector<float> h(n);
        const uint8_t* src = g.map + t->file_off;
        if (t->type == T_F32) {
            memcpy(h.data(), src, n * 4);
        } else if (t->type == T_F16) {
            for (size_t i = 0; i < n; i++) h[i] = host_f16((uint16_t)(src[2 * i] | (src[2 * i + 1] << 8)));
        } else {
            return false;
        }
        return dalloc(dst, n * 4) && cudaMemcpy(dst, h.data(), n * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    }

    bool load(const char* path, int ctx, size_t expert_budget = 0) {
        std::unique_ptr<Gguf> gfile(new Gguf());
        Gguf& g = *gfile;
        if (!g.open(path)) return fail("gguf: " + g.err);
        if (g.gets("general.architecture") != "qwen3moe") return fail("unsupported architecture (need qwen3moe)");
        this->path = path;
        const std::string a = "qwen3moe.";
        bool miss = false;
        n_layer = (int)g.geti(a + "block_count", 0, &miss);
        D = (int)g.geti(a + "embedding_length", 0, &miss);
        n_head = (int)g.geti(a + "attention.head_count", 0, &miss);
        n_kv = (int)g.geti(a + "attention.head_count_kv", 0, &miss);
        n_expert = (int)g.geti(a + "expert_count", 0, &miss);
        n_used = (int)g.geti(a + "expert_used_count", 0, &miss);
        FF = (int)g.geti(a + "expert_feed_forward_length", 0, &miss);
        if (miss || n_head <= 0 || n_kv <= 0) return fail("missing hyper-parameters");
        hd = (int)g.geti(a + "attention.key_length", D / n_head);
        eps = (float)g.getf(a + "attention.layer_norm_rms_epsilon", 1e-6);
        rope_base = (float)g.getf(a + "rope.freq_base", 1e6);
        const int n_ctx_train = (int)g.geti(a + "context_length", 4096);
        QD = n_head * hd;
        KD = n_kv * hd;
        n_ctx = std::min(ctx, n_ctx_train);
        if (n_ctx < 1) return fail("bad context length");
        if (hd % 2 || n_head % n_kv) return fail("bad head config");
        if (hd != 64 && hd != 128) return fail("head size must be 64 or 128");
        if (n_head / n_kv > ATT_MAXH * (ATT_NT / 32)) return fail("GQA group too large");
        if (D % 256 || FF % 256) return fail("hidden and expert sizes must be multiples of 256");

        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return fail("stream");
        // the data section, byte for byte; in oversubscribed mode everything but the expert tensors, each
        // tensor at a 256-byte aligned place of one allocation
        const size_t nbytes = g.size - g.data_start;
        auto is_expert = [](const std::string& n) {
            return n.size() > 12 && n.compare(n.size() - 12, 12, "_exps.weight") == 0;
        };
        std::map<const GgufTensor*, size_t> place;
        if (!expert_budget) {
            if (!dalloc(weights, nbytes)) return fail("cannot allocate device memory for the weights");
            if (!upload(g.map + g.data_start, nbytes)) return fail("weight upload failed");
        } else {
            size_t o = 0;
            for (auto& kv : g.tensors)
                if (!is_expert(kv.first)) {
                    place[&kv.second] = o;
                    o = (o + kv.second.bytes + 255) & ~(size_t)255;
                }
            if (!dalloc(weights, o)) return fail("cannot allocate device memory for the weights");
            size_t left = place.size();
            for (auto& kv : place)
                if (!upload(g.map + kv.first->file_off, kv.first->bytes, weights + kv.second, --left > 0))
                    return fail("weight upload failed");
        }
        auto dptr = [&](const GgufTensor* t) {
            return expert_budget ? weights + place.at(t) : weights + (t->file_off - g.data_start);
        };

        const GgufTensor* te = g.tensor("token_embd.weight");
        const GgufTensor* to = g.tensor("output.weight");
        if (!te) return fail("token_embd.weight missing");
        if (!to) to = te;  // tied embeddings
        if (te->ne[0] != D || to->ne[0] != D) return fail("embedding width mismatch");
        embd = dptr(te);
        embd_type = te->type;
        embd_rb = te->row_bytes;
        n_embd_rows = (int)te->ne[1];
        out_w = dptr(to);
        out_type = to->type;
        out_rb = to->row_bytes;
        n_vocab = (int)to->ne[1];
        if (!f32_tensor(g, g.tensor("output_norm.weight"), D, out_norm)) return fail("output_norm.weight");
        std::vector<float> invf(hd / 2);
        for (int i = 0; i < hd / 2; i++) invf[i] = (float)pow((double)rope_base, -2.0 * i / hd);
        if (!dalloc(inv_freq, invf.size() * 4) ||
            cudaMemcpy(inv_freq, invf.data(), invf.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return fail("inv_freq");

        layers.resize(n_layer);
        if (expert_budget) cache.reset(new ExpertCache());
        for (int l = 0; l < n_layer; l++) {
            Layer& L = layers[l];
            auto T = [&](const char* s) { return g.tensor("blk." + std::to_string(l) + "." + s); };
            if (!f32_tensor(g, T("attn_norm.weight"), D, L.attn_norm) ||
                !f32_tensor(g, T("ffn_norm.weight"), D, L.ffn_norm) ||
                !f32_tensor(g, T("attn_q_norm.weight"), hd, L.q_norm) ||
                !f32_tensor(g, T("attn_k_norm.weight"), hd, L.k_norm))
                return fail("norm weights of layer " + std::to_string(l));
            const GgufTensor* tq[3] = {T("attn_q.weight"), T("attn_k.weight"), T("attn_v.weight")};
            const int rows[3] = {QD, KD, KD};
            for (int c = 0; c < 3; c++)
                if (!tq[c] || tq[c]->ne[0] != D || tq[c]->ne[1] != rows[c]) return fail("attention projection shape");
            L.fused = tq[1]->type == tq[0]->type && tq[2]->type == tq[0]->type;
            if (L.fused) {  // one matrix of QD + 2 KD rows: one activation prep and one GEMV per layer
                uint8_t* f = nullptr;
                const size_t rb = tq[0]->row_bytes;
                if (!dalloc(f, rb * (size_t)(QD + 2 * KD))) return fail("fused qkv allocation");
                size_t o = 0;
                for (int c = 0; c < 3; c++) {
                    if (cudaMemcpy(f + o, dptr(tq[c]), tq[c]->bytes, cudaMemcpyDeviceToDevice) != cudaSuccess)
                        return fail("fused qkv copy");
                    o += tq[c]->bytes;
                }
                L.wq[0] = f;
                L.qkv_type[0] = tq[0]->type;
                L.qkv_rb[0] = rb;
            } else {
                for (int c = 0; c < 3; c++) {
                    L.wq[c] = dptr(tq[c]);
                    L.qkv_type[c] = tq[c]->type;
                    L.qkv_rb[c] = tq[c]->row_bytes;
                }
            }
            const GgufTensor* wo = T("attn_output.weight");
            if (!wo || wo->ne[0] != QD || wo->ne[1] != D) return fail("attn_output shape");
            L.wo = dptr(wo);
            L.wo_type = wo->type;
            L.wo_rb = wo->row_bytes;
            float* router = nullptr;
            if (!f32_tensor(g, T("ffn_gate_inp.weight"), (size_t)n_expert * D, router)) return fail("router");
            const GgufTensor* ex[3] = {T("ffn_gate_exps.weight"), T("ffn_up_exps.weight"), T("ffn_down_exps.weight")};
            for (int c = 0; c < 3; c++)
                if (!ex[c]) return fail("expert tensors missing");
            if (ex[0]->ne[0] != D || ex[0]->ne[1] != FF || ex[0]->ne[2] != n_expert || ex[1]->ne[0] != D ||
                ex[1]->ne[1] != FF || ex[1]->ne[2] != n_expert || ex[2]->ne[0] != FF || ex[2]->ne[1] != D ||
                ex[2]->ne[2] != n_expert)
                return fail("unexpected expert tensor shape");
            // per-expert component pointers (ExpertViews.gate/up/down, eahmmf.h:737-742)
            std::vector<const uint8_t*> ptr(3 * (size_t)n_expert);
            for (int c = 0; c < 3; c++) {
                const size_t per = ex[c]->row_bytes * (size_t)ex[c]->ne[1];
                if (expert_budget) {  // the cache fills the table; the file keeps the bytes
                    if (cache->comp[c] == 0) cache->comp[c] = per;
                    if (cache->comp[c] != per) return fail("expert sizes differ between layers");
                    for (int e = 0; e < n_expert; e++) cache->src[c].push_back(ex[c]->file_off + per * e);
                    continue;
                }
                for (int e = 0; e < n_expert; e++) {
                    ptr[(size_t)c * n_expert + e] = dptr(ex[c]) + per * e;
                    slices.push_back(Slice{dptr(ex[c]) + per * e, ex[c]->file_off + per * e, per});
                }
            }
            const uint8_t** dp = nullptr;
            if (!dalloc(dp, ptr.size() * sizeof(void*)) ||
                cudaMemcpy(dp, ptr.data(), ptr.size() * sizeof(void*), cudaMemcpyHostToDevice) != cudaSuccess)
                return fail("expert tables");
            EahmmfMoeLayer& M = L.moe;
            M.n_expert = n_expert;
            M.n_used = n_used;
            M.D = D;
            M.FF = FF;
            M.gate_type = ex[0]->type;
            M.up_type = ex[1]->type;
            M.down_type = ex[2]->type;
            M.gate_row_bytes = ex[0]->row_bytes;
            M.up_row_bytes = ex[1]->row_bytes;
            M.down_row_bytes = ex[2]->row_bytes;
            M.d_gate = dp;
            M.d_up = dp + n_expert;
            M.d_down = dp + 2 * n_expert;
            M.d_router = router;
        }
        if (expert_budget && !init_cache(std::move(gfile), expert_budget)) return false;
        moe_ws_bytes = eahmmf_cuda_moe_workspace_bytes(&layers[0].moe, MAXB);
        if (!moe_ws_bytes) return fail("expert layer not supported by the MoE kernels");
        gemv_ws_bytes = eahmmf_cuda_gemv_workspace_bytes(std::max(D, QD));
        const size_t kvn = (size_t)n_layer * n_slots * n_ctx * KD;
        amax_nblk = 148;
        const int nsplit_max = std::max(1, (n_ctx + ATT_CH - 1) / ATT_CH);
        if (!dalloc(kc, kvn * 4) || !dalloc(vc, kvn * 4) || !dalloc(x, (size_t)MAXB * D * 4) ||
            !dalloc(xn, (size_t)MAXB * D * 4) || !dalloc(qkv, (size_t)MAXB * (QD + 2 * KD) * 4) ||
            !dalloc(q, (size_t)MAXB * QD * 4) || !dalloc(att, (size_t)MAXB * QD * 4) ||
            !dalloc(logits, (size_t)n_vocab * 4) || !dalloc(rope_cs, (size_t)MAXB * (hd / 2) * 8) ||
            !dalloc(attn_part, (size_t)MAXB * n_head * std::min(nsplit_max, 128) * (hd + 2) * 4) ||
            !dalloc(amax_blk, (size_t)amax_nblk * 8) || !dalloc(moe_ws, moe_ws_bytes) ||
            !dalloc(gemv_ws, gemv_ws_bytes) || !dalloc(toks, MAXB * 4) || !dalloc(status, 4) ||
            !dalloc(xf_rows, xf_bytes(MAXB, D)) || !dalloc(xf_att, xf_bytes(MAXB, QD)) || !dalloc(att_cnt, n_kv * 4) ||
            !dalloc(state, sizeof(DecodeState)) || !dalloc(bstate, sizeof(DecodeState)) || !dalloc(d_tpos, MAXB * 4) ||
            !dalloc(d_tslot, MAXB * 4) || !dalloc(d_btok, MAXB * 4) ||
            !dalloc(logits_b, (size_t)MAXB * n_vocab * 4))
            return fail("cannot allocate activations / KV cache");
        {
            DecodeState b{};
            b.slot_rows = n_ctx;
            b.tpos = d_tpos;
            b.tslot = d_tslot;
            if (cudaMemcpy(bstate, &b, sizeof b, cudaMemcpyHostToDevice) != cudaSuccess) return fail("state");
        }
        if (cudaMemset(kc, 0, kvn * 4) != cudaSuccess || cudaMemset(vc, 0, kvn * 4) != cudaSuccess ||
            cudaMemset(status, 0, 4) != cudaSuccess || cudaMemset(att_cnt, 0, n_kv * 4) != cudaSuccess)
            return fail("memset");
        if (cudaHostAlloc((void**)&h_toks, MAXB * 4, cudaHostAllocDefault) != cudaSuccess ||
            cudaHostAlloc((void**)&h_b, 3 * MAXB * 4, cudaHostAllocDefault) != cudaSuccess ||
            cudaHostAlloc((void**)&h_state, sizeof(DecodeState), cudaHostAllocDefault) != cudaSuccess ||
            cudaHostAlloc((void**)&u_host, (size_t)(n_ctx + 1) * 4, cudaHostAllocDefault) != cudaSuccess)
            return fail("pinned buffers");
        if (!dalloc(u_dev, (size_t)(n_ctx + 1) * 4) || !dalloc(samp_ws, sample_ws_bytes(n_vocab)))
            return fail("sampler buffers");
        if (cudaEventCreate(&ev0) != cudaSuccess || cudaEventCreate(&ev1) != cudaSuccess) return fail("events");
        if (!set_state(0, 0)) return fail("state");
        return cudaDeviceSynchronize() == cudaSuccess || fail("device error after load");
    }

    // ---- oversubscribed mode ------------------------------------------------------------------------
    // The cache: slots of one expert footprint each (gate, up, down at 256-byte aligned offsets), at
    // least one layer's worth; the file mapping registered with the driver so that fills are DMA copies
    // from it (pageable copies otherwise); every layer's pointer table aimed at slot 0 until its experts
    // are made resident.
    bool init_cache(std::unique_ptr<Gguf> file, size_t budget) {
        ExpertCache& C = *cache;
        C.file = std::move(file);
        auto a256 = [](size_t v) { return (v + 255) & ~(size_t)255; };
        C.off[0] = 0;
        C.off[1] = a256(C.comp[0]);
        C.off[2] = a256(C.off[1] + C.comp[1]);
        C.foot = a256(C.off[2] + C.comp[2]);
        C.slots = (int)std::min<size_t>(budget / C.foot, (size_t)n_layer * n_expert);
        if (C.slots < n_expert) return fail("expert budget below one layer's experts");
        if (!dalloc(C.dev, (size_t)C.slots * C.foot)) return fail("cannot allocate the expert cache");
        // DMA source: the mapping registered read-only, else a pinned copy of the file, else the pageable
        // mapping (the driver then stages every fill)
        C.host = C.file->map;
        if (cudaHostRegister(const_cast<uint8_t*>(C.file->map), C.file->size, cudaHostRegisterReadOnly) == cudaSuccess) {
            C.pinned = true;
        } else {
            cudaGetLastError();
            if (cudaHostAlloc((void**)&C.host_copy, C.file->size, cudaHostAllocDefault) == cudaSuccess) {
                const unsigned nt = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
                std::vector<std::thread> pool;
                const size_t per = (C.file->size + nt - 1) / nt;
                for (unsigned t = 0; t < nt; t++)
                    pool.emplace_back([&, t]() {
                        const size_t b = std::min(C.file->size, (size_t)t * per), n = std::min(C.file->size - b, per);
                        memcpy(C.host_copy + b, C.file->map + b, n);
                    });
                for (auto& th : pool) th.join();
                C.host = C.host_copy;
                C.pinned = true;
            } else {
                cudaGetLastError();
                C.host_copy = nullptr;
            }
        }
        const size_t nk = (size_t)n_layer * n_expert;
        for (int c = 0; c < 3; c++)
            if (C.src[c].size() != nk) return fail("expert table of the cache incomplete");
        C.slot_of.assign(nk, -1);
        C.owner.assign(C.slots, -1);
        C.last_use.assign(C.slots, 0);
        C.pin.assign(C.slots, 0);
        C.from_prefetch.assign(C.slots, 0);
        C.last_set.assign(n_layer, {});
        C.ready.assign(C.slots, nullptr);
        for (auto& ev : C.ready)
            if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return fail("cache events");
        if (cudaStreamCreateWithFlags(&C.side, cudaStreamNonBlocking) != cudaSuccess) return fail("cache stream");
        if (cudaHostAlloc((void**)&C.h_tab, nk * 3 * 8, cudaHostAllocDefault) != cudaSuccess ||
            cudaHostAlloc((void**)&C.h_ids, (size_t)MAXB * n_used * 4, cudaHostAllocDefault) != cudaSuccess)
            return fail("cache pinned buffers");
        if (!dalloc(C.d_ids, (size_t)MAXB * n_used * 4) || !dalloc(C.d_w, (size_t)MAXB * n_used * 4))
            return fail("cache routing buffers");
        for (size_t i = 0; i < nk * 3; i++) C.h_tab[i] = reinterpret_cast<uint64_t>(C.dev);
        for (int l = 0; l < n_layer; l++)
            if (cudaMemcpy(const_cast<const uint8_t**>(layers[l].moe.d_gate), C.h_tab + (size_t)l * 3 * n_expert,
                           (size_t)3 * n_expert * 8, cudaMemcpyHostToDevice) != cudaSuccess)
                return fail("expert tables");
        return true;
    }
    // A free slot, or the least recently used one whose expert the current pass does not need (evicted).
    int cache_victim() {
        ExpertCache& C = *cache;
        int best = -1;
        for (int sl = 0; sl < C.slots; sl++) {
            if (C.pin[sl] == C.epoch) continue;
            if (C.owner[sl] < 0) return sl;
            if (best < 0 || C.last_use[sl] < C.last_use[best]) best = sl;
        }
        if (best >= 0) {
            C.slot_of[C.owner[best]] = -1;
            C.owner[best] = -1;
            C.evictions++;
        }
        return best;
    }
    // Copies expert `key` (layer * E + expert) into slot sl on the fill stream.
    bool cache_fill(int sl, int key) {
        ExpertCache& C = *cache;
        if (sl < 0 || sl >= C.slots || key < 0 || (size_t)key >= C.slot_of.size()) return false;
        for (int c = 0; c < 3; c++)
            if ((size_t)key >= C.src[c].size() || C.src[c][key] + C.comp[c] > C.file->size) return false;
        uint8_t* d = C.dev + (size_t)sl * C.foot;
        for (int c = 0; c < 3; c++)
            if (cudaMemcpyAsync(d + C.off[c], C.host + C.src[c][key], C.comp[c], cudaMemcpyHostToDevice, C.side) !=
                cudaSuccess)
                return false;
        if (cudaEventRecord(C.ready[sl], C.side) != cudaSuccess) return false;
        C.owner[sl] = key;
        C.slot_of[key] = sl;
        C.bytes += C.comp[0] + C.comp[1] + C.comp[2];
        return true;
    }
    // The MoE pass hook: the routing of the pass (the same top-k its kernels compute) read back, every
    // routed expert made resident (hits wait for a fill in flight; misses evict and fill), the layer's
    // pointer table uploaded, then the experts the next layer routed at its last pass prefetched into
    // slots this pass does not use, overlapping this layer's expert kernels.
    int cache_resident(const float* d_logits, int T, cudaStream_t s) {
        ExpertCache& C = *cache;
        const int l = cur_layer, E = n_expert, K = n_used;
        if (eahmmf_cuda_route_topk(d_logits, T, E, K, C.d_ids, C.d_w, s, status) != ST_OK ||
            cudaMemcpyAsync(C.h_ids, C.d_ids, (size_t)T * K * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess)
            return ST_CUDA;
        C.epoch++;
        std::vector<int> need(C.h_ids, C.h_ids + (size_t)T * K);
        std::sort(need.begin(), need.end());
        need.erase(std::unique(need.begin(), need.end()), need.end());
        uint64_t* tab = C.h_tab + (size_t)l * 3 * E;
        for (int e : need) {
            if (e < 0 || e >= E) return ST_BAD_INDEX;
            const int key = l * E + e;
            int sl = C.slot_of[key];
            if (sl >= 0) {
                C.hits++;
                if (C.from_prefetch[sl]) C.prefetch_hits++;
            } else {
                C.misses++;
                sl = cache_victim();
                if (sl < 0) return ST_CAPACITY;
                if (!cache_fill(sl, key)) return ST_CUDA;
            }
            C.from_prefetch[sl] = 0;
            if (cudaStreamWaitEvent(s, C.ready[sl], 0) != cudaSuccess) return ST_CUDA;
            C.pin[sl] = C.epoch;
            C.last_use[sl] = ++C.tick;
            for (int c = 0; c < 3; c++) tab[(size_t)c * E + e] = reinterpret_cast<uint64_t>(C.dev + (size_t)sl * C.foot + C.off[c]);
        }
        if (cudaMemcpyAsync(const_cast<const uint8_t**>(layers[l].moe.d_gate), tab, (size_t)3 * E * 8,
                            cudaMemcpyHostToDevice, s) != cudaSuccess)
            return ST_CUDA;
        C.last_set[l] = need;
        const int ln = (l + 1) % n_layer;
        for (int e : C.last_set[ln]) {
            const int key = ln * E + e;
            if (C.slot_of[key] >= 0) continue;
            const int sl = cache_victim();
            if (sl < 0) break;
            if (!cache_fill(sl, key)) return ST_CUDA;
            C.prefetched++;
            C.from_prefetch[sl] = 1;
            C.last_use[sl] = ++C.tick;
        }
        return ST_OK;
    }
    static int cache_hook(void* ctx, const float* d_logits, int T, int E, cudaStream_t s) {
        (void)E;
        return static_cast<EahmmfEngine*>(ctx)->cache_resident(d_logits, T, s);
    }

    // host -> device through two pinned staging halves (the mapping is pageable)
    // (keep_staging: the pinned halves stay allocated for the next call; the last call passes false)
    uint8_t* up_stage[2] = {nullptr, nullptr};
    cudaEvent_t up_ev[2] = {nullptr, nullptr};
    bool upload(const uint8_t* src, size_t n, uint8_t* dst = nullptr, bool keep_staging = false) {
        if (!dst) dst = weights;
        const size_t half = 64u << 20;
        uint8_t** stage = up_stage;
        cudaEvent_t* ev = up_ev;
        bool ok = true;
        for (int i = 0; i < 2 && ok; i++) {
            if (!stage[i]) ok = cudaHostAlloc((void**)&stage[i], half, cudaHostAllocDefault) == cudaSuccess;
            if (ok && !ev[i]) ok = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) == cudaSuccess;
        }
        bool live[2] = {false, false};
        for (size_t o = 0, k = 0; ok && o < n; o += half, k ^= 1) {
            const size_t c = std::min(half, n - o);
            if (live[k]) ok = cudaEventSynchronize(ev[k]) == cudaSuccess;
            if (!ok) break;
            memcpy(stage[k], src + o, c);
            ok = cudaMemcpyAsync(dst + o, stage[k], c, cudaMemcpyHostToDevice, st) == cudaSuccess &&
                 cudaEventRecord(ev[k], st) == cudaSuccess;
            live[k] = true;
        }
        if (cudaStreamSynchronize(st) != cudaSuccess) ok = false;
        if (!keep_staging)
            for (int i = 0; i < 2; i++) {
                if (stage[i]) cudaFreeHost(stage[i]);
                if (ev[i]) cudaEventDestroy(ev[i]);
                stage[i] = nullptr;
                ev[i] = nullptr;
            }
        return ok;
    }

    bool set_state(int pos, int n_out_cap) {
        DecodeState s{};
        s.pos = pos;
        s.token = 0;
        s.ticket = 0;
        s.n_out = 0;
        s.cap_out = n_out_cap;
        s.out = out;
        *h_state = s;
        hpos = pos;
        hn_out = 0;
        return cudaMemcpyAsync(state, h_state, sizeof(DecodeState), cudaMemcpyHostToDevice, st) == cudaSuccess;
    }
    bool ensure_out(int n) {
        if (n <= cap_out) return true;
        int* p = nullptr;
        if (!dalloc(p, (size_t)n * 4)) return false;
        out = p;  // the old buffer stays in `allocs` until the engine is freed; the captured step reads the
        cap_out = n;  // history pointer from the device state, so it needs no re-capture
        return true;
    }
    // Context splits of the attention kernel: independent of the tokens per pass, so that every token's
    // softmax is merged in the same order however the prompt is split into passes.
    int nsplit_for(int) const {
        const int nch = std::max(1, (n_ctx + ATT_CH - 1) / ATT_CH);
        return std::max(1, std::min({nch, 128, 2 * 148 / std::max(1, n_kv)}));
    }

    // profile: an event after each operation, tagged with the operation's class
    bool mark(int cls) {
        if (!prof) return true;
        if (pn == (int)pev.size()) {
            cudaEvent_t v;
            if (cudaEventCreate(&v) != cudaSuccess) return false;
            pev.push_back(v);
            pcls.push_back(0);
        }
        pcls[pn] = cls;
        return cudaEventRecord(pev[pn++], st) == cudaSuccess;
    }
    bool collect() {
        if (!prof || pn < 2) return true;
        if (cudaEventSynchronize(pev[pn - 1]) != cudaSuccess) return false;
        for (int i = 1; i < pn; i++) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, pev[i - 1], pev[i]) != cudaSuccess) return false;
            psum[pcls[i]] += ms * 1000.0;
        }
        psteps++;
        pn = 0;
        return true;
    }

    // The single-token layer with the norm and merge kernels fused away: the q|k|v GEMV forms its
    // activations itself (pending MoE combine + attention RMSNorm), the attention launch merges its
    // splits, the o-projection forms its activations from the merged row and adds the pending combine
    // to the residual rows it owns; then the router launch (FFN RMSNorm) and the MoE block, whose combine
    // is left pending for the next layer. Same arithmetic as the multi-token path.
    bool fused_step_ok(const Layer& L) const {
        return L.fused && gemv_mma_ok(QMat{L.wq[0], L.qkv_type[0], D, QD + 2 * KD, L.qkv_rb[0]}) &&
               gemv_mma_ok(QMat{L.wo, L.wo_type, QD, D, L.wo_rb}) && n_used <= 32 && L.moe.d_router;
    }
    int layer_step1(const Layer& L, float* lk, float* lv, float scale, int nsplit, MoeDeferred& pending) {
        const int ldq = QD + 2 * KD;
        if (!mark(1)) return ST_CUDA;
        GemvXArgs g{};
        g.W = QMat{L.wq[0], L.qkv_type[0], D, ldq, L.qkv_rb[0]};
        g.m = 1;
        g.Y = qkv;
        g.ldy = ldq;
        g.status = status;
        g.pro = GEMV_PRO_NORM;
        g.prow = x;
        g.py = pending.y;
        g.pslots = nullptr;  // single-token MoE call: the token's slots are 0..K-1 in expert order
        g.pw = pending.slot_w;
        g.pK = pending.y ? pending.K : 0;
        g.pnw = L.attn_norm;
        g.peps = eps;
        if (launch_gemv_xf(g, st) != cudaSuccess || !mark(2)) return ST_CUDA;
        RopeFuse rf{};
        rf.qkv = qkv;
        rf.qn = L.q_norm;
        rf.kn = L.k_norm;
        rf.eps = eps;
        rf.cs = rope_cs;
        rf.cnt = att_cnt;
        rf.att = att;
        if (!mark(3) ||
            launch_attention(hd, q, lk, lv, n_head, n_kv, scale, fst, 1, nsplit, attn_part, att, XF{}, rf, -1, st) !=
                cudaSuccess ||
            !mark(4))
            return ST_CUDA;
        GemvXArgs o{};
        o.W = QMat{L.wo, L.wo_type, QD, D, L.wo_rb};
        o.m = 1;
        o.Y = x;
        o.ldy = D;
        o.accumulate = 1;
        o.status = status;
        o.pro = GEMV_PRO_ROW;
        o.prow = att;
        o.ey = pending.y;
        o.eslots = nullptr;
        o.ew = pending.slot_w;
        o.eK = pending.y ? pending.K : 0;
        if (launch_gemv_xf(o, st) != cudaSuccess || !mark(5)) return ST_CUDA;
        pending = MoeDeferred{};
        if (!mark(6)) return ST_CUDA;
        const MoeHook hk{&EahmmfEngine::cache_hook, this};
        const int rc = moe_layer_run(&L.moe, 1, x, nullptr, x, moe_ws, moe_ws_bytes, st, status, &pending, L.ffn_norm, eps,
                                     cache ? &hk : nullptr);
        if (rc != ST_OK || !mark(7)) return rc != ST_OK ? rc : ST_CUDA;
        return trace_layer(1);
    }
    // routing of the layer just run (ids, then weights, at the head of the MoE workspace) into the trace
    int trace_layer(int nb) {
        if (!trace) return ST_OK;
        const size_t nk = (size_t)nb * n_used;
        h_ids.resize(nk);
        h_w.resize(nk);
        const size_t woff = (nk * 4 + 255) & ~(size_t)255;
        if (cudaMemcpyAsync(h_ids.data(), moe_ws, nk * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(h_w.data(), static_cast<uint8_t*>(moe_ws) + woff, nk * 4, cudaMemcpyDeviceToHost, st) !=
                cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            return ST_CUDA;
        trace_ids.insert(trace_ids.end(), h_ids.begin(), h_ids.end());
        trace_w.insert(trace_w.end(), h_w.begin(), h_w.end());
        return ST_OK;
    }

    // One forward pass of nb tokens at the device position state->pos (which it does not change).
    // tok: device pointer to nb token ids. want_logits: logits of the last token into `logits`.
    int forward(const int* tok, int nb, bool want_logits, bool batch = false) {
        fst = batch ? bstate : state;
        const int nsplit = nsplit_for(nb);
        const float scale = 1.0f / sqrtf((float)hd);
        if (!mark(0)) return ST_CUDA;
        if (launch_rope_table(fst, inv_freq, hd / 2, nb, rope_cs, st) != cudaSuccess) return ST_CUDA;
        if (launch_embed(embd, embd_type, embd_rb, D, n_embd_rows, tok, nb, x, status, st) != cudaSuccess)
            return ST_CUDA;
        if (!mark(0)) return ST_CUDA;
        const int ldq = QD + 2 * KD;
        const XF xf_all = xf_carve(xf_rows, MAXB, D);
        auto xf_row = [&](int t0) {  // XF view starting at row t0 of xf_all
            XF v = xf_all;
            v.frag += (size_t)t0 * (D >> 5) * 12;
            v.sum += (size_t)t0 * ((D >> 4) + XF_SUM_PAD);
            v.gs += (size_t)t0 * xf_gs_bytes(D);
            return v;
        };
        // GEMV of a matrix with K = D over the rows prepared in xf_all (tensor-core path), or over xn
        auto gemv_d = [&](const uint8_t* w, int type, int rows, size_t rb, float* out, int ldo) -> int {
            const QMat W{w, type, D, rows, rb};
            if (!gemv_mma_ok(W))
                return eahmmf_cuda_gemv(w, type, D, rows, rb, xn, nb, D, out, ldo, 0, gemv_ws, gemv_ws_bytes, st);
            if (nb > XPASS && gemm_xf_ok(W)) {  // prompt passes: every weight tile read once
                GemvXArgs g{};
                g.W = W;
                g.xf = xf_all;
                g.m = nb;
                g.Y = out;
                g.ldy = ldo;
                g.accumulate = 0;
                g.status = status;
                return launch_gemm_xf(g, st) == cudaSuccess ? ST_OK : ST_CUDA;
            }
            for (int t0 = 0; t0 < nb; t0 += XPASS) {
                GemvXArgs g{};
                g.W = W;
                g.xf = xf_row(t0);
                g.m = std::min(XPASS, nb - t0);
                g.Y = out + (size_t)t0 * ldo;
                g.ldy = ldo;
                g.accumulate = 0;
                g.status = status;
                if (launch_gemv_xf(g, st) != cudaSuccess) return ST_CUDA;
            }
            return ST_OK;
        };
        MoeDeferred pending;  // combine of the previous layer's MoE block, fused into the next norm
        const MoeHook hk{&EahmmfEngine::cache_hook, this};  // oversubscribed mode: residency before the experts
        for (int l = 0; l < n_layer; l++) {
            const Layer& L = layers[l];
            cur_layer = l;
            // the layer's cache; a single-sequence pass sees its slot's rows, a multi-sequence step all
            // slots (rows slot * n_ctx + position, from bstate)
            const size_t lo = ((size_t)l * n_slots + (batch ? 0 : slot_cur)) * n_ctx * KD;
            float* lk = kc + lo;
            float* lv = vc + lo;
            if (nb == 1 && !batch && fused_step_ok(L)) {  // single-token step: 6 launches per layer
                const int rc = layer_step1(L, lk, lv, scale, nsplit, pending);
                if (rc != ST_OK) return rc;
                continue;
            }
            NormPrepArgs na{};
            na.x = x;
            na.ldx = D;
            na.n = D;
            na.t0 = 0;
            na.w = L.attn_norm;
            na.eps = eps;
            na.y = pending.y;
            na.token_slots = pending.token_slots;
            na.slot_w = pending.slot_w;
            na.K = pending.K;
            na.xf = xf_all;
            na.xn = xn;
            if (launch_norm_prep(na, nb, st) != cudaSuccess || !mark(1)) return ST_CUDA;
            pending = MoeDeferred{};
            int rc;
            if (L.fused) {
                rc = gemv_d(L.wq[0], L.qkv_type[0], ldq, L.qkv_rb[0], qkv, ldq);
            } else {
                const int rows[3] = {QD, KD, KD}, col[3] = {0, QD, QD + KD};
                rc = ST_OK;
                for (int c = 0; c < 3 && rc == ST_OK; c++)
                    rc = gemv_d(L.wq[c], L.qkv_type[c], rows[c], L.qkv_rb[c], qkv + col[c], ldq);
            }
            if (rc != ST_OK || !mark(2)) return rc != ST_OK ? rc : ST_CUDA;
            RopeFuse rf{};
            if (nb == 1 && !batch) {  // single-token step: norms, rotation and KV append inside the attention kernel
                rf.qkv = qkv;
                rf.qn = L.q_norm;
                rf.kn = L.k_norm;
                rf.eps = eps;
                rf.cs = rope_cs;
                if (!mark(3)) return ST_CUDA;
            } else if (launch_qk_rope_kv(hd, qkv, n_head, n_kv, L.q_norm, L.k_norm, eps, rope_cs, fst, nb, q, lk,
                                         lv, st) != cudaSuccess ||
                       !mark(3)) {
                return ST_CUDA;
            }
            const XF xf_o = xf_carve(xf_att, MAXB, QD);
            if (launch_attention(hd, q, lk, lv, n_head, n_kv, scale, fst, nb, nsplit, attn_part, att, xf_o, rf, pos_host,
                                 st) !=
                    cudaSuccess ||
                !mark(4))
                return ST_CUDA;
            {  // o-projection accumulated into the residual, over the merged rows in fragment form
                const QMat W{L.wo, L.wo_type, QD, D, L.wo_rb};
                if (!gemv_mma_ok(W)) {
                    rc = eahmmf_cuda_gemv(L.wo, L.wo_type, QD, D, L.wo_rb, att, nb, QD, x, D, 1, gemv_ws, gemv_ws_bytes,
                                          st);
                    if (rc != ST_OK) return rc;
                } else if (nb > XPASS && gemm_xf_ok(W)) {
                    GemvXArgs g{};
                    g.W = W;
                    g.xf = xf_o;
                    g.m = nb;
                    g.Y = x;
                    g.ldy = D;
                    g.accumulate = 1;
                    g.status = status;
                    if (launch_gemm_xf(g, st) != cudaSuccess) return ST_CUDA;
                } else {
                    for (int t0 = 0; t0 < nb; t0 += XPASS) {
                        GemvXArgs g{};
                        g.W = W;
                        g.xf = xf_o;
                        g.xf.frag += (size_t)t0 * (QD >> 5) * 12;
                        g.xf.sum += (size_t)t0 * ((QD >> 4) + XF_SUM_PAD);
                        g.xf.gs += (size_t)t0 * xf_gs_bytes(QD);
                        g.m = std::min(XPASS, nb - t0);
                        g.Y = x + (size_t)t0 * D;
                        g.ldy = D;
                        g.accumulate = 1;
                        g.status = status;
                        if (launch_gemv_xf(g, st) != cudaSuccess) return ST_CUDA;
                    }
                }
                if (!mark(5)) return ST_CUDA;
            }
            if (nb <= FUSED_ROUTE_TMAX) {  // the FFN RMSNorm runs inside the router launch
                if (!mark(6)) return ST_CUDA;
                rc = moe_layer_run(&L.moe, nb, x, nullptr, x, moe_ws, moe_ws_bytes, st, status, &pending, L.ffn_norm,
                                   eps, cache ? &hk : nullptr);
            } else {
                if (launch_rmsnorm(x, D, L.ffn_norm, xn, D, nb, D, eps, st) != cudaSuccess || !mark(6)) return ST_CUDA;
                rc = moe_layer_run(&L.moe, nb, xn, nullptr, x, moe_ws, moe_ws_bytes, st, status, &pending, nullptr, 0.f,
                                   cache ? &hk : nullptr);
            }
            if (rc != ST_OK || !mark(7)) return rc != ST_OK ? rc : ST_CUDA;
            if (trace_layer(nb) != ST_OK) return ST_CUDA;
        }
        if (want_logits) {  // last row: the pending combine, the output norm, the output GEMV
            NormPrepArgs na{};
            na.x = x;
            na.ldx = D;
            na.n = D;
            na.t0 = nb - 1;
            na.w = out_norm;
            na.eps = eps;
            na.y = pending.y;
            na.token_slots = pending.token_slots;
            na.slot_w = pending.slot_w;
            na.K = pending.K;
            na.xf = xf_all;
            na.xn = xn;
            if (batch) {  // every row is a sequence's next-token logits
                na.t0 = 0;
                if (launch_norm_prep(na, nb, st) != cudaSuccess) return ST_CUDA;
                const int rc = gemv_d(out_w, out_type, n_vocab, out_rb, logits_b, n_vocab);
                if (rc != ST_OK || !mark(8)) return rc != ST_OK ? rc : ST_CUDA;
                return ST_OK;
            }
            if (launch_norm_prep(na, 1, st) != cudaSuccess) return ST_CUDA;
            const int save_nb = nb;
            nb = 1;  // gemv_d over the single prepared row
            const int rc = gemv_d(out_w, out_type, n_vocab, out_rb, logits, n_vocab);
            nb = save_nb;
            if (rc != ST_OK || !mark(8)) return rc != ST_OK ? rc : ST_CUDA;
        }
        return ST_OK;
    }

    // Prompt tokens through forward passes of up to n_batch tokens from position p0 (Engine::eval,
    // qwen3moe.cpp:1078-1084); leaves state->pos = p0 + n and the last token's logits in `logits`.
    int eval_dev(const int* htoks, int n, int p0, int n_batch) {
        if (!set_state(p0, cap_out) || cudaMemsetAsync(status, 0, 4, st) != cudaSuccess) return ST_CUDA;
        for (int i = 0; i < n; i += n_batch) {
            const int nb = std::min(n_batch, n - i);
            // the pinned staging is reused per chunk: wait for the previous chunk's copy to be consumed
            if (cudaStreamSynchronize(st) != cudaSuccess) return ST_CUDA;
            memcpy(h_toks, htoks + i, (size_t)nb * 4);
            if (cudaMemcpyAsync(toks, h_toks, (size_t)nb * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
                return ST_CUDA;
            pos_host = p0 + i;  // the pass's position, known here (the captured decode step reads it on the device)
            const int rc = forward(toks, nb, i + nb == n);
            pos_host = -1;
            if (rc != ST_OK) return rc;
            if (launch_advance(state, nb, st) != cudaSuccess) return ST_CUDA;
            hpos += nb;
        }
        return ST_OK;
    }

    // KV caches for n sequence slots of n_ctx positions each (zeroed); the previous caches are freed.
    bool set_slots(int n) {
        if (n < 1) return false;
        if (cudaStreamSynchronize(st) != cudaSuccess) return false;
        const size_t kvn = (size_t)n_layer * n * n_ctx * KD;
        float *k2 = nullptr, *v2 = nullptr;
        if (cudaMalloc(&k2, kvn * 4) != cudaSuccess) return false;
        if (cudaMalloc(&v2, kvn * 4) != cudaSuccess) {
            cudaFree(k2);
            return false;
        }
        if (cudaMemset(k2, 0, kvn * 4) != cudaSuccess || cudaMemset(v2, 0, kvn * 4) != cudaSuccess) {
            cudaFree(k2);
            cudaFree(v2);
            return false;
        }
        for (void*& a : allocs)
            if (a == kc || a == vc) {
                cudaFree(a);
                a = nullptr;
            }
        allocs.push_back(k2);
        allocs.push_back(v2);
        kc = k2;
        vc = v2;
        n_slots = n;
        slot_cur = 0;
        if (step_graph) {  // the captured step holds the old cache pointers
            cudaGraphExecDestroy(step_graph);
            step_graph = nullptr;
            graph_nodes = 0;
        }
        return true;
    }

    // The uniform draws of the next m generated indices, from the sampler's stream (the reference draws
    // one per sampled token, qwen3moe.cpp:1125), into u_dev[hn_out ..]; nothing when greedy.
    bool prepare_draws(int m) {
        if (!sampling || sparams.temp <= 0.f || m <= 0) return true;
        if (hn_out + m > n_ctx + 1) return false;
        for (int i = 0; i < m; i++) u_host[hn_out + i] = eahmmf_rng_uniform(rng);
        return cudaMemcpyAsync(u_dev + hn_out, u_host + hn_out, (size_t)m * 4, cudaMemcpyHostToDevice, st) ==
               cudaSuccess;
    }
    // Token selection over `logits` into the state (token, history, position + advance).
    // The caller has prepared the index's draw (prepare_draws) and advanced hn_out.
    cudaError_t select(int advance) {
        if (!sampling) return launch_argmax(logits, n_vocab, amax_blk, amax_nblk, state, advance, st);
        SampleArgs a{};
        a.logits = logits;
        a.n = n_vocab;
        a.p = sparams;
        a.st = state;
        a.u_arr = u_dev;
        a.advance = advance;
        a.cand = static_cast<uint64_t*>(samp_ws);
        return launch_sample(a, st);
    }

    // One decode step: forward of state->token at state->pos, then the argmax records the next token
    // and advances the position. Captured once, replayed per token.
    int step(bool use_graph) {
        hpos++;  // the step's argmax advances the position
        if (!prepare_draws(1)) return ST_CUDA;
        hn_out++;
        if (!use_graph || trace || prof || cache) {  // oversubscribed mode: the host acts inside the step
            pn = 0;
            const int rc = forward(&state->token, 1, true);
            if (rc != ST_OK) return rc;
            if (select(1) != cudaSuccess || !mark(9) || !collect()) return ST_CUDA;
            return ST_OK;
        }
        if (!step_graph) {
            cudaGraph_t gr = nullptr;
            if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return ST_CUDA;
            int rc = forward(&state->token, 1, true);
            if (rc == ST_OK && select(1) != cudaSuccess) rc = ST_CUDA;
            const cudaError_t ce = cudaStreamEndCapture(st, &gr);
            if (rc != ST_OK || ce != cudaSuccess) {
                if (gr) cudaGraphDestroy(gr);
                return rc != ST_OK ? rc : ST_CUDA;
            }
            size_t nodes = 0;
            if (cudaGraphGetNodes(gr, nullptr, &nodes) == cudaSuccess) graph_nodes = (int)nodes;
            const cudaError_t ie = cudaGraphInstantiate(&step_graph, gr, 0);
            cudaGraphDestroy(gr);
            if (ie != cudaSuccess) {
                step_graph = nullptr;
                return ST_CUDA;
            }
        }
        return cudaGraphLaunch(step_graph, st) == cudaSuccess ? ST_OK : ST_CUDA;
    }

    int read_status() {
        int s = 0;
        if (cudaMemcpyAsync(h_toks, status, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            return ST_CUDA;
        s = h_toks[0];
        return s;
    }
};

// ---------------------------------------------------------------------------------------------------
// 4. engine entry points
// ---------------------------------------------------------------------------------------------------
extern "C" EahmmfEngine* eahmmf_engine_load_budget(const char* gguf_path, int n_ctx, size_t expert_vram_bytes,
                                                   char* err, size_t err_cap) {
    EahmmfEngine* e = new EahmmfEngine();
    if (!gguf_path || !e->load(gguf_path, n_ctx, expert_vram_bytes)) {
        if (err && err_cap) snprintf(err, err_cap, "%s", gguf_path ? e->err.c_str() : "null path");
        delete e;
        return nullptr;
    }
    return e;
}

extern "C" int eahmmf_engine_cache_stats(EahmmfEngine* e, uint64_t* v, int cap) {
    if (!e || !v || cap < EAHMMF_CACHE_STATS) return ST_BAD_ARG;
    if (!e->cache) {
        for (int i = 0; i < EAHMMF_CACHE_STATS; i++) v[i] = 0;
        return ST_OK;
    }
    const auto& C = *e->cache;
    const uint64_t vals[EAHMMF_CACHE_STATS] = {(uint64_t)C.slots, C.hits, C.misses, C.prefetched, C.prefetch_hits,
                                               C.evictions, C.bytes, (uint64_t)C.pinned};
    for (int i = 0; i < EAHMMF_CACHE_STATS; i++) v[i] = vals[i];
    return ST_OK;
}

extern "C" EahmmfEngine* eahmmf_engine_load(const char* gguf_path, int n_ctx, char* err, size_t err_cap) {
    EahmmfEngine* e = new EahmmfEngine();
    if (!gguf_path || !e->load(gguf_path, n_ctx)) {
        if (err && err_cap) snprintf(err, err_cap, "%s", gguf_path ? e->err.c_str() : "null path");
        delete e;
        return nullptr;
    }
    return e;
}

extern "C" void eahmmf_engine_free(EahmmfEngine* e) { delete e; }

extern "C" int eahmmf_engine_dims(EahmmfEngine* e, int* dims) {
    if (!e || !dims) return ST_BAD_ARG;
    const int v[11] = {e->n_layer, e->D,  e->n_head,  e->n_kv,  e->hd, e->n_expert,
                       e->n_used,  e->FF, e->n_vocab, e->n_ctx, e->n_embd_rows};
    memcpy(dims, v, sizeof v);
    return ST_OK;
}

extern "C" int eahmmf_engine_eval(EahmmfEngine* e, const int* toks, int n, int p0, int n_batch, float* logits) {
    if (!e || !toks || n < 1 || n_batch < 1 || n_batch > MAXB || p0 < 0 || p0 + n > e->n_ctx) return ST_BAD_ARG;
    int rc = e->eval_dev(toks, n, p0, n_batch);
    if (rc != ST_OK) return rc;
    if (logits && cudaMemcpyAsync(logits, e->logits, (size_t)e->n_vocab * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess)
        return ST_CUDA;
    rc = e->read_status();
    return rc;
}

namespace {
// The prompt from position 0, then n_gen tokens chosen by the engine's selection (the first maximum, or
// the configured sampler), out[0] being the prompt's: the reference's generate loop
// (qwen3moe.cpp:1294-1310) with the whole prompt in one eval.
int generate(EahmmfEngine* e, const int* prompt, int n_prompt, int n_gen, int n_batch, int* out, float* first_logits) {
    if (!e || !prompt || !out || n_prompt < 1 || n_gen < 1 || n_batch < 1 || n_batch > MAXB ||
        n_prompt + n_gen > e->n_ctx)
        return ST_BAD_ARG;
    if (!e->ensure_out(n_gen)) return ST_CUDA;
    int rc = e->eval_dev(prompt, n_prompt, 0, n_batch);
    if (rc != ST_OK) return rc;
    // state: pos = n_prompt; cap_out was set by eval_dev's set_state
    if (first_logits &&
        cudaMemcpyAsync(first_logits, e->logits, (size_t)e->n_vocab * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess)
        return ST_CUDA;
    if (!e->prepare_draws(1)) return ST_CUDA;
    e->hn_out++;
    if (e->select(0) != cudaSuccess) return ST_CUDA;
    for (int i = 1; i < n_gen; i++) {
        rc = e->step(true);
        if (rc != ST_OK) return rc;
    }
    if (cudaMemcpyAsync(out, e->out, (size_t)n_gen * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess) return ST_CUDA;
    return e->read_status();
}
}  // namespace

extern "C" int eahmmf_engine_greedy(EahmmfEngine* e, const int* prompt, int n_prompt, int n_gen, int n_batch, int* out,
                                    float* first_logits) {
    if (e && e->sampling) return ST_BAD_ARG;  // a sampler is configured: eahmmf_engine_generate
    return generate(e, prompt, n_prompt, n_gen, n_batch, out, first_logits);
}

extern "C" int eahmmf_engine_generate(EahmmfEngine* e, const int* prompt, int n_prompt, int n_gen, int n_batch,
                                      int* out) {
    return generate(e, prompt, n_prompt, n_gen, n_batch, out, nullptr);
}

extern "C" int eahmmf_engine_sampler(EahmmfEngine* e, const EahmmfSamplerParams* p, uint64_t seed) {
    if (!e) return ST_BAD_ARG;
    if (p && !sample_ok(*p, e->n_vocab)) return ST_BAD_ARG;
    if (cudaStreamSynchronize(e->st) != cudaSuccess) return ST_CUDA;
    if (e->step_graph) {  // the captured step holds the previous selection
        cudaGraphExecDestroy(e->step_graph);
        e->step_graph = nullptr;
        e->graph_nodes = 0;
    }
    e->sampling = p != nullptr;
    if (p) e->sparams = *p;
    if (e->rng) eahmmf_rng_free(e->rng);
    e->rng = p ? eahmmf_rng_create(seed) : nullptr;
    return ST_OK;
}

extern "C" int eahmmf_engine_decode(EahmmfEngine* e, int n_steps, int* out, float* device_ms) {
    if (!e || n_steps < 1) return ST_BAD_ARG;
    if (cudaMemcpyAsync(e->h_state, e->state, sizeof(DecodeState), cudaMemcpyDeviceToHost, e->st) != cudaSuccess ||
        cudaStreamSynchronize(e->st) != cudaSuccess)
        return ST_CUDA;
    if (e->h_state->pos + n_steps > e->n_ctx) return ST_BAD_ARG;
    e->hpos = e->h_state->pos;
    e->hn_out = e->h_state->n_out;
    const int have = e->h_state->n_out;
    if (have + n_steps > e->cap_out) {
        // grow the history and re-point the state at it (copying what was recorded)
        int* old = e->out;
        const int cap_old = e->cap_out;
        if (!e->ensure_out(have + n_steps)) return ST_CUDA;
        if (old && cap_old && cudaMemcpyAsync(e->out, old, (size_t)std::min(have, cap_old) * 4,
                                              cudaMemcpyDeviceToDevice, e->st) != cudaSuccess)
            return ST_CUDA;
        DecodeState s = *e->h_state;
        s.out = e->out;
        s.cap_out = e->cap_out;
        *e->h_state = s;
        if (cudaMemcpyAsync(e->state, e->h_state, sizeof(DecodeState), cudaMemcpyHostToDevice, e->st) != cudaSuccess)
            return ST_CUDA;
    }
    if (cudaEventRecord(e->ev0, e->st) != cudaSuccess) return ST_CUDA;
    for (int i = 0; i < n_steps; i++) {
        const int rc = e->step(true);
        if (rc != ST_OK) return rc;
    }
    if (cudaEventRecord(e->ev1, e->st) != cudaSuccess || cudaEventSynchronize(e->ev1) != cudaSuccess) return ST_CUDA;
    if (device_ms) cudaEventElapsedTime(device_ms, e->ev0, e->ev1);
    if (out && cudaMemcpyAsync(out, e->out + have, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess)
        return ST_CUDA;
    return e->read_status();
}

extern "C" int eahmmf_engine_step(EahmmfEngine* e, int token, int* next) {
    if (!e || !next || token >= e->n_embd_rows) return ST_BAD_ARG;
    if (e->hpos < 0 || e->hpos >= e->n_ctx) return ST_BAD_ARG;  // no room for the token's KV row
    if (token >= 0) {
        e->h_toks[0] = token;
        if (cudaMemcpyAsync(&e->state->token, e->h_toks, 4, cudaMemcpyHostToDevice, e->st) != cudaSuccess)
            return ST_CUDA;
    }
    int rc = e->step(true);
    if (rc != ST_OK) return rc;
    if (cudaMemcpyAsync(e->h_toks + 1, &e->state->token, 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess ||
        cudaMemcpyAsync(e->h_toks + 2, e->status, 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess ||
        cudaStreamSynchronize(e->st) != cudaSuccess)
        return ST_CUDA;
    *next = e->h_toks[1];
    return e->h_toks[2];
}

extern "C" int eahmmf_engine_set_slots(EahmmfEngine* e, int n_slots) {
    if (!e || n_slots < 1 || n_slots > 4096) return ST_BAD_ARG;
    return e->set_slots(n_slots) ? ST_OK : ST_CUDA;
}

extern "C" int eahmmf_engine_prefill_slot(EahmmfEngine* e, int slot, const int* prompt, int n, int n_batch, int* first) {
    if (!e || !prompt || !first || slot < 0 || slot >= e->n_slots || n < 1 || n >= e->n_ctx || n_batch < 1 ||
        n_batch > MAXB)
        return ST_BAD_ARG;
    e->slot_cur = slot;
    int rc = e->eval_dev(prompt, n, 0, n_batch);
    e->slot_cur = 0;
    if (rc != ST_OK) return rc;
    if (launch_argmax_rows(e->logits, e->n_vocab, e->n_vocab, 1, e->d_btok, e->st) != cudaSuccess ||
        cudaMemcpyAsync(e->h_b, e->d_btok, 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess)
        return ST_CUDA;
    rc = e->read_status();
    *first = e->h_b[0];
    return rc;
}

extern "C" int eahmmf_engine_step_slots(EahmmfEngine* e, int n, const int* slots, const int* pos, const int* toks,
                                        int* next) {
    if (!e || !slots || !pos || !toks || !next || n < 1 || n > MAXB) return ST_BAD_ARG;
    for (int i = 0; i < n; i++) {
        if (slots[i] < 0 || slots[i] >= e->n_slots || pos[i] < 0 || pos[i] >= e->n_ctx || toks[i] < 0 ||
            toks[i] >= e->n_embd_rows)
            return ST_BAD_ARG;
        for (int j = 0; j < i; j++)
            if (slots[j] == slots[i]) return ST_BAD_ARG;  // one row per sequence per step
    }
    int* h = e->h_b;
    if (cudaStreamSynchronize(e->st) != cudaSuccess) return ST_CUDA;  // the staging is free
    memcpy(h, toks, (size_t)n * 4);
    memcpy(h + MAXB, pos, (size_t)n * 4);
    memcpy(h + 2 * MAXB, slots, (size_t)n * 4);
    if (cudaMemsetAsync(e->status, 0, 4, e->st) != cudaSuccess ||
        cudaMemcpyAsync(e->d_btok, h, (size_t)n * 4, cudaMemcpyHostToDevice, e->st) != cudaSuccess ||
        cudaMemcpyAsync(e->d_tpos, h + MAXB, (size_t)n * 4, cudaMemcpyHostToDevice, e->st) != cudaSuccess ||
        cudaMemcpyAsync(e->d_tslot, h + 2 * MAXB, (size_t)n * 4, cudaMemcpyHostToDevice, e->st) != cudaSuccess)
        return ST_CUDA;
    e->pn = 0;
    int rc = e->forward(e->d_btok, n, true, true);
    if (rc != ST_OK) return rc;
    if (launch_argmax_rows(e->logits_b, e->n_vocab, e->n_vocab, n, e->d_btok, e->st) != cudaSuccess ||
        cudaMemcpyAsync(h, e->d_btok, (size_t)n * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess)
        return ST_CUDA;
    rc = e->read_status();
    memcpy(next, h, (size_t)n * 4);
    return rc;
}

extern "C" int eahmmf_engine_verify(EahmmfEngine* e, int* n_checked, int* n_bad) {
    if (!e || !n_checked || !n_bad) return ST_BAD_ARG;
    if (e->cache) {  // oversubscribed mode: the resident copies in the cache's slots
        if (cudaStreamSynchronize(e->cache->side) != cudaSuccess) return ST_CUDA;
        const auto& C = *e->cache;
        e->slices.clear();
        for (int sl = 0; sl < C.slots; sl++)
            if (C.owner[sl] >= 0)
                for (int c = 0; c < 3; c++)
                    e->slices.push_back(EahmmfEngine::Slice{C.dev + (size_t)sl * C.foot + C.off[c],
                                                            C.src[c][C.owner[sl]], C.comp[c]});
    }
    const int n = (int)e->slices.size();
    *n_checked = n;
    *n_bad = 0;
    if (n == 0) return ST_OK;
    // device side: one hash per slice, all slices in one launch
    std::vector<const uint8_t*> hp(n);
    std::vector<size_t> hs(n);
    for (int i = 0; i < n; i++) {
        hp[i] = e->slices[i].dev;
        hs[i] = e->slices[i].bytes;
    }
    void* buf = nullptr;
    const size_t bytes = (size_t)n * (sizeof(void*) + sizeof(size_t) + 8);
    if (cudaMalloc(&buf, bytes) != cudaSuccess) return ST_CUDA;
    auto* dp = static_cast<const uint8_t**>(buf);
    auto* ds = reinterpret_cast<size_t*>(dp + n);
    auto* dh = reinterpret_cast<uint64_t*>(ds + n);
    std::vector<uint64_t> got(n);
    bool ok = cudaMemcpyAsync(dp, hp.data(), (size_t)n * sizeof(void*), cudaMemcpyHostToDevice, e->st) == cudaSuccess &&
              cudaMemcpyAsync(ds, hs.data(), (size_t)n * sizeof(size_t), cudaMemcpyHostToDevice, e->st) == cudaSuccess &&
              launch_hash64(dp, ds, n, dh, e->st) == cudaSuccess &&
              cudaMemcpyAsync(got.data(), dh, (size_t)n * 8, cudaMemcpyDeviceToHost, e->st) == cudaSuccess;
    // host side meanwhile: the sources, from the file as it is now, over all host threads
    Gguf g;
    std::vector<uint64_t> want(n, 0);
    const bool src_ok = g.open(e->path.c_str());
    if (src_ok) {
        const int nt = std::max(1u, std::min(64u, std::thread::hardware_concurrency()));
        std::vector<std::thread> pool;
        for (int t = 0; t < nt; t++)
            pool.emplace_back([&, t]() {
                for (int i = t; i < n; i += nt) {
                    const EahmmfEngine::Slice& sl = e->slices[i];
                    if (sl.file_off + sl.bytes <= g.size) want[i] = host_hash64(g.map + sl.file_off, sl.bytes);
                }
            });
        for (auto& th : pool) th.join();
    }
    ok = ok && cudaStreamSynchronize(e->st) == cudaSuccess;
    cudaFree(buf);
    if (!ok) return ST_CUDA;
    if (!src_ok) return ST_BAD_ARG;
    for (int i = 0; i < n; i++) *n_bad += got[i] != want[i];
    return ST_OK;
}

extern "C" void eahmmf_engine_trace(EahmmfEngine* e, int enable) {
    if (!e) return;
    e->trace = enable != 0;
    e->trace_ids.clear();
    e->trace_w.clear();
}

extern "C" int eahmmf_engine_trace_get(EahmmfEngine* e, int* ids, float* w, int cap) {
    if (!e) return 0;
    const int n = (int)std::min<size_t>((size_t)(cap > 0 ? cap : 0), e->trace_ids.size());
    if (ids) memcpy(ids, e->trace_ids.data(), sizeof(int) * n);
    if (w) memcpy(w, e->trace_w.data(), sizeof(float) * n);
    return (int)e->trace_ids.size();
}

extern "C" int eahmmf_engine_graph_nodes(EahmmfEngine* e) { return e && e->step_graph ? e->graph_nodes : 0; }

extern "C" int eahmmf_engine_profile(EahmmfEngine* e, int enable) {
    if (!e) return ST_BAD_ARG;
    e->prof = enable != 0;
    for (double& v : e->psum) v = 0;
    e->psteps = 0;
    e->pn = 0;
    return ST_OK;
}

extern "C" int eahmmf_engine_profile_read(EahmmfEngine* e, float* us, int cap) {
    if (!e || !us || cap < EahmmfEngine::NPROF || e->psteps == 0) return 0;
    for (int i = 0; i < EahmmfEngine::NPROF; i++) us[i] = (float)(e->psum[i] / e->psteps);
    for (double& v : e->psum) v = 0;
    e->psteps = 0;
    return EahmmfEngine::NPROF;
}
