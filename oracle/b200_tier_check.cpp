// oracle/b200_tier_check.cpp -- TEST INFRASTRUCTURE: the reference engine's residency tiers with
// eahmmf::B200Device as the ExpertStore's backend.
//
// The reference's own suite (tests/test_eahmmf.cpp) runs its tier matrix, residency walk and fault
// injection on SimDevice, a host-memory stand-in. This program runs the same kinds of cases on the real
// device backend of this project (include/eahmmf_b200_device.hpp), with the reference engine compiled
// unmodified (through ref_harness.cpp) and CPU matmuls: experts served from VRAM reach the CPU kernels
// through the store's d2h bounce (B200Device::cpu_readable() is false), so every case must reproduce the
// SSD-tier run bit for bit -- logits, greedy ids and the routing trace.
//
//   1. tier matrix: exec tier RAM / VRAM with unlimited, 3-, 2-, 1-expert and sub-expert budgets, and the
//      two constrained cases that exercise every pager path and the VRAM->SSD drop (the case list of the
//      reference suite's section 3, eahmmf.h's Config fields), each bitwise against the SSD baseline,
//      with store invariants and pin balance checked;
//   2. residency walk SSD -> RAM -> VRAM -> RAM -> SSD of one expert with --verify checksums, the bytes
//      read back through the backend at every step equal to the GGUF source;
//   3. backend faults (eahmmf_dev_inject_fault: failed alloc, h2d, d2h on the host side, before any CUDA
//      call): the store falls back to a valid tier and the run stays bitwise equal to the baseline.
//
// Usage: b200_tier_check <model.gguf>. Prints `key value...` lines; tests/test_gpu_store.py parses them.
#include "ref_harness.cpp"

#include <cuda_runtime.h>

#include "../include/eahmmf_b200_device.hpp"

namespace {

using namespace eahmmf;

const std::vector<int> kPrompt = {5, 17, 200, 33, 99, 3, 150, 256, 42, 77, 8, 9, 10, 11, 12};

struct Run {
    std::vector<float> logits;
    std::vector<int> gen, ids;
    std::vector<float> w;
};

bool bitwise_equal(const Run& a, const Run& b) {
    auto feq = [](const std::vector<float>& x, const std::vector<float>& y) {
        return x.size() == y.size() && (x.empty() || memcmp(x.data(), y.data(), x.size() * 4) == 0);
    };
    return feq(a.logits, b.logits) && a.gen == b.gen && a.ids == b.ids && feq(a.w, b.w);
}

// The prompt in passes of 4 tokens, then 12 greedy single-token steps, with the routing trace on.
Run decode(Engine& E) {
    E.trace_routing = true;
    E.trace_ids.clear();
    E.trace_w.clear();
    Run r;
    r.logits.resize(E.n_vocab);
    E.eval(kPrompt, 0, 4, r.logits.data());
    std::vector<float> lg = r.logits;
    int pos = (int)kPrompt.size();
    for (int i = 0; i < 12; i++) {
        int t = (int)(std::max_element(lg.begin(), lg.end()) - lg.begin());
        r.gen.push_back(t);
        E.forward(&t, 1, pos++, lg.data());
    }
    r.ids = E.trace_ids;
    r.w = E.trace_w;
    E.trace_routing = false;
    return r;
}

Config tier(Residency t, size_t ram, size_t vram, bool verify) {
    Config c;
    c.exec_tier = t;
    c.ram_budget = ram;
    c.vram_budget = vram;
    c.verify = verify;
    c.record_events = true;
    c.log_acquires = false;
    return c;
}

// Bytes of expert (l, x) as a lease serves them (through the backend's bounce when VRAM-resident) against
// the GGUF source.
bool lease_matches_source(Engine& E, int l, int x, Residency* served) {
    ExpertLease lease = E.store->acquire_lease(l, x);
    if (!lease) return false;
    const ExpertViews& v = lease.views();
    const ExpertDescriptor d = E.store->descriptor(l, x);
    const WeightView* c[3] = {&v.gate, &v.up, &v.down};
    bool ok = true;
    for (int k = 0; k < 3; k++) ok &= memcmp(c[k]->data, E.g.map + d.slice[k].file_offset, d.bytes[k]) == 0;
    if (served) *served = v.served_from;
    return ok;
}

// Device copy of expert (l, x), read back through the backend, against the GGUF source.
bool device_matches_source(Engine& E, int l, int x) {
    const ExpertDescriptor d = E.store->descriptor(l, x);
    if (!d.vram_ptr) return false;
    for (int k = 0; k < 3; k++) {
        std::vector<uint8_t> h(d.bytes[k]);
        if (!E.dev->d2h(h.data(), static_cast<const uint8_t*>(d.vram_ptr) + d.res_off[k], h.size()) ||
            memcmp(h.data(), E.g.map + d.slice[k].file_offset, h.size()) != 0)
            return false;
    }
    return true;
}

int g_all = 1;
void report(const char* name, bool ok) {
    printf("check %s %d\n", name, ok ? 1 : 0);
    if (!ok) g_all = 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: %s model.gguf\n", argv[0]);
        return 2;
    }
    eref_init(4);
    Engine E;
    E.load(argv[1], 128, false);
    const size_t FP = E.store->descriptor(0, 0).footprint;
    const Run base = decode(E);  // SSD tier, the engine's default store
    printf("baseline_trace %zu\n", base.ids.size());

    // 1. tier matrix on the device backend
    struct Case {
        const char* name;
        Config cfg;
    };
    const size_t U = SIZE_MAX;
    const Case cases[] = {
        {"ram_unlimited", tier(Residency::RAM, U, U, true)},
        {"vram_unlimited", tier(Residency::VRAM, U, U, true)},
        {"ram_3_experts", tier(Residency::RAM, 3 * FP, U, true)},
        {"vram_2_ram_unlimited", tier(Residency::VRAM, U, 2 * FP, true)},
        {"vram_2_ram_1", tier(Residency::VRAM, 1 * FP, 2 * FP, true)},
        {"vram_1_ram_1", tier(Residency::VRAM, 1 * FP, 1 * FP, true)},
        {"vram_below_one_expert", tier(Residency::VRAM, U, FP / 2, false)},
        {"vram_2_ram_2_every_path", tier(Residency::VRAM, 2 * FP, 2 * FP, true)},
        {"vram_2_ram_1_drop_path", tier(Residency::VRAM, 1 * FP, 2 * FP, true)},
    };
    for (const Case& c : cases) {
        auto* dev = new B200Device();
        if (!dev->ok()) {
            printf("backend_create 0\n");
            return 1;
        }
        if (!E.init_experts(c.cfg, std::unique_ptr<DeviceBackend>(dev))) {
            report(c.name, false);
            continue;
        }
        const Run r = decode(E);
        const Stats st = E.store->stats();
        const std::string inv = E.store->check_invariants();
        printf("case %s same %d invariants %d pinned %llu acq %llu rel %llu ssd_ram %llu ram_vram %llu vram_ram %llu "
               "ram_ssd %llu vram_ssd %llu fallbacks %llu vram_used %zu ram_used %zu\n",
               c.name, (int)bitwise_equal(r, base), (int)inv.empty(), (unsigned long long)st.pinned_now,
               (unsigned long long)st.acquires, (unsigned long long)st.releases, (unsigned long long)st.mig_n[SSD_RAM],
               (unsigned long long)st.mig_n[RAM_VRAM], (unsigned long long)st.mig_n[VRAM_RAM],
               (unsigned long long)st.mig_n[RAM_SSD], (unsigned long long)st.mig_n[VRAM_SSD],
               (unsigned long long)st.fallbacks, E.store->vram_used(), E.store->ram_used());
        if (!bitwise_equal(r, base) || !inv.empty() || st.pinned_now != 0 || st.acquires != st.releases) g_all = 0;
    }

    // 2. residency walk with checksums, bytes checked at every tier
    {
        Config c;
        c.verify = true;
        c.log_acquires = false;
        E.init_experts(c, std::unique_ptr<DeviceBackend>(new B200Device()));
        Residency sv = Residency::ERROR;
        report("walk_ssd", E.store->residency(0, 7) == Residency::SSD && lease_matches_source(E, 0, 7, &sv) &&
                               sv == Residency::SSD);
        report("walk_ram", E.store->promote(0, 7, Residency::RAM) && lease_matches_source(E, 0, 7, &sv) &&
                               sv == Residency::RAM);
        report("walk_vram", E.store->promote(0, 7, Residency::VRAM) && E.store->residency(0, 7) == Residency::VRAM &&
                                E.store->ram_used() == 0 && E.store->vram_used() == FP && device_matches_source(E, 0, 7) &&
                                lease_matches_source(E, 0, 7, &sv) && sv == Residency::VRAM);
        report("walk_back_ram", E.store->demote(0, 7, Residency::RAM) && E.store->vram_used() == 0 &&
                                    lease_matches_source(E, 0, 7, &sv) && sv == Residency::RAM);
        report("walk_back_ssd", E.store->demote(0, 7, Residency::SSD) && E.store->ram_used() == 0 &&
                                    lease_matches_source(E, 0, 7, &sv) && sv == Residency::SSD);
        report("walk_invariants", E.store->check_invariants().empty());
    }

    // 3. backend faults, injected on the host before any CUDA call
    {
        const struct {
            const char* name;
            int kind;  // 0 alloc, 1 h2d, 2 d2h
        } faults[] = {{"fault_alloc", 0}, {"fault_h2d", 1}, {"fault_d2h", 2}};
        for (const auto& f : faults) {
            auto* dev = new B200Device();
            Config c = tier(Residency::VRAM, U, U, true);
            E.init_experts(c, std::unique_ptr<DeviceBackend>(dev));
            eahmmf_dev_inject_fault(dev->d, f.kind, 3);
            const Run r = decode(E);
            const Stats st = E.store->stats();
            uint64_t fails = 0;
            for (int p = 0; p < 5; p++) fails += st.mig_fail[p];
            printf("fault %s same %d migration_failures %llu alloc_failures %llu fallbacks %llu invariants %d pinned %llu\n",
                   f.name, (int)bitwise_equal(r, base), (unsigned long long)fails,
                   (unsigned long long)st.vram_alloc_failures, (unsigned long long)st.fallbacks,
                   (int)E.store->check_invariants().empty(), (unsigned long long)st.pinned_now);
            if (!bitwise_equal(r, base) || !E.store->check_invariants().empty() || st.pinned_now != 0 ||
                (fails == 0 && st.vram_alloc_failures == 0))
                g_all = 0;
        }
    }
    E.init_experts(Config());  // release every device allocation before the backend goes away
    printf("done %d\n", g_all);
    return 0;
}
