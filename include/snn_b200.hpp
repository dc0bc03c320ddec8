// snn_b200.hpp - header-only C++ host API over the C ABI (snn_b200.h), with
// the names, argument meanings and error behaviour of the reference's host
// classes, so that a caller of the reference can switch with minimal edits:
//
//   snnb::stage2e::BioMechanismScheduler  <- stage2e::BioMechanismScheduler
//       (src/stage2e/scheduler.cuh:66-224) together with MemoryAllocator +
//       init_network (src/stage2e/memory_allocator.cuh:306-339,
//       src/stage2e/network_init.cuh:42) and load_text_corpus
//       (src/stage2e/input_encoding.cuh:35-50)
//   snnb::SNNNetwork                      <- SNNNetwork (src/include/network.h:11-95)
//
// Differences, by design: device memory belongs to the object (no raw device
// pointers are handed out; snn_get_state copies fields to host buffers), and
// failures throw snnb::SnnException carrying the SNN_ERR_* code instead of
// calling exit().
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>
#include "snn_b200.h"

namespace snnb {

struct SnnException : std::runtime_error {
    int code;
    SnnException(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

namespace detail {
inline void check(int rc, const snn_ctx* ctx, const char* what) {
    if (rc != SNN_OK)
        throw SnnException(rc, std::string(what) + ": " + snn_last_error(ctx));
}
struct Handle {
    snn_ctx* ctx = nullptr;
    Handle(int32_t model, int32_t preset, int32_t device, int32_t e0) {
        snn_config cfg;
        check(snn_config_init(&cfg, model, preset), nullptr, "snn_config_init");
        cfg.device = device;
        cfg.e0 = e0;
        check(snn_create(&cfg, &ctx), nullptr, "snn_create");
    }
    ~Handle() { snn_destroy(ctx); }
    Handle(const Handle&) = delete;
    Handle& operator=(const Handle&) = delete;
};
}  // namespace detail

namespace stage2e {

// Reference-shaped Stage 2e scheduler: construct (allocates + builds the
// network, like MemoryAllocator::allocate_all + init_network), optionally
// load a corpus, then call step(t) with t = 0, 1, 2, ...
class BioMechanismScheduler {
public:
    explicit BioMechanismScheduler(int32_t n_columns = 50, int32_t device = 0,
                                   int32_t preset = SNN_PRESET_REF)
        : h_(SNN_MODEL_STAGE2E, preset, device, 0) {
        snn_topology_spec spec;
        detail::check(snn_topology_init(&spec, SNN_MODEL_STAGE2E, n_columns), h_.ctx,
                      "snn_topology_init");
        detail::check(snn_build_columns(h_.ctx, &spec), h_.ctx, "snn_build_columns");
    }

    // E0 ablation (src/stage2e/scheduler.cuh:72, synapse_kernels.cuh:82)
    void set_e0_ablation(bool enable) { detail::check(snn_set_e0(h_.ctx, enable), h_.ctx, "snn_set_e0"); }

    // load_text_corpus (src/stage2e/input_encoding.cu:40-96): the reference's
    // filter is applied by the C ABI; returns the number of bytes kept
    size_t load_text_corpus(const std::vector<uint8_t>& bytes) {
        int64_t kept = 0;
        detail::check(snn_set_corpus_ex(h_.ctx, bytes.data(), (int64_t)bytes.size(),
                                        SNN_CORPUS_TEXT_FILTER, &kept),
                      h_.ctx, "snn_set_corpus_ex");
        return (size_t)kept;
    }
    // the same from a file path, as the reference's load_text_corpus(const char*)
    size_t load_text_corpus(const char* path) {
        int64_t kept = 0;
        detail::check(snn_load_text_corpus(h_.ctx, path, &kept), h_.ctx, "snn_load_text_corpus");
        return (size_t)kept;
    }

    void step(int current_step) { detail::check(snn_step(h_.ctx, current_step, -1, 1), h_.ctx, "snn_step"); }

    // many steps without host synchronisation between them
    void run(int n_steps) {
        detail::check(snn_run(h_.ctx, n_steps, nullptr, 0, 1, nullptr, nullptr), h_.ctx, "snn_run");
    }

    snn_counters counters() const {
        snn_counters c;
        detail::check(snn_get_counters(h_.ctx, &c), h_.ctx, "snn_get_counters");
        return c;
    }
    int total_steps_executed() const { return (int)counters().step; }
    long long total_spikes_accum() const { return counters().total_spikes; }
    long long arrived_events_accum() const { return counters().arrivals; }
    long long dispatched_events_accum() const { return counters().dispatched; }
    long long dropped_events_accum() const { return counters().dropped_ref; }
    int total_single_neuron_burst_spikes() const { return (int)counters().burst_spikes; }
    // run_semantic_eval (src/stage2e/scheduler.cuh:126): the result instead
    // of the reference's cached members (p3_silhouette_score_, ...)
    snn_semantic run_semantic_eval(int step) const {
        snn_semantic r;
        detail::check(snn_semantic_eval(h_.ctx, step, &r, nullptr, 0), h_.ctx, "snn_semantic_eval");
        return r;
    }

    template <typename T>
    std::vector<T> state(int32_t which, size_t n) const {
        std::vector<T> v(n);
        detail::check(snn_get_state(h_.ctx, which, v.data(), (int64_t)(n * sizeof(T))), h_.ctx,
                      "snn_get_state");
        return v;
    }

    // save_checkpoint (src/stage2e/scheduler.cu:411-483); returns 0 on success
    int save_checkpoint(int step, const char* dir = "checkpoints") {
        std::string path = std::string(dir) + "/ckpt_step" + std::to_string(step) + ".bin";
        return snn_save(h_.ctx, path.c_str(), SNN_FMT_SCKP_V2) == SNN_OK ? 0 : 2;
    }

    snn_ctx* handle() { return h_.ctx; }

private:
    detail::Handle h_;
};

}  // namespace stage2e

// Reference-shaped Stage 0 / Stage 2 network (src/include/network.h:11-95).
class SNNNetwork {
public:
    explicit SNNNetwork(unsigned seed = 42, int32_t n_columns = 0, int32_t device = 0,
                        int32_t preset = SNN_PRESET_BASELINE)
        : h_(SNN_MODEL_STAGE0, preset, device, 0), seed_(seed), ncol_(n_columns) {}

    void initialize() {
        snn_topology_spec spec;
        detail::check(snn_topology_init(&spec, SNN_MODEL_STAGE0, ncol_), h_.ctx, "snn_topology_init");
        spec.seed = seed_;
        detail::check(snn_build_columns(h_.ctx, &spec), h_.ctx, "snn_build_columns");
        snn_counters c;
        detail::check(snn_get_counters(h_.ctx, &c), h_.ctx, "snn_get_counters");
        n_ = (int)c.n_neurons;
    }

    // one step; byte >= 0 drives the one-hot input (the reference passes the
    // one-hot host vector instead), -1 = no input
    void step(int byte, int time_step) { detail::check(snn_step(h_.ctx, time_step, byte, 1), h_.ctx, "snn_step"); }
    void set_dopamine(float level) { detail::check(snn_set_dopamine(h_.ctx, level), h_.ctx, "snn_set_dopamine"); }
    void save_weights(const std::string& path) const {
        detail::check(snn_save(h_.ctx, path.c_str(), SNN_FMT_RAW_F32), h_.ctx, "snn_save");
    }
    void load_weights(const std::string& path) {
        detail::check(snn_load(h_.ctx, path.c_str(), SNN_FMT_RAW_F32), h_.ctx, "snn_load");
    }
    int n_neurons() const { return n_; }
    snn_ctx* handle() { return h_.ctx; }

private:
    detail::Handle h_;
    unsigned seed_;
    int32_t ncol_;
    int n_ = 0;
};

}  // namespace snnb
