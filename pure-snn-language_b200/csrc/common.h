// common.h - internal helpers shared by the engines (not part of the C ABI).
#pragma once
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include "snn_b200.h"

namespace snnb {

// Internal error type; converted to an SNN_ERR_* code at the C boundary.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define SNN_CUDA(call)                                                            \
    do {                                                                          \
        cudaError_t e_ = (call);                                                  \
        if (e_ != cudaSuccess)                                                    \
            throw ::snnb::Error(e_ == cudaErrorMemoryAllocation ? SNN_ERR_OOM     \
                                                                 : SNN_ERR_CUDA,  \
                                std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

#define SNN_REQUIRE(cond, code, msg)                 \
    do {                                             \
        if (!(cond)) throw ::snnb::Error(code, msg); \
    } while (0)

// The reference's text-corpus filter (src/stage2e/input_encoding.cu:49-64,
// src/stage2/text_stream.cu:38-52): NUL dropped, CR / LF / TAB mapped to a
// space, every other byte kept.  Writes the kept bytes to out (which may be
// `in` itself) and returns their count.
inline int64_t text_filter(const uint8_t* in, int64_t n, uint8_t* out) {
    int64_t k = 0;
    for (int64_t i = 0; i < n; ++i) {
        const uint8_t c = in[i];
        if (c == 0x00) continue;
        out[k++] = (c == '\r' || c == '\n' || c == '\t') ? (uint8_t)' ' : c;
    }
    return k;
}

// Owning device allocation.
template <typename T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    void alloc(size_t count) {
        release();
        if (count == 0) count = 1;
        SNN_CUDA(cudaMalloc((void**)&p, count * sizeof(T)));
        n = count;
    }
    void zero(cudaStream_t s = 0) { SNN_CUDA(cudaMemsetAsync(p, 0, n * sizeof(T), s)); }
    void upload(const T* h, size_t count, cudaStream_t s = 0) {
        SNN_REQUIRE(count <= n, SNN_ERR_ARG, "upload larger than buffer");
        SNN_CUDA(cudaMemcpyAsync(p, h, count * sizeof(T), cudaMemcpyHostToDevice, s));
    }
    void download(T* h, size_t count, cudaStream_t s = 0) const {
        SNN_REQUIRE(count <= n, SNN_ERR_ARG, "download larger than buffer");
        SNN_CUDA(cudaMemcpyAsync(h, p, count * sizeof(T), cudaMemcpyDeviceToHost, s));
    }
    size_t bytes() const { return n * sizeof(T); }
};

// Abstract engine behind one snn_ctx.
struct Engine {
    virtual ~Engine() {}
    virtual void build(const snn_topology_spec& spec) = 0;
    virtual void set_corpus(const uint8_t* b, int64_t n) = 0;
    // n steps; byte_override >= 0 forces the byte of the first step's
    // injection (single-step API); learn = 0 freezes plasticity.
    virtual void run(int32_t n_steps, int32_t byte_override, int32_t learn, uint32_t* raster,
                     int32_t* counts) = 0;
    virtual void get_state(int32_t which, void* buf, int64_t nbytes) = 0;
    virtual void counters(snn_counters* c) = 0;
    virtual void get_spikes(uint32_t* words, int64_t n_words) = 0;
    virtual void set_dopamine(float) { throw Error(SNN_ERR_UNSUPPORTED, "no dopamine control in this model"); }
    virtual void set_e0(int32_t) { throw Error(SNN_ERR_UNSUPPORTED, "no E0 ablation in this model"); }
    // column sharding over `world` ranks (one per GPU); uid = ncclUniqueId
    virtual void set_shard(int32_t, int32_t, const void*) {
        throw Error(SNN_ERR_UNSUPPORTED, "this model does not shard");
    }
    virtual void save(const char* path, int32_t fmt) = 0;
    virtual void load(const char* path, int32_t fmt) = 0;
    virtual int64_t steps_done() const = 0;
    virtual void set_profiling(int32_t) { throw Error(SNN_ERR_UNSUPPORTED, "profiling not available"); }
    virtual void get_profile(snn_profile*) { throw Error(SNN_ERR_UNSUPPORTED, "profiling not available"); }
    virtual void sync() = 0;
    virtual void semantic_eval(int64_t, snn_semantic*, int32_t*, int64_t) {
        throw Error(SNN_ERR_UNSUPPORTED, "semantic evaluation exists for the Stage 2e network only");
    }
};

Engine* make_engine_stage2e(const snn_config& cfg);
Engine* make_engine_stage0(const snn_config& cfg);
Engine* make_engine_prop(const snn_config& cfg);
void propagate(const int32_t* post, const float* w, int64_t n_pre, int32_t fanout, const uint8_t* spikes,
               int32_t* acc, int64_t n_post, int32_t frac_bits, cudaStream_t stream);
void propagate_static(const int32_t* post, const float* w, int64_t n_pre, int32_t fanout,
                      const uint8_t* spikes, int32_t* acc, int64_t n_post, int32_t frac_bits,
                      cudaStream_t stream);

}  // namespace snnb
