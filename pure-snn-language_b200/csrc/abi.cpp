// abi.cpp - extern "C" boundary: handle management, error codes, dispatch to
// the engines.  No exception crosses this boundary and nothing calls exit().
#include <cstdio>
#include <memory>
#include <string>
#include <nccl.h>
#include "nccl_dl.h"
#include "common.h"
#include "net2e.h"

struct snn_ctx {
    snn_config cfg;
    std::unique_ptr<snnb::Engine> eng;
    std::string err;
};

namespace {
thread_local std::string g_create_err;

template <typename F>
int guard(snn_ctx* ctx, F&& f) {
    if (!ctx) return SNN_ERR_ARG;
    try {
        f();
        ctx->err.clear();
        return SNN_OK;
    } catch (const snnb::Error& e) {
        ctx->err = e.what();
        return e.code;
    } catch (const std::bad_alloc&) {
        ctx->err = "host allocation failed";
        return SNN_ERR_OOM;
    } catch (const std::exception& e) {
        ctx->err = e.what();
        return SNN_ERR_STATE;
    }
}

snn_topology_spec reference_columns(int32_t n_columns) {
    snn_topology_spec s;
    memset(&s, 0, sizeof(s));
    s.n_columns = n_columns;
    s.l4 = 200; s.l23 = 350; s.l5 = 200; s.l6 = 250;
    s.pf_groups = n_columns; s.pf_group_size = 100;
    s.deg_intra = 150; s.deg_inter = 30; s.deg_l5_pf = 15;
    s.deg_pf_self = 100; s.deg_pf_assoc = 50;
    s.total_synapses = (int64_t)10700000 * n_columns / 50;
    s.seed = 42;
    s.rule = 0;
    return s;
}
}  // namespace

extern "C" {

const char* snn_version(void) { return "snn_b200 0.1 (sm_100a)"; }

int snn_config_init(snn_config* cfg, int32_t model, int32_t preset) {
    if (!cfg) return SNN_ERR_ARG;
    if (model != SNN_MODEL_STAGE2E && model != SNN_MODEL_STAGE0 && model != SNN_MODEL_PROP)
        return SNN_ERR_ARG;
    if (preset != SNN_PRESET_REF && preset != SNN_PRESET_BASELINE) return SNN_ERR_ARG;
    memset(cfg, 0, sizeof(*cfg));
    cfg->model = model;
    cfg->preset = preset;
    cfg->raster_steps = 1024;
    if (model == SNN_MODEL_PROP) cfg->prop_rate = 0.01f;
    return SNN_OK;
}

int snn_topology_init(snn_topology_spec* spec, int32_t model, int32_t n_columns) {
    if (!spec) return SNN_ERR_ARG;
    if (model == SNN_MODEL_STAGE2E) {
        if (n_columns < 2) return SNN_ERR_ARG;
        *spec = reference_columns(n_columns);
        return SNN_OK;
    }
    if (model == SNN_MODEL_STAGE0) {
        memset(spec, 0, sizeof(*spec));
        spec->n_columns = n_columns;  // 0 = Stage 0 single block
        if (n_columns == 0) {  // Stage 0: 100 out-edges anywhere
            spec->l4 = 2000; spec->l23 = 6000; spec->l5 = 2000;
            spec->deg_intra = 100;
        } else {               // Stage 2 columns: 80 intra + 20 inter out-edges
            spec->l4 = 200; spec->l23 = 600; spec->l5 = 200;
            spec->deg_intra = 80;
            spec->deg_inter = 20;
        }
        spec->seed = 42;
        spec->rule = 1;
        return SNN_OK;
    }
    if (model == SNN_MODEL_PROP) {  // n_columns unused: 1M neurons, fan-out 1000
        memset(spec, 0, sizeof(*spec));
        spec->l4 = 1000000;
        spec->deg_intra = 1000;
        spec->seed = 42;
        spec->rule = 1;
        return SNN_OK;
    }
    return SNN_ERR_ARG;
}

int snn_create(const snn_config* cfg, snn_ctx** out) {
    if (!cfg || !out) return SNN_ERR_ARG;
    *out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return SNN_ERR_NO_DEVICE;
    }
    if (cfg->device < 0 || cfg->device >= ndev) return SNN_ERR_ARG;
    snn_ctx* ctx = new (std::nothrow) snn_ctx();
    if (!ctx) return SNN_ERR_OOM;
    ctx->cfg = *cfg;
    int rc = guard(ctx, [&] {
        if (cfg->model == SNN_MODEL_STAGE2E) ctx->eng.reset(snnb::make_engine_stage2e(*cfg));
        else if (cfg->model == SNN_MODEL_STAGE0) ctx->eng.reset(snnb::make_engine_stage0(*cfg));
        else if (cfg->model == SNN_MODEL_PROP) ctx->eng.reset(snnb::make_engine_prop(*cfg));
        else throw snnb::Error(SNN_ERR_ARG, "unknown model");
    });
    if (rc != SNN_OK) {
        g_create_err = ctx->err;
        delete ctx;
        return rc;
    }
    *out = ctx;
    return SNN_OK;
}

void snn_destroy(snn_ctx* ctx) { delete ctx; }

const char* snn_last_error(const snn_ctx* ctx) {
    return ctx ? ctx->err.c_str() : g_create_err.c_str();
}

int snn_build_columns(snn_ctx* ctx, const snn_topology_spec* spec) {
    return guard(ctx, [&] {
        SNN_REQUIRE(spec, SNN_ERR_ARG, "null topology");
        ctx->eng->build(*spec);
    });
}

int snn_set_corpus(snn_ctx* ctx, const uint8_t* bytes, int64_t n) {
    return guard(ctx, [&] { ctx->eng->set_corpus(bytes, n); });
}

int snn_set_corpus_ex(snn_ctx* ctx, const uint8_t* bytes, int64_t n, int32_t flags,
                      int64_t* n_kept) {
    return guard(ctx, [&] {
        SNN_REQUIRE(n >= 0 && (n == 0 || bytes), SNN_ERR_ARG, "bad corpus");
        SNN_REQUIRE((flags & ~SNN_CORPUS_TEXT_FILTER) == 0, SNN_ERR_ARG, "unknown corpus flags");
        if (!(flags & SNN_CORPUS_TEXT_FILTER)) {
            ctx->eng->set_corpus(bytes, n);
            if (n_kept) *n_kept = n;
            return;
        }
        std::vector<uint8_t> kept((size_t)n);
        const int64_t k = snnb::text_filter(bytes, n, kept.data());
        ctx->eng->set_corpus(kept.data(), k);
        if (n_kept) *n_kept = k;
    });
}

int snn_load_text_corpus(snn_ctx* ctx, const char* path, int64_t* n_kept) {
    return guard(ctx, [&] {
        SNN_REQUIRE(path, SNN_ERR_ARG, "null path");
        FILE* f = fopen(path, "rb");
        SNN_REQUIRE(f, SNN_ERR_IO, std::string("cannot open ") + path);
        std::vector<uint8_t> raw;
        uint8_t buf[1 << 16];
        size_t got;
        while ((got = fread(buf, 1, sizeof(buf), f)) > 0) raw.insert(raw.end(), buf, buf + got);
        const bool bad = ferror(f) != 0;
        fclose(f);
        SNN_REQUIRE(!bad, SNN_ERR_IO, std::string("read error on ") + path);
        const int64_t k = snnb::text_filter(raw.data(), (int64_t)raw.size(), raw.data());
        SNN_REQUIRE(k > 0, SNN_ERR_IO, std::string("no text left in ") + path);
        ctx->eng->set_corpus(raw.data(), k);
        if (n_kept) *n_kept = k;
    });
}

int snn_byte_classes(const uint8_t* bytes, int64_t n, int64_t* out, int32_t n_out) {
    if ((n > 0 && !bytes) || n < 0 || !out || n_out < 3) return SNN_ERR_ARG;
    int64_t a = 0, h = 0, c = 0;
    for (int64_t i = 0; i < n; ++i) {
        const uint8_t b = bytes[i];
        if (b < 0x80) ++a;
        else if (b < 0xC0) ++c;
        else if (b < 0xF8) ++h;
    }
    out[0] = a;
    out[1] = h;
    out[2] = c;
    return SNN_OK;
}

int snn_step(snn_ctx* ctx, int32_t step, int32_t inject_byte, int32_t learn) {
    return guard(ctx, [&] {
        SNN_REQUIRE(step == ctx->eng->steps_done(), SNN_ERR_STATE,
                    "step index must equal the number of executed steps");
        SNN_REQUIRE(inject_byte >= -1 && inject_byte < 256, SNN_ERR_ARG, "inject_byte out of range");
        ctx->eng->run(1, inject_byte, learn, nullptr, nullptr);
    });
}

int snn_run(snn_ctx* ctx, int32_t n_steps, const uint8_t* bytes, int64_t n_bytes, int32_t learn,
            uint32_t* raster_out, int32_t* counts_out) {
    return guard(ctx, [&] {
        SNN_REQUIRE(n_steps >= 0, SNN_ERR_ARG, "negative step count");
        if (bytes) ctx->eng->set_corpus(bytes, n_bytes);
        ctx->eng->run(n_steps, -1, learn, raster_out, counts_out);
    });
}

int snn_synchronize(snn_ctx* ctx) {
    return guard(ctx, [&] { ctx->eng->sync(); });
}

int snn_get_spikes(snn_ctx* ctx, uint32_t* bitmask, int64_t n_words) {
    return guard(ctx, [&] {
        SNN_REQUIRE(bitmask, SNN_ERR_ARG, "null buffer");
        ctx->eng->get_spikes(bitmask, n_words);
    });
}

int snn_get_state(snn_ctx* ctx, int32_t which, void* host_buf, int64_t n_bytes) {
    return guard(ctx, [&] {
        SNN_REQUIRE(host_buf, SNN_ERR_ARG, "null buffer");
        ctx->eng->get_state(which, host_buf, n_bytes);
    });
}

int snn_get_counters(snn_ctx* ctx, snn_counters* out) {
    return guard(ctx, [&] {
        SNN_REQUIRE(out, SNN_ERR_ARG, "null counters");
        ctx->eng->counters(out);
        if (out->local_hi == 0) out->local_hi = out->n_neurons;  // unsharded: all neurons
    });
}

int snn_semantic_eval(snn_ctx* ctx, int64_t step, snn_semantic* out, int32_t* assign, int64_t n_assign) {
    return guard(ctx, [&] {
        SNN_REQUIRE(out, SNN_ERR_ARG, "null result");
        ctx->eng->semantic_eval(step, out, assign, n_assign);
    });
}

int snn_set_dopamine(snn_ctx* ctx, float level) {
    return guard(ctx, [&] { ctx->eng->set_dopamine(level); });
}

int snn_set_e0(snn_ctx* ctx, int32_t enable) {
    return guard(ctx, [&] { ctx->eng->set_e0(enable); });
}

int snn_set_profiling(snn_ctx* ctx, int32_t enable) {
    return guard(ctx, [&] { ctx->eng->set_profiling(enable); });
}

int snn_get_profile(snn_ctx* ctx, snn_profile* out) {
    return guard(ctx, [&] {
        SNN_REQUIRE(out, SNN_ERR_ARG, "null profile");
        ctx->eng->get_profile(out);
    });
}

int snn_save(snn_ctx* ctx, const char* path, int32_t fmt) {
    return guard(ctx, [&] {
        SNN_REQUIRE(path, SNN_ERR_ARG, "null path");
        ctx->eng->save(path, fmt);
    });
}

int snn_load(snn_ctx* ctx, const char* path, int32_t fmt) {
    return guard(ctx, [&] {
        SNN_REQUIRE(path, SNN_ERR_ARG, "null path");
        ctx->eng->load(path, fmt);
    });
}

int snn_nccl_unique_id(uint8_t* out, int64_t n) {
    if (!out || n < (int64_t)sizeof(ncclUniqueId)) return SNN_ERR_ARG;
    try {
        const snnb::NcclApi& nc = snnb::nccl();
        ncclUniqueId id;
        const ncclResult_t r = nc.GetUniqueId(&id);
        if (r != ncclSuccess) {
            g_create_err = std::string("ncclGetUniqueId: ") + nc.GetErrorString(r);
            return SNN_ERR_CUDA;
        }
        memcpy(out, &id, sizeof(id));
        return SNN_OK;
    } catch (const snnb::Error& e) {
        g_create_err = e.what();
        return e.code;
    }
}

int snn_set_shard(snn_ctx* ctx, int32_t rank, int32_t world, const uint8_t* uid, int64_t n) {
    return guard(ctx, [&] {
        // Stage 2e needs the id for world > 1 (checked by its engine); the
        // microbench's post-bucket shards exchange nothing and take none
        SNN_REQUIRE(!uid || n >= (int64_t)sizeof(ncclUniqueId), SNN_ERR_ARG,
                    "an NCCL unique id is 128 bytes");
        ctx->eng->set_shard(rank, world, uid);
    });
}

int snn_shard_plan(const snn_topology_spec* spec, int32_t rank, int32_t world, int64_t* out,
                   int32_t n_out) {
    if (!spec || !out || n_out < 10) return SNN_ERR_ARG;
    try {
        const snn2e::Shard sh = snn2e::make_shard(*spec, rank, world);
        snn2e::HostNet net;
        snn2e::generate_reference(*spec, net, &sh);
        snn2e::Layout lay;
        snn2e::build_layout(net, lay);
        int64_t g_local = 0, g_mirror = 0, m = 0, remote_syn = 0, remote_short = 0;
        for (int gi = 0; gi < net.N; ++gi) {
            const int64_t ng = lay.gbeg[gi + 1] - lay.gbeg[gi];
            if (sh.owns(gi)) g_local += ng;
            else if (ng > 0) { g_mirror += ng; ++m; }
            if (sh.owns(gi)) continue;
            for (int32_t sid = net.row_ptr[gi]; sid < net.row_ptr[gi + 1]; ++sid) {
                ++remote_syn;
                if (snn2e::eff_delay(net.delay[sid]) < 5) ++remote_short;
            }
        }
        const int64_t vals[10] = {sh.n_local(), sh.a0, sh.a1, sh.pf0, sh.pf1, net.S,
                                  g_local, g_mirror, m, remote_short};
        (void)remote_syn;
        for (int q = 0; q < 10; ++q) out[q] = vals[q];
        return SNN_OK;
    } catch (const snnb::Error& e) {
        g_create_err = e.what();
        return e.code;
    } catch (const std::exception& e) {
        g_create_err = e.what();
        return SNN_ERR_STATE;
    }
}

int snn_propagate(const int32_t* post, const float* w, int64_t n_pre, int32_t fanout,
                  const uint8_t* spikes, int32_t* acc, int64_t n_post, int32_t frac_bits,
                  void* stream) {
    try {
        snnb::propagate(post, w, n_pre, fanout, spikes, acc, n_post, frac_bits, (cudaStream_t)stream);
        g_create_err.clear();
        return SNN_OK;
    } catch (const snnb::Error& e) {
        g_create_err = e.what();
        return e.code;
    } catch (const std::exception& e) {
        g_create_err = e.what();
        return SNN_ERR_STATE;
    }
}

int snn_propagate_static(const int32_t* post, const float* w, int64_t n_pre, int32_t fanout,
                         const uint8_t* spikes, int32_t* acc, int64_t n_post, int32_t frac_bits,
                         void* stream) {
    try {
        snnb::propagate_static(post, w, n_pre, fanout, spikes, acc, n_post, frac_bits,
                               (cudaStream_t)stream);
        g_create_err.clear();
        return SNN_OK;
    } catch (const snnb::Error& e) {
        g_create_err = e.what();
        return e.code;
    } catch (const std::exception& e) {
        g_create_err = e.what();
        return SNN_ERR_STATE;
    }
}

}  // extern "C"
