// oracle4.cpp - CPU oracle of the propagation microbench (SNN_MODEL_PROP).
//
// TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and the CPU
// baseline leg of the benchmark call this; the product never does.
//
// The reference has no propagation microbench, so this oracle is the
// definition of the model (include/snn_prop_rules.h and the step comment in
// include/snn_b200.h).  Its pieces follow the reference where it has them:
// the LIF update is Stage 0's (src/cuda/neuron_kernel.cu:52-114, threshold
// without homeostasis), the pair-STDP window is Stage 0's A = 0.05, tau = 20
// with dw computed before the timestamp update (src/cuda/stdp_kernel.cu:29-88),
// and propagation is the event form of synaptic_transmission_kernel
// (src/cuda/synapse_kernel.cu:28-47) with exact fixed-point sums.
// "Parity unpinned" against the reference for this model: there is nothing
// in the reference to pin it to; it is pinned by its own closed forms in the
// tests (exact integer sums, round-trip properties).
#include <cstdint>
#include <cstring>
#include <vector>
#include <atomic>
#include <omp.h>
#include "snn_prop_rules.h"

namespace {

struct O4Params {
    int32_t n;          // neurons
    int32_t fanout;     // out-edges per neuron
    uint32_t seed;
    int32_t mode;       // bit 0 STDP, bit 1 STP
    float rate;
    float w_max;
    float dopamine;
    int32_t n_threads;
};

struct O4 {
    O4Params P;
    int64_t S;
    int32_t n_exc;
    uint32_t thr;
    uint64_t key;
    std::vector<int32_t> post;
    std::vector<float> w;
    std::vector<int64_t> in_ptr;   // reverse CSR (STDP only)
    std::vector<uint32_t> in_syn;  // ascending synapse ids per post
    std::vector<int32_t> acc;
    std::vector<float> V, I, u, R;
    std::vector<int8_t> ref;
    std::vector<int32_t> last_post, last_pre;
    std::vector<uint8_t> spike;    // LIF spikes of the last step
    std::vector<float> exp_tab;
    int64_t step = 0, total_spikes = 0, events = 0, pre_spikes = 0, ltp_visits = 0;
    int32_t last_spikes = 0;
};

inline float e20(const O4& o, int32_t dt) { return dt <= SNN_PROP_EXP_STEPS ? o.exp_tab[dt] : 0.0f; }

void build(O4& o) {
    const int32_t N = o.P.n, F = o.P.fanout;
    o.S = (int64_t)N * F;
    o.n_exc = (int32_t)(((int64_t)N * 4) / 5);
    double t = (double)o.P.rate * 4294967296.0;
    o.thr = t >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)t;
    o.key = snn_prop_spike_key(o.P.seed);
    o.post.resize(o.S);
    o.w.resize(o.S);
#pragma omp parallel for schedule(static)
    for (int64_t s = 0; s < o.S; ++s) {
        uint64_t h = snn_prop_syn_hash(o.P.seed, (uint64_t)s);
        o.post[s] = snn_prop_post(h, (uint32_t)N);
        o.w[s] = snn_prop_weight(h, o.P.w_max, (s / F) < o.n_exc);
    }
    if (o.P.mode & 1) {
        // reverse CSR by a parallel counting sort: thread k counts, then
        // fills, the synapses of its own range [lo_k, hi_k), so every post's
        // list comes out in ascending synapse order
        const int nt = omp_get_max_threads();
        std::vector<std::vector<int64_t>> cnt(nt);
#pragma omp parallel num_threads(nt)
        {
            const int k = omp_get_thread_num();
            const int64_t lo = o.S * k / nt, hi = o.S * (k + 1) / nt;
            cnt[k].assign((size_t)N, 0);
            for (int64_t s = lo; s < hi; ++s) cnt[k][o.post[s]]++;
        }
        o.in_ptr.assign((size_t)N + 1, 0);
        int64_t run = 0;
        for (int32_t j = 0; j < N; ++j) {
            o.in_ptr[j] = run;
            for (int k = 0; k < nt; ++k) {
                const int64_t c = cnt[k][j];
                cnt[k][j] = run;  // becomes thread k's cursor for post j
                run += c;
            }
        }
        o.in_ptr[N] = run;
        o.in_syn.resize(o.S);
#pragma omp parallel num_threads(nt)
        {
            const int k = omp_get_thread_num();
            const int64_t lo = o.S * k / nt, hi = o.S * (k + 1) / nt;
            for (int64_t s = lo; s < hi; ++s) o.in_syn[cnt[k][o.post[s]]++] = (uint32_t)s;
        }
    }
    o.acc.assign(N, 0);
    o.V.assign(N, 0.0f);
    o.I.assign(N, 0.0f);
    o.u.assign(N, SNN_PROP_STP_U);
    o.R.assign(N, 1.0f);
    o.ref.assign(N, 0);
    o.last_post.assign(N, -1);
    o.last_pre.assign(N, -1);
    o.spike.assign(N, 0);
    o.exp_tab.resize(SNN_PROP_EXP_STEPS + 1);
    for (int k = 0; k <= SNN_PROP_EXP_STEPS; ++k)
        o.exp_tab[k] = snn_expf(pm_div(-pm_i2f(k), 20.0f));
}

void step(O4& o, uint32_t* raster_row) {
    const int32_t N = o.P.n, F = o.P.fanout, t = (int32_t)o.step;
    const bool stdp = o.P.mode & 1, stp = o.P.mode & 2;
    const float lr = pm_mul(o.P.dopamine, o.P.w_max);
    // 1. forced pre-spikes (+ STP release)
    std::vector<int32_t> pre;
    std::vector<float> rel;
    {
        const int nt = omp_get_max_threads();
        std::vector<std::vector<int32_t>> tp(nt);
        std::vector<std::vector<float>> tr(nt);
#pragma omp parallel
        {
            const int me = omp_get_thread_num(), cnt = omp_get_num_threads();
            const int32_t lo = (int32_t)((int64_t)N * me / cnt), hi = (int32_t)((int64_t)N * (me + 1) / cnt);
            for (int32_t i = lo; i < hi; ++i) {
                if (!snn_prop_spikes(o.key, t, (uint32_t)i, o.thr)) continue;
                float r = 1.0f;
                if (stp) r = snn_prop_stp(&o.u[i], &o.R[i], o.last_pre[i] >= 0 ? t - o.last_pre[i] : -1);
                tp[me].push_back(i);
                tr[me].push_back(r);
            }
        }
        for (int k = 0; k < nt; ++k) {
            pre.insert(pre.end(), tp[k].begin(), tp[k].end());
            rel.insert(rel.end(), tr[k].begin(), tr[k].end());
        }
    }
    const int64_t np = (int64_t)pre.size();
    // 2. push (+ LTD on excitatory out-synapses)
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t e = 0; e < np; ++e) {
        const int32_t i = pre[e];
        const int64_t b = (int64_t)i * F;
        const bool plastic = stdp && i < o.n_exc;
        for (int32_t k = 0; k < F; ++k) {
            const int32_t q = o.post[b + k];
            const int32_t add = snn_prop_quant(o.w[b + k], rel[e], stp);
#pragma omp atomic
            o.acc[q] += add;
            if (plastic && o.last_post[q] >= 0) {
                float dw = pm_mul(-0.05f, e20(o, t - o.last_post[q]));
                float x = pm_fma(lr, dw, o.w[b + k]);
                o.w[b + k] = pm_min(pm_max(x, 0.0f), o.P.w_max);
            }
        }
    }
    // 3. LIF (Stage 0 form)
    int32_t nsp = 0;
#pragma omp parallel for schedule(static) reduction(+ : nsp)
    for (int32_t j = 0; j < N; ++j) {
        const float in = pm_mul(pm_i2f(o.acc[j]), 5.9604644775390625e-8f);
        o.acc[j] = 0;
        if (o.ref[j] > 0) {
            o.ref[j]--;
            o.spike[j] = 0;
            o.V[j] = pm_mul(o.V[j], 0.95f);
            continue;
        }
        o.I[j] = pm_fma(o.I[j], 0.95f, in);
        float v = pm_fma(o.V[j], 0.95f, o.I[j]);
        if (v < 0.0f) v = 0.0f;
        const bool sp = v >= 1.0f;
        if (sp) { v = 0.0f; o.ref[j] = 2; o.last_post[j] = t; nsp++; }
        o.spike[j] = sp;
        o.V[j] = v;
    }
    // 4. LTP over the incoming excitatory synapses of LIF spikes
    int64_t visits = 0;
    if (stdp) {
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : visits)
        for (int32_t j = 0; j < N; ++j) {
            if (!o.spike[j]) continue;
            visits += o.in_ptr[j + 1] - o.in_ptr[j];
            for (int64_t x = o.in_ptr[j]; x < o.in_ptr[j + 1]; ++x) {
                const int64_t s = (int64_t)o.in_syn[x];
                const int32_t p = (int32_t)(s / F);
                if (p >= o.n_exc || o.last_pre[p] < 0) continue;
                float dw = pm_mul(0.05f, e20(o, t - o.last_pre[p]));
                float y = pm_fma(lr, dw, o.w[s]);
                o.w[s] = pm_min(pm_max(y, 0.0f), o.P.w_max);
            }
        }
    }
    for (int64_t e = 0; e < np; ++e) o.last_pre[pre[e]] = t;
    if (raster_row) {
        memset(raster_row, 0, sizeof(uint32_t) * (size_t)((N + 31) / 32));
        for (int32_t j = 0; j < N; ++j)
            if (o.spike[j]) raster_row[j >> 5] |= 1u << (j & 31);
    }
    o.total_spikes += nsp;
    o.last_spikes = nsp;
    o.pre_spikes += np;
    o.events += np * F;
    o.ltp_visits += visits;
    o.step++;
}

}  // namespace

extern "C" {

struct O4Counters {
    int64_t step, total_spikes, events, pre_spikes, ltp_visits;
    int32_t last_spikes, n_exc;
    int64_t n_synapses;
};

void* o4_create(const O4Params* p) {
    O4* o = new O4();
    o->P = *p;
    if (o->P.n_threads > 0) omp_set_num_threads(o->P.n_threads);
    build(*o);
    return o;
}

void o4_destroy(void* h) { delete (O4*)h; }

void o4_set_dopamine(void* h, float da) { ((O4*)h)->P.dopamine = da; }

// n steps; raster (nullable) receives n rows of ceil(N/32) words
void o4_run(void* h, int32_t n, uint32_t* raster) {
    O4& o = *(O4*)h;
    const int64_t words = (o.P.n + 31) / 32;
    for (int32_t k = 0; k < n; ++k) step(o, raster ? raster + k * words : nullptr);
}

void o4_counters(void* h, O4Counters* c) {
    O4& o = *(O4*)h;
    c->step = o.step; c->total_spikes = o.total_spikes; c->events = o.events;
    c->pre_spikes = o.pre_spikes; c->ltp_visits = o.ltp_visits;
    c->last_spikes = o.last_spikes; c->n_exc = o.n_exc; c->n_synapses = o.S;
}

// which: 0 V, 1 I, 2 u, 3 R (f32[N]); 4 w (f32[S]); 5 post (i32[S]);
// 6 ref (i8 widened to i32[N]); 7 last_post (i32[N]); 8 last_pre (i32[N])
void o4_get(void* h, int32_t which, void* out) {
    O4& o = *(O4*)h;
    const size_t N = (size_t)o.P.n;
    switch (which) {
        case 0: memcpy(out, o.V.data(), N * 4); break;
        case 1: memcpy(out, o.I.data(), N * 4); break;
        case 2: memcpy(out, o.u.data(), N * 4); break;
        case 3: memcpy(out, o.R.data(), N * 4); break;
        case 4: memcpy(out, o.w.data(), (size_t)o.S * 4); break;
        case 5: memcpy(out, o.post.data(), (size_t)o.S * 4); break;
        case 6: for (size_t j = 0; j < N; ++j) ((int32_t*)out)[j] = o.ref[j]; break;
        case 7: memcpy(out, o.last_post.data(), N * 4); break;
        case 8: memcpy(out, o.last_pre.data(), N * 4); break;
    }
}

// Exact push of one spike vector through (post, w): the closed form the
// product's snn_propagate must reproduce.  acc is int32 with wrapping adds.
void o4_propagate(const int32_t* post, const float* w, int64_t n_pre, int32_t fanout,
                  const uint8_t* spikes, int32_t* acc, int32_t frac_bits) {
    const float scale = pm_bits2f((uint32_t)(127 + frac_bits) << 23);
    for (int64_t i = 0; i < n_pre; ++i) {
        if (!spikes[i]) continue;
        for (int32_t k = 0; k < fanout; ++k) {
            const int64_t s = i * fanout + k;
            const int32_t q = (int32_t)pm_rint(pm_mul(w[s], scale));
            acc[post[s]] = (int32_t)((uint32_t)acc[post[s]] + (uint32_t)q);
        }
    }
}

}  // extern "C"
