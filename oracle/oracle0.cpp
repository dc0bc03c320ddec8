// oracle0.cpp - CPU oracle for the Stage 0 / Stage 2 step (LIF + pair STDP +
// eligibility trace + dopamine + homeostatic threshold, delay 1).
//
// TEST INFRASTRUCTURE ONLY: the checker for the CUDA path; never linked into
// or called by the product library.
//
// Restates SNNNetwork::step (src/host/network.cpp:143-191) operation by
// operation:
//   clear + CSR pull propagation of the previous step's spikes with the
//     reference's fixed 256-thread shared-memory tree
//     (src/cuda/synapse_kernel.cu:54-98) - deterministic in the reference;
//   one-hot external input (src/cuda/io_kernel.cu:12-21,
//     src/stage2/text_stream.cu:266-295);
//   LIF (src/cuda/neuron_kernel.cu:52-105);
//   pair STDP + eligibility + dopamine with delta-w before the timestamp
//     update (src/cuda/stdp_kernel.cu:29-85);
//   fire rate + homeostatic threshold (src/cuda/neuron_kernel.cu:117-153);
//   periodic reset (src/stage2/unsupervised_trainer.cu:154-157,
//     src/host/network.cpp:193-199, src/cuda/neuron_kernel.cu:158-173).
// Topologies: the reference's own are generated with device curand; here the
// seeded out-degree generators of the benchmark configurations are used (see
// gen_topology), identical to the product's generator.
// Canonical choices shared with the CUDA path: snn_expf for the STDP kernel
// (tabulated per integer dt), fma contraction of `a*b + c` statements, and
// explicit comparisons for clamps (sign of zero fixed).
#include <cstdint>
#include <cstring>
#include <cmath>
#include <vector>
#include "snn_pmath.h"
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

struct O0Params {
    int32_t n_columns;   // 0 = Stage 0 block layout; > 0 = columns of (sens, assoc, motor)
    int32_t n_sens, n_assoc, n_motor;  // per block (Stage 0) or per column
    int32_t deg_intra;   // out-edges inside the column (or anywhere for Stage 0)
    int32_t deg_inter;   // out-edges to other columns
    uint32_t seed;
    float w_max;         // exc w ~ U[0, w_max), inh w ~ -U[0, w_max)
    float input_gain;    // one-hot drive of the injected byte
    float homeo_lr, homeo_max, target_sa, target_m;
    int32_t reset_interval;  // 0 = never
    float dopamine;
    int32_t n_threads;
};

struct SplitMix64 {
    uint64_t s;
    uint64_t next() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    uint32_t below(uint32_t n) { return (uint32_t)((next() >> 32) * (uint64_t)n >> 32); }
    float unit() { return pm_mul(pm_u2f((uint32_t)(next() >> 40)), 5.9604644775390625e-08f); }
};

struct O0 {
    O0Params P;
    int N = 0;
    long long S = 0;
    std::vector<int32_t> pre, post;       // pre-major synapse list (generation order)
    std::vector<int32_t> in_ptr, in_syn;  // post-major: incoming synapse ids, ascending
    std::vector<float> w, elig;           // per synapse
    std::vector<float> V, I, fr;
    std::vector<int32_t> ref, last_lif;
    std::vector<int8_t> off;
    std::vector<uint8_t> type, region;    // region 0 sensory, 1 association, 2 motor
    std::vector<float> last_spk;          // STDP timestamps (never reset)
    std::vector<uint8_t> spike;
    std::vector<float> input;
    std::vector<float> exp_tab;           // snn_expf(-k/20), k = 0..2200
    long long step_no = 0, total_spikes = 0, events = 0;
    int last_spikes = 0;
    bool reset_pending = false;
};

// neuron types and regions: the first 80 % of every region (Stage 0) or
// layer of a column (Stage 2) are excitatory (src/include/types.h:173-205)
void gen_layout(O0& o) {
    const O0Params& P = o.P;
    const int per = P.n_sens + P.n_assoc + P.n_motor;
    const int ncol = P.n_columns > 0 ? P.n_columns : 1;
    o.N = ncol * per;
    o.type.assign(o.N, 0);
    o.region.assign(o.N, 0);
    for (int i = 0; i < o.N; ++i) {
        int off = i % per;
        int r, lo, sz;
        if (off < P.n_sens) { r = 0; lo = off; sz = P.n_sens; }
        else if (off < P.n_sens + P.n_assoc) { r = 1; lo = off - P.n_sens; sz = P.n_assoc; }
        else { r = 2; lo = off - P.n_sens - P.n_assoc; sz = P.n_motor; }
        o.region[i] = (uint8_t)r;
        o.type[i] = lo < (int)pm_mul(pm_i2f(sz), 0.8f) ? 0 : 1;
    }
}

// incoming lists: every post's synapses in ascending synapse id
void build_in_lists(O0& o) {
    o.in_ptr.assign(o.N + 1, 0);
    for (long long s = 0; s < o.S; ++s) o.in_ptr[o.post[s] + 1]++;
    for (int i = 0; i < o.N; ++i) o.in_ptr[i + 1] += o.in_ptr[i];
    o.in_syn.resize(o.S);
    std::vector<int32_t> fill(o.in_ptr.begin(), o.in_ptr.end() - 1);
    for (long long s = 0; s < o.S; ++s) o.in_syn[fill[o.post[s]]++] = (int32_t)s;
}

void gen_topology(O0& o) {
    const O0Params& P = o.P;
    gen_layout(o);
    const int per = P.n_sens + P.n_assoc + P.n_motor;
    const int ncol = P.n_columns > 0 ? P.n_columns : 1;
    SplitMix64 rng{P.seed};
    const int deg = P.deg_intra + (P.n_columns > 0 ? P.deg_inter : 0);
    o.S = (long long)o.N * deg;
    o.pre.resize(o.S); o.post.resize(o.S); o.w.resize(o.S); o.elig.assign(o.S, 0.0f);
    long long k = 0;
    for (int p = 0; p < o.N; ++p) {
        const int col = p / per;
        for (int e = 0; e < deg; ++e) {
            int q;
            if (P.n_columns <= 0) {
                q = (int)rng.below((uint32_t)(o.N - 1));
                if (q >= p) q++;
            } else if (e < P.deg_intra) {
                int r = (int)rng.below((uint32_t)(per - 1));
                int base = col * per;
                q = base + r;
                if (q >= p) q++;
            } else {
                int c = (int)rng.below((uint32_t)(ncol - 1));
                if (c >= col) c++;
                q = c * per + (int)rng.below((uint32_t)per);
            }
            float u = pm_mul(rng.unit(), P.w_max);
            o.pre[k] = p;
            o.post[k] = q;
            o.w[k] = o.type[p] == 0 ? u : -u;
            ++k;
        }
    }
    build_in_lists(o);
}

void init_state(O0& o) {
    const int N = o.N;
    o.V.assign(N, 0.0f); o.I.assign(N, 0.0f); o.fr.assign(N, 0.0f);
    o.ref.assign(N, 0); o.last_lif.assign(N, -1000); o.off.assign(N, 0);
    o.last_spk.assign(N, -1000.0f);
    o.spike.assign(N, 0);
    o.input.assign(N, 0.0f);
    o.exp_tab.resize(2201);
    for (int k = 0; k <= 2200; ++k) o.exp_tab[k] = snn_expf(pm_div(-pm_i2f(k), 20.0f));
}

// exp(-k/20) for integer k >= 1 (dt values are exact integers in float)
inline float exp_neg_over_20(const O0& o, float k) {
    int ki = (int)k;
    return ki <= 2200 ? o.exp_tab[ki] : 0.0f;
}

// src/cuda/synapse_kernel.cu:54-98 - 256 partial sums, then the tree
float tree256(const O0& o, int j) {
    const int b = o.in_ptr[j], n = o.in_ptr[j + 1] - b;
    if (n == 0) return 0.0f;
    float sd[256];
    for (int t = 0; t < 256; ++t) {
        float acc = 0.0f;
        for (int i = t; i < n; i += 256) {
            int s = o.in_syn[b + i];
            if (o.spike[o.pre[s]]) acc = pm_add(acc, o.w[s]);
        }
        sd[t] = acc;
    }
    for (int s = 128; s > 0; s >>= 1)
        for (int t = 0; t < s; ++t) sd[t] = pm_add(sd[t], sd[t + s]);
    return pm_add(0.0f, sd[0]);
}

void step(O0& o, int inject_byte) {
    const int N = o.N;
    const long long S = o.S;
    const long long t = o.step_no;
    const float tf = pm_ll2f(t);
    // 1-2. propagation of the previous step's spikes
    if (o.reset_pending) {
        std::fill(o.input.begin(), o.input.end(), 0.0f);
    } else {
#pragma omp parallel for schedule(static)
        for (int j = 0; j < N; ++j) o.input[j] = tree256(o, j);
    }
    // the event count: out-edges of the previous step's spikers
    // 3. one-hot input
    if (inject_byte >= 0 && inject_byte < N)
        o.input[inject_byte] = pm_add(o.input[inject_byte], pm_mul(o.P.input_gain, 1.0f));
    // 4. LIF
    int nsp = 0;
    for (int i = 0; i < N; ++i) {
        if (o.ref[i] > 0) {
            o.ref[i]--;
            o.spike[i] = 0;
            o.V[i] = pm_fma(pm_sub(o.V[i], 0.0f), 0.95f, 0.0f);
            continue;
        }
        o.I[i] = pm_fma(o.I[i], 0.95f, o.input[i]);
        float v = pm_fma(o.V[i], 0.95f, o.I[i]);
        if (v < 0.0f) v = 0.0f;
        float thr = pm_add(1.0f, pm_div(pm_i2f(o.off[i]), 16.0f));
        bool sp = v >= thr;
        if (sp) { o.last_lif[i] = (int32_t)t; v = 0.0f; o.ref[i] = 2; nsp++; }
        o.spike[i] = sp;
        o.V[i] = v;
    }
    // 5. STDP with eligibility + dopamine; dw before the timestamp update
    const float da = o.P.dopamine;
#pragma omp parallel for schedule(static)
    for (long long s = 0; s < S; ++s) {
        const int p = o.pre[s], q = o.post[s];
        const bool pf = o.spike[p], qf = o.spike[q];
        float dw = 0.0f;
        if (pf) {
            float dt = pm_sub(o.last_spk[q], tf);
            if (dt < 0.0f && o.last_spk[q] > -500.0f)
                dw = pm_fma(-0.05f, exp_neg_over_20(o, -dt), dw);
        }
        if (qf) {
            float dt = pm_sub(tf, o.last_spk[p]);
            if (dt > 0.0f && o.last_spk[p] > -500.0f)
                dw = pm_fma(0.05f, exp_neg_over_20(o, dt), dw);
        }
        float e = pm_fma(0.95f, o.elig[s], dw);
        o.elig[s] = e;
        float w = pm_fma(da, e, o.w[s]);
        if (o.type[p] == 0) { if (w > 1.0f) w = 1.0f; if (w < 0.0f) w = 0.0f; }
        else { if (w > 0.0f) w = 0.0f; if (w < -1.0f) w = -1.0f; }
        o.w[s] = w;
    }
    for (int i = 0; i < N; ++i)
        if (o.spike[i]) o.last_spk[i] = tf;
    // 7. fire rate + homeostasis
    const float om = pm_sub(1.0f, 0.95f);
    for (int i = 0; i < N; ++i) {
        float sp = o.spike[i] ? 1.0f : 0.0f;
        o.fr[i] = pm_fma(o.fr[i], 0.95f, pm_mul(sp, om));
        float tgt = o.region[i] == 2 ? o.P.target_m : o.P.target_sa;
        float err = pm_sub(o.fr[i], tgt);
        float nv = pm_fma(pm_mul(o.P.homeo_lr, err), 16.0f, pm_i2f(o.off[i]));
        float mx = pm_mul(o.P.homeo_max, 16.0f);
        if (nv > mx) nv = mx;
        if (nv < -mx) nv = -mx;
        o.off[i] = (int8_t)nv;
    }
    o.total_spikes += nsp;
    o.last_spikes = nsp;
    o.reset_pending = false;
    // 9. periodic reset after this step
    if (o.P.reset_interval > 0 && t > 0 && t % o.P.reset_interval == 0) {
        for (int i = 0; i < N; ++i) {
            o.V[i] = 0.0f; o.I[i] = 0.0f; o.last_lif[i] = -1000; o.ref[i] = 0; o.fr[i] = 0.0f;
        }
        o.reset_pending = true;  // spikes cleared for the next propagation
    }
    o.step_no++;
}

}  // namespace

extern "C" {

void* o0_create(const O0Params* p) {
    O0* o = new O0();
    o->P = *p;
    gen_topology(*o);
    init_state(*o);
    return o;
}
// the network of an explicit synapse list (e.g. a topology the reference
// generated): synapse s runs pre[s] -> post[s] with weight w[s]; every post's
// incoming synapses are propagated in ascending s.  Returns null when the
// list does not fit the layout of p.
void* o0_create_synapses(const O0Params* p, int64_t S, const int32_t* pre, const int32_t* post,
                         const float* w) {
    O0* o = new O0();
    o->P = *p;
    gen_layout(*o);
    o->S = S;
    o->pre.assign(pre, pre + S);
    o->post.assign(post, post + S);
    o->w.assign(w, w + S);
    o->elig.assign(S, 0.0f);
    for (int64_t s = 0; s < S; ++s)
        if (pre[s] < 0 || pre[s] >= o->N || post[s] < 0 || post[s] >= o->N) {
            delete o;
            return nullptr;
        }
    build_in_lists(*o);
    init_state(*o);
    return o;
}
void o0_destroy(void* h) { delete (O0*)h; }
void o0_run(void* h, int32_t n, const int32_t* bytes) {
    O0* o = (O0*)h;
#ifdef _OPENMP
    if (o->P.n_threads > 0) omp_set_num_threads(o->P.n_threads);
#endif
    for (int k = 0; k < n; ++k) step(*o, bytes ? bytes[k] : -1);
}
void o0_sizes(void* h, int64_t* out) {
    O0* o = (O0*)h;
    out[0] = o->N; out[1] = o->S; out[2] = o->step_no; out[3] = o->total_spikes;
    out[4] = o->last_spikes;
}
void o0_spikes(void* h, uint8_t* out) { O0* o = (O0*)h; memcpy(out, o->spike.data(), o->N); }
// 0 V, 1 I, 2 fr, 3 input, 4 last_spk (STDP timestamps), 5 off, 6 ref
void o0_neuron(void* h, int32_t which, float* out) {
    O0* o = (O0*)h;
    for (int i = 0; i < o->N; ++i) {
        float v = 0;
        switch (which) {
            case 0: v = o->V[i]; break;
            case 1: v = o->I[i]; break;
            case 2: v = o->fr[i]; break;
            case 3: v = o->input[i]; break;
            case 4: v = o->last_spk[i]; break;
            case 5: v = (float)o->off[i]; break;
            case 6: v = (float)o->ref[i]; break;
        }
        out[i] = v;
    }
}
// synapse arrays in generation (pre-major) order: 0 w, 1 elig
void o0_synapse(void* h, int32_t which, float* out) {
    O0* o = (O0*)h;
    memcpy(out, which == 0 ? o->w.data() : o->elig.data(), o->S * sizeof(float));
}
void o0_topology(void* h, int32_t* pre, int32_t* post) {
    O0* o = (O0*)h;
    if (pre) memcpy(pre, o->pre.data(), o->S * 4);
    if (post) memcpy(post, o->post.data(), o->S * 4);
}
void o0_set_dopamine(void* h, float da) { ((O0*)h)->P.dopamine = da; }

}  // extern "C"
