// engine0.cu - Stage 0 / Stage 2 engine on sm_100a: LIF neurons, delay-1
// spike propagation, pair STDP with eligibility trace and dopamine, fire
// rate and homeostatic threshold (src/host/network.cpp:143-191).
//
// Per step, two kernels over the post-major incoming lists (warp per neuron):
//   k0_prop_lif  propagation of the previous step's spikes + one-hot input +
//                LIF + fire rate / homeostasis of the post neuron
//   k0_stdp      pair STDP + eligibility + dopamine on every incoming synapse
// The propagation sum reproduces the reference's fixed 256-thread tree
// (src/cuda/synapse_kernel.cu:54-98): tree slot t accumulates incoming
// synapses t, t+256, ... in order, then slots are halved 128, 64, ..., 1.  A
// warp lane l holds slots l + 32m (m = 0..7); the first three halvings stay
// in the lane, the last five are shfl_down steps, so the result is the
// reference's bit for bit.
// STDP timestamps (the reference's per-synapse last_pre / last_post, which are
// the pre's / post's last spike times because every synapse is updated every
// step) are kept per neuron: A = last spike, B = the spike before A.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include "ckpt.h"
#include "common.h"
#include "snn_pmath.h"

namespace snn0 {

constexpr int EXP_TAB = 2201;  // snn_expf(-k/20) for k = 0..2200 (0 beyond)

struct Args {        // per launch
    long long t0;    // step of graph node k = 0
    long long corpus_pos0;
    long long corpus_len;
    int byte_override;  // >= 0: byte of the first step of this launch
    int reset_interval;
    float dopamine;
    int learn;
};

struct Ctrl {
    unsigned long long spikes, events;
    unsigned long long step_events[2];  // outgoing synapses of the step's spikes (by step parity)
    int step_spikes[2];
    long long raster_base;
    int reset_pending;
};

struct Consts {
    float beta, thr, in_gain, a_plus, a_minus, elig_decay, w_max, fr_decay;
    float homeo_lr, homeo_max, target_sa, target_m;
    int refr;
};

struct Dev {
    float *V, *I, *fr, *A, *B, *input;
    int *ref, *last, *off;
    unsigned char* info;     // type | region << 1
    unsigned char* spk;      // [2][N]
    int *in_ptr, *outdeg;
    unsigned* pre;           // pre index | (pre inhibitory) << 31, post-major
    float *w, *e;            // post-major
    float* exp_tab;
    const unsigned char* corpus;
    unsigned* raster;
    Ctrl* ctrl;
    const Args* args;
    int N, words, raster_cap;
};

__device__ __forceinline__ float exp_dt(const float* tab, float k) {
    int ki = (int)k;
    return ki < EXP_TAB ? tab[ki] : 0.0f;
}

// --- propagation + LIF ------------------------------------------------------
__global__ void __launch_bounds__(256) k0_prop_lif(Dev d, Consts k, int kstep) {
    const int lane = threadIdx.x & 31;
    const int j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (j >= d.N) return;
    const Args& a = *d.args;
    const long long t = a.t0 + kstep;
    const unsigned char* sprev = d.spk + ((t - 1) & 1) * (long long)d.N;
    const bool silent = d.ctrl->reset_pending || t == 0;
    const int b = d.in_ptr[j], n = d.in_ptr[j + 1] - b;
    float part[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) part[m] = 0.0f;
    if (!silent) {
        for (int c = 0; c * 32 < n; ++c) {
            const int i = c * 32 + lane;
            float term = 0.0f;
            bool add = false;
            if (i < n) {
                const unsigned p = d.pre[b + i] & 0x7fffffffu;
                if (sprev[p]) { term = d.w[b + i]; add = true; }
            }
            const int m = c & 7;
            // slot (c & 7) * 32 + lane accumulates synapses in ascending order
#pragma unroll
            for (int q = 0; q < 8; ++q)
                if (q == m && add) part[q] = pm_add(part[q], term);
        }
    }
    // 256 -> 32 inside the lane, then 16..1 across lanes
#pragma unroll
    for (int q = 0; q < 4; ++q) part[q] = pm_add(part[q], part[q + 4]);
    part[0] = pm_add(part[0], part[2]);
    part[1] = pm_add(part[1], part[3]);
    float v = pm_add(part[0], part[1]);
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const float o = __shfl_down_sync(0xffffffffu, v, s);
        if (lane < s) v = pm_add(v, o);
    }
    if (lane != 0) return;
    float in = (n == 0 || silent) ? 0.0f : pm_add(0.0f, v);
    // one-hot input of this step's byte
    int byte = -1;
    if (kstep == 0 && a.byte_override >= 0) byte = a.byte_override;
    else if (a.corpus_len > 0) byte = d.corpus[(a.corpus_pos0 + kstep) % a.corpus_len];
    if (byte >= 0 && byte == j) in = pm_add(in, pm_mul(k.in_gain, 1.0f));
    d.input[j] = in;
    // LIF (src/cuda/neuron_kernel.cu:52-105)
    int ref = d.ref[j];
    float V = d.V[j];
    bool sp = false;
    if (ref > 0) {
        d.ref[j] = ref - 1;
        d.V[j] = pm_fma(pm_sub(V, 0.0f), k.beta, 0.0f);
    } else {
        const float I = pm_fma(d.I[j], k.beta, in);
        d.I[j] = I;
        V = pm_fma(V, k.beta, I);
        if (V < 0.0f) V = 0.0f;
        const float thr = pm_add(k.thr, pm_div(pm_i2f(d.off[j]), 16.0f));
        if (V >= thr) {
            sp = true;
            d.last[j] = (int)t;
            V = 0.0f;
            d.ref[j] = k.refr;
        }
        d.V[j] = V;
    }
    d.spk[(t & 1) * (long long)d.N + j] = sp;
    if (sp) {
        const float tf = pm_ll2f(t);
        d.B[j] = d.A[j];
        d.A[j] = tf;
        atomicAdd(&d.ctrl->spikes, 1ull);
        atomicAdd(&d.ctrl->events, (unsigned long long)d.outdeg[j]);
        atomicAdd(&d.ctrl->step_spikes[t & 1], 1);
        atomicAdd(&d.ctrl->step_events[t & 1], (unsigned long long)d.outdeg[j]);
        const long long row = (t - d.ctrl->raster_base) % d.raster_cap;
        atomicOr(&d.raster[row * d.words + (j >> 5)], 1u << (j & 31));
    }
    // fire rate + homeostasis (src/cuda/neuron_kernel.cu:117-153)
    const float om = pm_sub(1.0f, k.fr_decay);
    const float fr = pm_fma(d.fr[j], k.fr_decay, pm_mul(sp ? 1.0f : 0.0f, om));
    d.fr[j] = fr;
    const int region = (d.info[j] >> 1) & 3;
    const float err = pm_sub(fr, region == 2 ? k.target_m : k.target_sa);
    float nv = pm_fma(pm_mul(k.homeo_lr, err), 16.0f, pm_i2f(d.off[j]));
    const float mx = pm_mul(k.homeo_max, 16.0f);
    if (nv > mx) nv = mx;
    if (nv < -mx) nv = -mx;
    d.off[j] = (int)(signed char)(int)nv;
}

// --- pair STDP + eligibility + dopamine (src/cuda/stdp_kernel.cu:29-85) ---
__global__ void __launch_bounds__(256) k0_stdp(Dev d, Consts k, int kstep) {
    const int lane = threadIdx.x & 31;
    const int j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const Args& a = *d.args;
    const long long t = a.t0 + kstep;
    // clear the raster row and the spike / event counts of the next step
    if (blockIdx.x == 0) {
        const long long row = (t + 1 - d.ctrl->raster_base) % d.raster_cap;
        for (int q = threadIdx.x; q < d.words; q += blockDim.x) d.raster[row * d.words + q] = 0u;
        if (threadIdx.x == 0) {
            d.ctrl->step_spikes[(t + 1) & 1] = 0;
            d.ctrl->step_events[(t + 1) & 1] = 0ull;
        }
    }
    if (j >= d.N) return;
    const unsigned char* snow = d.spk + (t & 1) * (long long)d.N;
    const float tf = pm_ll2f(t);
    const bool qf = snow[j];
    // post's last spike strictly before t
    const float LSq = qf ? d.B[j] : d.A[j];
    const float da = a.learn ? a.dopamine : 0.0f;
    const int b = d.in_ptr[j], e = d.in_ptr[j + 1];
    for (int i = b + lane; i < e; i += 32) {
        const unsigned pp = d.pre[i];
        const unsigned p = pp & 0x7fffffffu;
        const bool inh = pp >> 31;
        const bool pf = snow[p];
#ifdef SNN_REFMATH
        // the reference's expressions as written (CUDA expf, the compiler's
        // default contraction), for agreement with the reference binary
        float delta_w = 0.0f;
        if (pf) {
            const float dt = LSq - tf;
            if (dt < 0.0f && LSq > -500.0f) delta_w -= 0.05f * expf(dt / 20.0f);
        }
        if (qf) {
            const float LSp = pf ? d.B[p] : d.A[p];
            const float dt = tf - LSp;
            if (dt > 0.0f && LSp > -500.0f) delta_w += 0.05f * expf(-dt / 20.0f);
        }
        const float el = 0.95f * d.e[i] + delta_w;
        d.e[i] = el;
        const float weight_delta = da * el;
        float w = d.w[i];
        w += weight_delta;
#else
        float dw = 0.0f;
        if (pf) {
            const float dt = pm_sub(LSq, tf);
            if (dt < 0.0f && LSq > -500.0f) dw = pm_fma(-k.a_minus, exp_dt(d.exp_tab, -dt), dw);
        }
        if (qf) {
            const float LSp = pf ? d.B[p] : d.A[p];
            const float dt = pm_sub(tf, LSp);
            if (dt > 0.0f && LSp > -500.0f) dw = pm_fma(k.a_plus, exp_dt(d.exp_tab, dt), dw);
        }
        const float el = pm_fma(k.elig_decay, d.e[i], dw);
        d.e[i] = el;
        float w = pm_fma(da, el, d.w[i]);
#endif
        if (!inh) { if (w > k.w_max) w = k.w_max; if (w < 0.0f) w = 0.0f; }
        else { if (w > 0.0f) w = 0.0f; if (w < -k.w_max) w = -k.w_max; }
        d.w[i] = w;
    }
}

// reset after step t (src/cuda/neuron_kernel.cu:158-173): membrane state
// cleared, threshold offsets and STDP timestamps kept
__global__ void k0_reset(Dev d, int kstep) {
    const Args& a = *d.args;
    const long long t = a.t0 + kstep;
    const bool do_reset = a.reset_interval > 0 && t > 0 && (t % a.reset_interval) == 0;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) d.ctrl->reset_pending = do_reset ? 1 : 0;
    if (!do_reset || i >= d.N) return;
    d.V[i] = 0.0f; d.I[i] = 0.0f; d.last[i] = -1000; d.ref[i] = 0; d.fr[i] = 0.0f;
}

// ---------------------------------------------------------------------------
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

struct Engine0 : snnb::Engine {
    snn_config cfg;
    cudaStream_t stream = nullptr;
    Consts K{};
    Dev D{};
    int N = 0, ncol = 0, per = 0;
    int64_t S = 0;
    bool built = false;
    long long steps = 0;
    long long corpus_pos = 0, corpus_len = 0;
    int raster_cap = 1024;
    long long raster_base_host = 0;  // first step of the current raster rows
    float dopamine = 1.0f;
    int reset_interval = 0;
    std::vector<int32_t> h_pre, h_post, perm, in_ptr_h;  // perm: post-major -> generation id
    std::vector<int32_t> out_ptr_h;  // pre-major row pointer of the generation order
    std::vector<uint8_t> h_type;
    snnb::DevBuf<float> V, I, fr, A, B, input, w, e, exp_tab;
    snnb::DevBuf<int> ref, last, off, in_ptr, outdeg;
    snnb::DevBuf<unsigned char> info, spk, corpus;
    snnb::DevBuf<unsigned> pre, raster;
    snnb::DevBuf<Ctrl> ctrl;
    snnb::DevBuf<Args> args;
    Args* h_args = nullptr;  // pinned
    cudaGraphExec_t gexec = nullptr;
    cudaGraph_t graph = nullptr;
    int gsteps = 0;
    bool profiling = false;
    std::vector<cudaEvent_t> pev;
    snn_profile prof{};

    explicit Engine0(const snn_config& c) : cfg(c) {
        if (cfg.raster_steps > 0) raster_cap = cfg.raster_steps;
        SNN_CUDA(cudaSetDevice(cfg.device));
        SNN_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        SNN_CUDA(cudaMallocHost((void**)&h_args, sizeof(Args)));
        // LIF / STDP constants (src/include/config.h:16-41)
        K.beta = 0.95f; K.thr = 1.0f; K.refr = 2; K.a_plus = 0.05f; K.a_minus = 0.05f;
        K.elig_decay = 0.95f; K.w_max = 1.0f; K.fr_decay = 0.95f;
    }

    // homeostasis and input drive: the benchmark's constants, or those of the
    // reference's own build of the layout (block network = Stage 0 build,
    // columns = Stage 2 build)
    void set_preset_consts(bool columnar) {
        if (cfg.preset == SNN_PRESET_BASELINE) {
            // benchmark configuration: I_ext 1.5, homeostatic LR 1e-4, 5 / 30 Hz targets
            K.in_gain = 1.5f; K.homeo_lr = 1e-4f; K.homeo_max = 2.0f;
            K.target_sa = 0.005f; K.target_m = 0.030f;
        } else if (!columnar) {
            // Stage 0 build of the reference (src/include/config.h:33-40):
            // LR 0.05, max offset 2.0, 5 / 30 Hz; one-hot drive 1.5
            K.in_gain = 1.5f; K.homeo_lr = 0.05f; K.homeo_max = 2.0f;
            K.target_sa = 0.005f; K.target_m = 0.030f;
        } else {
            // Stage 2 build of the reference (src/include/config.h:74-83,
            // src/stage2/config.h:127-128): gain 5, LR 0.005, max 0.1, 15 / 30 Hz
            K.in_gain = 5.0f; K.homeo_lr = 0.005f; K.homeo_max = 0.1f;
            K.target_sa = 0.015f; K.target_m = 0.030f;
        }
    }
    ~Engine0() override {
        for (auto ev : pev) cudaEventDestroy(ev);
        if (gexec) cudaGraphExecDestroy(gexec);
        if (graph) cudaGraphDestroy(graph);
        if (stream) { cudaStreamSynchronize(stream); cudaStreamDestroy(stream); }
        if (h_args) cudaFreeHost(h_args);
    }

    void build(const snn_topology_spec& sp) override {
        SNN_REQUIRE(!built, SNN_ERR_STATE, "network already built");
        SNN_REQUIRE(sp.l4 > 0 && sp.l23 > 0 && sp.l5 > 0 && sp.deg_intra > 0, SNN_ERR_ARG,
                    "stage0 topology: sensory / association / motor sizes and degree needed");
        ncol = sp.n_columns;
        set_preset_consts(ncol > 0);
        per = sp.l4 + sp.l23 + sp.l5;
        N = (ncol > 0 ? ncol : 1) * per;
        SNN_REQUIRE(ncol != 1, SNN_ERR_ARG, "columnar stage0 needs >= 2 columns");
        reset_interval = ncol > 0 ? 10000 : 0;  // Stage 2 trainer resets every 10K steps
        const float wmax = cfg.preset == SNN_PRESET_BASELINE ? 1.0f : 0.3f;
        // neurons: first 80 % of each region / layer excitatory
        h_type.assign(N, 0);
        std::vector<unsigned char> h_info(N);
        for (int i = 0; i < N; ++i) {
            int o = i % per, r, lo, sz;
            if (o < sp.l4) { r = 0; lo = o; sz = sp.l4; }
            else if (o < sp.l4 + sp.l23) { r = 1; lo = o - sp.l4; sz = sp.l23; }
            else { r = 2; lo = o - sp.l4 - sp.l23; sz = sp.l5; }
            h_type[i] = lo < (int)pm_mul(pm_i2f(sz), 0.8f) ? 0 : 1;
            h_info[i] = (unsigned char)(h_type[i] | (r << 1));
        }
        // seeded out-degree topology
        SplitMix64 rng{sp.seed};
        const int deg = sp.deg_intra + (ncol > 0 ? sp.deg_inter : 0);
        S = (int64_t)N * deg;
        h_pre.resize(S); h_post.resize(S);
        std::vector<float> h_w(S);
        int64_t k = 0;
        for (int p = 0; p < N; ++p) {
            const int col = p / per;
            for (int q = 0; q < deg; ++q) {
                int t;
                if (ncol <= 0) { t = (int)rng.below((uint32_t)(N - 1)); if (t >= p) t++; }
                else if (q < sp.deg_intra) { t = col * per + (int)rng.below((uint32_t)(per - 1)); if (t >= p) t++; }
                else {
                    int c = (int)rng.below((uint32_t)(ncol - 1));
                    if (c >= col) c++;
                    t = c * per + (int)rng.below((uint32_t)per);
                }
                const float u = pm_mul(rng.unit(), wmax);
                h_pre[k] = p; h_post[k] = t; h_w[k] = h_type[p] == 0 ? u : -u;
                ++k;
            }
        }
        // post-major, ascending generation id
        in_ptr_h.assign(N + 1, 0);
        for (int64_t s = 0; s < S; ++s) in_ptr_h[h_post[s] + 1]++;
        for (int i = 0; i < N; ++i) in_ptr_h[i + 1] += in_ptr_h[i];
        perm.resize(S);
        std::vector<unsigned> pm_pre(S);
        std::vector<float> pm_w(S);
        std::vector<int32_t> fill(in_ptr_h.begin(), in_ptr_h.end() - 1);
        for (int64_t s = 0; s < S; ++s) {
            int32_t pos = fill[h_post[s]]++;
            perm[pos] = (int32_t)s;
            pm_pre[pos] = (unsigned)h_pre[s] | ((unsigned)h_type[h_pre[s]] << 31);
            pm_w[pos] = h_w[s];
        }
        std::vector<int> h_outdeg(N, deg);
        out_ptr_h.resize((size_t)N + 1);
        for (int i = 0; i <= N; ++i) out_ptr_h[i] = i * deg;
        // device
        V.alloc(N); I.alloc(N); fr.alloc(N); A.alloc(N); B.alloc(N); input.alloc(N);
        ref.alloc(N); last.alloc(N); off.alloc(N); info.alloc(N); spk.alloc(2 * (size_t)N);
        in_ptr.alloc(N + 1); outdeg.alloc(N); pre.alloc(S); w.alloc(S); e.alloc(S);
        exp_tab.alloc(EXP_TAB); corpus.alloc(1); ctrl.alloc(1); args.alloc(1);
        D.words = (N + 31) / 32;
        raster.alloc((size_t)raster_cap * D.words);
        for (auto* b : {&V, &I, &fr, &input, &e}) b->zero(stream);
        ref.zero(stream); off.zero(stream); spk.zero(stream); raster.zero(stream); ctrl.zero(stream);
        std::vector<float> m1000(N, -1000.0f);
        A.upload(m1000.data(), N, stream);
        B.upload(m1000.data(), N, stream);
        std::vector<int> l1000(N, -1000);
        last.upload(l1000.data(), N, stream);
        info.upload(h_info.data(), N, stream);
        in_ptr.upload(in_ptr_h.data(), N + 1, stream);
        outdeg.upload(h_outdeg.data(), N, stream);
        pre.upload(pm_pre.data(), S, stream);
        w.upload(pm_w.data(), S, stream);
        std::vector<float> tab(EXP_TAB);
        for (int q = 0; q < EXP_TAB; ++q) tab[q] = snn_expf(pm_div(-pm_i2f(q), 20.0f));
        exp_tab.upload(tab.data(), EXP_TAB, stream);
        SNN_CUDA(cudaStreamSynchronize(stream));
        D.V = V.p; D.I = I.p; D.fr = fr.p; D.A = A.p; D.B = B.p; D.input = input.p;
        D.ref = ref.p; D.last = last.p; D.off = off.p; D.info = info.p; D.spk = spk.p;
        D.in_ptr = in_ptr.p; D.outdeg = outdeg.p; D.pre = pre.p; D.w = w.p; D.e = e.p;
        D.exp_tab = exp_tab.p; D.corpus = corpus.p; D.raster = raster.p; D.ctrl = ctrl.p;
        D.args = args.p; D.N = N; D.raster_cap = raster_cap;
        built = true;
    }

    void set_corpus(const uint8_t* b, int64_t n) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_REQUIRE(n >= 0 && (n == 0 || b), SNN_ERR_ARG, "bad corpus");
        SNN_CUDA(cudaStreamSynchronize(stream));
        if ((size_t)n > corpus.n) {
            corpus.alloc(n);
            D.corpus = corpus.p;
            drop_graph();
        }
        if (n > 0) corpus.upload(b, n, stream);
        corpus_len = n;
        corpus_pos = 0;
        SNN_CUDA(cudaStreamSynchronize(stream));
    }

    void drop_graph() {
        if (gexec) cudaGraphExecDestroy(gexec);
        if (graph) cudaGraphDestroy(graph);
        gexec = nullptr; graph = nullptr; gsteps = 0;
    }

    void launch(int kstep, cudaEvent_t* ev, bool cap) {
        const unsigned fl = cap ? cudaEventRecordExternal : cudaEventRecordDefault;
        const unsigned blocks = (unsigned)(((long long)N * 32 + 255) / 256);
        if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[0], stream, fl));
        k0_prop_lif<<<blocks, 256, 0, stream>>>(D, K, kstep);
        if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[1], stream, fl));
        k0_stdp<<<blocks, 256, 0, stream>>>(D, K, kstep);
        k0_reset<<<(N + 255) / 256, 256, 0, stream>>>(D, kstep);
        if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[2], stream, fl));
    }

    void ensure_events(int n) {
        while (pev.size() < (size_t)(3 * n)) {
            cudaEvent_t ev;
            SNN_CUDA(cudaEventCreate(&ev));
            pev.push_back(ev);
        }
    }

    void ensure_graph(int n) {
        if (gexec && gsteps == n) return;
        drop_graph();
        if (profiling) ensure_events(n);
        SNN_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
        for (int q = 0; q < n; ++q) launch(q, profiling ? &pev[3 * q] : nullptr, true);
        SNN_CUDA(cudaStreamEndCapture(stream, &graph));
        SNN_CUDA(cudaGraphInstantiate(&gexec, graph, 0));
        gsteps = n;
    }

    void harvest(int n) {
        SNN_CUDA(cudaStreamSynchronize(stream));
        for (int q = 0; q < n; ++q)
            for (int kk = 0; kk < 2; ++kk) {
                float ms = 0;
                SNN_CUDA(cudaEventElapsedTime(&ms, pev[3 * q + kk], pev[3 * q + kk + 1]));
                prof.kernel_ms[kk] += ms;
                prof.launches[kk] += 1;
                prof.step_ms += ms;
            }
        prof.steps += n;
    }

    void put_args(int byte_override, int learn) {
        h_args->t0 = steps;
        h_args->corpus_pos0 = corpus_pos;
        h_args->corpus_len = corpus_len;
        h_args->byte_override = byte_override;
        h_args->reset_interval = reset_interval;
        h_args->dopamine = dopamine;
        h_args->learn = learn;
        SNN_CUDA(cudaMemcpyAsync(args.p, h_args, sizeof(Args), cudaMemcpyHostToDevice, stream));
    }

    void run(int32_t n_steps, int32_t byte_override, int32_t learn, uint32_t* raster_out,
             int32_t* counts_out) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        if (n_steps <= 0) return;
        long long rb = steps;
        raster_base_host = rb;
        SNN_CUDA(cudaMemcpyAsync((char*)ctrl.p + offsetof(Ctrl, raster_base), &rb, sizeof(rb),
                                 cudaMemcpyHostToDevice, stream));
        SNN_CUDA(cudaMemsetAsync(raster.p, 0, (size_t)D.words * sizeof(unsigned), stream));
        const int chunk = 50;
        int done = 0;
        while (done < n_steps) {
            const int span = std::min(n_steps - done, raster_cap - (done % raster_cap));
            int q = 0;
            while (q < span) {
                const int n = (span - q >= chunk) ? chunk : 1;
                // the pinned args buffer is reused: wait for the previous launch
                SNN_CUDA(cudaStreamSynchronize(stream));
                put_args(done + q == 0 ? byte_override : -1, learn ? 1 : 0);
                if (n == chunk) {
                    ensure_graph(chunk);
                    SNN_CUDA(cudaGraphLaunch(gexec, stream));
                } else {
                    if (profiling) ensure_events(1);
                    launch(0, profiling ? &pev[0] : nullptr, false);
                }
                SNN_CUDA(cudaGetLastError());
                if (profiling) harvest(n);
                steps += n;
                if (corpus_len > 0) corpus_pos = (corpus_pos + n) % corpus_len;
                q += n;
            }
            if (raster_out || counts_out) {
                const long long row0 = done % raster_cap;
                std::vector<unsigned> tmp((size_t)span * D.words);
                SNN_CUDA(cudaMemcpyAsync(tmp.data(), raster.p + row0 * D.words,
                                         tmp.size() * sizeof(unsigned), cudaMemcpyDeviceToHost, stream));
                SNN_CUDA(cudaStreamSynchronize(stream));
                if (raster_out) memcpy(raster_out + (size_t)done * D.words, tmp.data(), tmp.size() * 4);
                if (counts_out)
                    for (int r = 0; r < span; ++r) {
                        int c = 0;
                        for (int x = 0; x < D.words; ++x) c += __builtin_popcount(tmp[(size_t)r * D.words + x]);
                        counts_out[done + r] = c;
                    }
            }
            done += span;
        }
    }

    void sync() override { SNN_CUDA(cudaStreamSynchronize(stream)); }
    int64_t steps_done() const override { return steps; }

    void counters(snn_counters* o) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        Ctrl h;
        SNN_CUDA(cudaMemcpyAsync(&h, ctrl.p, sizeof(Ctrl), cudaMemcpyDeviceToHost, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
        memset(o, 0, sizeof(*o));
        o->step = steps;
        o->total_spikes = (int64_t)h.spikes;
        o->dispatched = (int64_t)h.events;
        // the last step's dispatches arrive at the next step
        o->arrivals = (int64_t)h.events - (steps > 0 ? (int64_t)h.step_events[(steps - 1) & 1] : 0);
        o->n_neurons = N;
        o->n_synapses = S;
        o->last_spikes = steps > 0 ? h.step_spikes[(steps - 1) & 1] : 0;
        o->last_byte = -1;
        o->modeled_bytes = (double)steps * 12.0 * (double)S;
    }

    void get_spikes(uint32_t* words, int64_t n_words) override {
        SNN_REQUIRE(built && steps > 0, SNN_ERR_STATE, "no step executed yet");
        SNN_REQUIRE(n_words >= D.words, SNN_ERR_ARG, "bitmask buffer too small");
        const long long row = (steps - 1 - raster_base_host) % raster_cap;
        SNN_CUDA(cudaMemcpyAsync(words, raster.p + row * D.words, D.words * 4, cudaMemcpyDeviceToHost, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
    }

    void get_state(int32_t which, void* buf, int64_t nbytes) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        auto need = [&](int64_t b) { SNN_REQUIRE(nbytes >= b, SNN_ERR_ARG, "state buffer too small"); };
        auto dl = [&](auto& db, size_t n) {
            db.download((typename std::remove_reference<decltype(*db.p)>::type*)buf, n, stream);
            SNN_CUDA(cudaStreamSynchronize(stream));
        };
        auto syn = [&](snnb::DevBuf<float>& db) {
            need(S * 4);
            std::vector<float> h(S);
            db.download(h.data(), S, stream);
            SNN_CUDA(cudaStreamSynchronize(stream));
            float* o = (float*)buf;
            for (int64_t p = 0; p < S; ++p) o[perm[p]] = h[p];
        };
        switch (which) {
            case SNN_STATE_V: need(N * 4); dl(V, N); break;
            case SNN_STATE_SYN_CURRENT: need(N * 4); dl(I, N); break;
            case SNN_STATE_FIRE_RATE: need(N * 4); dl(fr, N); break;
            case SNN_STATE_INPUT: need(N * 4); dl(input, N); break;
            case SNN_STATE_LAST_SPIKE: need(N * 4); dl(last, N); break;
            case SNN_STATE_REFRACTORY: need(N * 4); dl(ref, N); break;
            case SNN_STATE_THRESH_OFF: need(N * 4); dl(off, N); break;
            case SNN_STATE_WEIGHT: syn(w); break;
            case SNN_STATE_ELIG: syn(e); break;
            case SNN_STATE_POST: need(S * 4); memcpy(buf, h_post.data(), S * 4); break;
            case SNN_STATE_ROW_PTR:  // pre-major row pointer of the generation order
                need((int64_t)(N + 1) * 4);
                memcpy(buf, out_ptr_h.data(), (size_t)(N + 1) * 4);
                break;
            default: throw snnb::Error(SNN_ERR_UNSUPPORTED, "state field not available for stage0");
        }
    }

    void set_dopamine(float level) override { dopamine = level; }

    void set_profiling(int32_t en) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_CUDA(cudaStreamSynchronize(stream));
        profiling = en != 0;
        drop_graph();
        memset(&prof, 0, sizeof(prof));
        prof.n_kernels = 2;
        strcpy(prof.names[0], "k0_prop_lif");
        strcpy(prof.names[1], "k0_stdp");
    }
    void get_profile(snn_profile* o) override { *o = prof; }

    // ---- checkpoints ------------------------------------------------------
    // Device synapse order is the reference CSR order (incoming synapses by
    // post), the order of its d_synapses_ / d_col_idx_ / d_weights_ arrays.
    struct NativeBlob {
        int64_t steps, raster_base, corpus_pos, corpus_len, N, S;
        float dopamine;
        int32_t raster_cap, preset, ncol;
    };
    NativeBlob blob() const {
        NativeBlob b{};
        b.steps = steps; b.raster_base = raster_base_host; b.corpus_pos = corpus_pos;
        b.corpus_len = corpus_len; b.N = N; b.S = S; b.dopamine = dopamine;
        b.raster_cap = raster_cap; b.preset = cfg.preset; b.ncol = ncol;
        return b;
    }
    std::vector<snnb::DevSection> native_sections() {
        std::vector<snnb::DevSection> v;
        auto add = [&](const char* n, auto& b) { v.push_back({n, (void*)b.p, b.bytes()}); };
        add("V", V); add("I", I); add("fr", fr); add("A", A); add("B", B); add("input", input);
        add("w", w); add("e", e); add("ref", ref); add("last", last); add("off", off); add("spk", spk);
        add("raster", raster); add("ctrl", ctrl);
        return v;
    }
    // SNN2 v1 (src/stage2/unsupervised_trainer.cu:176-262): u32 magic
    // 0x534E4E32, u32 version 1, i64 step, u64 text_pos, i32 n_neurons,
    // i32 n_synapses, Synapse[n] {pre, post, w, delay, last_pre, last_post,
    // eligibility, pad} (32 B), i32 row_ptr[N+1], i32 col_idx[S], f32 w[S]
    struct Syn32 {
        int32_t pre, post;
        float w, delay, last_pre, last_post, elig, pad;
    };
    static_assert(sizeof(Syn32) == 32, "Synapse record");
    // Replace the synapse topology by a post-major CSR (row pointer rp[N+1],
    // pre index col[S]) read from a checkpoint; the caller has checked that
    // rp starts at 0, ends at S and ascends and that every col is in [0, N).
    // Generation order of the adopted synapses: by pre, and within a pre by
    // CSR position.
    void adopt_topology(const std::vector<int32_t>& rp, const std::vector<int32_t>& col) {
        std::vector<int32_t> optr((size_t)N + 1, 0);
        for (int64_t p = 0; p < S; ++p) optr[col[p] + 1]++;
        std::vector<int> h_outdeg(N);
        for (int i = 0; i < N; ++i) {
            h_outdeg[i] = optr[i + 1];
            optr[i + 1] += optr[i];
        }
        std::vector<int32_t> fill(optr.begin(), optr.end() - 1), np((size_t)S), npre((size_t)S), npost((size_t)S);
        std::vector<unsigned> pm_pre((size_t)S);
        for (int j = 0; j < N; ++j)
            for (int32_t p = rp[j]; p < rp[j + 1]; ++p) {
                const int32_t q = col[p], g = fill[q]++;
                np[p] = g;
                npre[g] = q;
                npost[g] = j;
                pm_pre[p] = (unsigned)q | ((unsigned)h_type[q] << 31);
            }
        in_ptr.upload(rp.data(), N + 1, stream);
        outdeg.upload(h_outdeg.data(), N, stream);
        pre.upload(pm_pre.data(), S, stream);
        SNN_CUDA(cudaStreamSynchronize(stream));
        in_ptr_h = rp;
        out_ptr_h = optr;
        perm = np;
        h_pre = npre;
        h_post = npost;
    }
    void save(const char* path, int32_t fmt) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_CUDA(cudaStreamSynchronize(stream));
        if (fmt == SNN_FMT_NATIVE) {
            const NativeBlob b = blob();
            snnb::save_native(path, SNN_MODEL_STAGE0, &b, sizeof(b), native_sections(), stream);
            return;
        }
        if (fmt == SNN_FMT_RAW_F32) {  // src/host/network.cpp:224-246
            snnb::BinFile f(path, true);
            f.put_dev(w.p, (size_t)S * 4, stream);
            f.close();
            return;
        }
        SNN_REQUIRE(fmt == SNN_FMT_SNN2_V1, SNN_ERR_UNSUPPORTED,
                    "Stage 0 writes the native, SNN2 v1 and raw formats");
        std::vector<float> hw((size_t)S), he((size_t)S), hA((size_t)N);
        std::vector<unsigned> hp((size_t)S);
        w.download(hw.data(), S, stream);
        e.download(he.data(), S, stream);
        A.download(hA.data(), N, stream);
        pre.download(hp.data(), S, stream);
        SNN_CUDA(cudaStreamSynchronize(stream));
        std::vector<Syn32> aos((size_t)S);
        std::vector<int32_t> col((size_t)S);
        for (int j = 0; j < N; ++j)
            for (int32_t p = in_ptr_h[j]; p < in_ptr_h[j + 1]; ++p) {
                const int32_t q = (int32_t)(hp[p] & 0x7fffffffu);
                aos[p] = Syn32{q, j, hw[p], 1.0f, hA[q], hA[j], he[p], 0.0f};
                col[p] = q;
            }
        snnb::BinFile f(path, true);
        f.put_v<uint32_t>(0x534E4E32u);
        f.put_v<uint32_t>(1u);
        f.put_v<int64_t>(steps);
        f.put_v<uint64_t>((uint64_t)corpus_pos);
        f.put_v<int32_t>(N);
        f.put_v<int32_t>((int32_t)S);
        f.put(aos.data(), sizeof(Syn32) * aos.size());
        f.put(in_ptr_h.data(), 4 * (size_t)(N + 1));
        f.put(col.data(), 4 * col.size());
        f.put(hw.data(), 4 * hw.size());
        f.close();
    }
    void load(const char* path, int32_t fmt) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_CUDA(cudaStreamSynchronize(stream));
        if (fmt == SNN_FMT_NATIVE) {
            const NativeBlob want = blob();
            NativeBlob got{};
            snnb::load_native(path, SNN_MODEL_STAGE0, &got, sizeof(got), native_sections(), stream,
                              [&](const void* p) {
                                  NativeBlob f;
                                  memcpy(&f, p, sizeof(f));
                                  SNN_REQUIRE(f.N == want.N && f.S == want.S && f.raster_cap == want.raster_cap &&
                                                  f.preset == want.preset && f.ncol == want.ncol,
                                              SNN_ERR_IO, "checkpoint of another network");
                              });
            steps = got.steps; raster_base_host = got.raster_base; corpus_pos = got.corpus_pos;
            dopamine = got.dopamine;
            SNN_REQUIRE(got.corpus_len == corpus_len, SNN_ERR_IO,
                        "set the checkpoint's corpus (same length) before loading it");
            return;
        }
        if (fmt == SNN_FMT_RAW_F32) {  // src/host/network.cpp:248-290: exactly S floats
            snnb::BinFile f(path, false);
            SNN_REQUIRE(f.size() == S * 4, SNN_ERR_IO, "raw weight file size differs from the network");
            f.get_dev(w.p, (size_t)S * 4, stream);
            return;
        }
        SNN_REQUIRE(fmt == SNN_FMT_SNN2_V1, SNN_ERR_UNSUPPORTED,
                    "Stage 0 reads the native, SNN2 v1 and raw formats");
        // src/stage2/unsupervised_trainer.cu:264-348: header, sizes, then the
        // synapse records (their weight, eligibility and spike times) and
        // the CSR, which replaces this network's when it differs (a file
        // written by another build of the same sizes: neuron count, synapse
        // count; the neuron types stay this network's)
        snnb::BinFile f(path, false);
        SNN_REQUIRE(f.size() >= 32, SNN_ERR_IO, "truncated SNN2 file");
        SNN_REQUIRE(f.get_v<uint32_t>() == 0x534E4E32u, SNN_ERR_IO, "not an SNN2 file (bad magic)");
        SNN_REQUIRE(f.get_v<uint32_t>() == 1u, SNN_ERR_IO, "SNN2 version differs");
        const int64_t step = f.get_v<int64_t>();
        const uint64_t pos = f.get_v<uint64_t>();
        const int32_t nn = f.get_v<int32_t>(), ns = f.get_v<int32_t>();
        SNN_REQUIRE(nn == N && ns == (int32_t)S, SNN_ERR_IO, "SNN2 sizes differ from this network");
        SNN_REQUIRE(f.size() == 32 + 32 * S + 4 * (int64_t)(N + 1) + 8 * S, SNN_ERR_IO, "truncated SNN2 file");
        std::vector<Syn32> aos((size_t)S);
        f.get(aos.data(), sizeof(Syn32) * aos.size());
        std::vector<int32_t> rp((size_t)N + 1), col((size_t)S);
        f.get(rp.data(), 4 * rp.size());
        f.get(col.data(), 4 * col.size());
        std::vector<unsigned> hp((size_t)S);
        pre.download(hp.data(), S, stream);
        SNN_CUDA(cudaStreamSynchronize(stream));
        // the CSR spans the synapses, every pre is a neuron, and every
        // record agrees with the CSR it comes with (checked before any use)
        SNN_REQUIRE(rp[0] == 0 && rp[N] == (int32_t)S, SNN_ERR_IO, "SNN2 row pointer does not span the synapses");
        for (int j = 0; j < N; ++j) SNN_REQUIRE(rp[j] <= rp[j + 1], SNN_ERR_IO, "SNN2 row pointer not ascending");
        for (int64_t p = 0; p < S; ++p)
            SNN_REQUIRE(col[p] >= 0 && col[p] < N, SNN_ERR_IO, "SNN2 column index out of range");
        for (int j = 0; j < N; ++j)
            for (int32_t p = rp[j]; p < rp[j + 1]; ++p)
                SNN_REQUIRE(aos[p].post == j && aos[p].pre == col[p], SNN_ERR_IO,
                            "SNN2 synapse records disagree with the CSR");
        bool same = rp == in_ptr_h;
        for (int64_t p = 0; same && p < S; ++p) same = col[p] == (int32_t)(hp[p] & 0x7fffffffu);
        if (!same) adopt_topology(rp, col);
        std::vector<float> hw((size_t)S), he((size_t)S), hA((size_t)N, -1000.0f);
        for (int64_t p = 0; p < S; ++p) {
            hw[p] = aos[p].w;
            he[p] = aos[p].elig;
            hA[aos[p].pre] = aos[p].last_pre;
            hA[aos[p].post] = aos[p].last_post;
        }
        w.upload(hw.data(), S, stream);
        e.upload(he.data(), S, stream);
        A.upload(hA.data(), N, stream);
        B.upload(hA.data(), N, stream);  // only read within a spiking step, after it is set
        SNN_CUDA(cudaStreamSynchronize(stream));
        steps = step;
        corpus_pos = corpus_len > 0 ? (long long)(pos % (uint64_t)corpus_len) : 0;
    }
};

}  // namespace snn0

namespace snnb {
Engine* make_engine_stage0(const snn_config& cfg) { return new snn0::Engine0(cfg); }
}  // namespace snnb
