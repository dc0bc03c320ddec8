// oracle2e.cpp - CPU oracle for the Stage 2e step (AdEx + NMDA/Ca + STP +
// dual-trace PSW STDP + axonal delay ring + thalamic gate + modulators).
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
// compared against; it is never linked into, loaded by, or called from the
// product library.  Only tests/, __graft_entry__.smoke() and the cpu_baseline
// leg of bench.py may load it.
//
// It restates, operation by operation and in the same order, the reference
// step of TSOFTP-afk/pure-snn-language:
//   step order ............ src/stage2e/scheduler.cu:485-676
//   topology .............. src/stage2e/network_init.cu:158-473 (xorshift32)
//   neurons ............... src/stage2e/network_init.cu:38-127
//   AdEx .................. src/stage2e/neuron_kernels.cu:61-165
//   delay ring ............ src/stage2e/neuron_kernels.cu:37-56, 170-302
//   NMDA / Ca ............. src/stage2e/synapse_kernels.cu:45-141
//   dual-trace STDP ....... src/stage2e/synapse_kernels.cu:153-329
//   STP ................... src/stage2e/synapse_kernels.cu:334-387
//   CaMKII / eligibility .. src/stage2e/synapse_kernels.cu:469-543
//   input ................. src/stage2e/input_encoding.cu:117-203
//   thalamic gate ......... src/stage2e/thalamic_gate.cu:53-142
//   modulators / TD ....... src/stage2e/modulatory_kernels.cu:22-254,
//                           src/stage2e/scheduler.cu:724-751
//   inhibition / kWTA ..... src/stage2e/scheduler.cu:112-133, 234-265, 688-722
//   structural decay ...... src/stage2e/scheduler.cu:55-86, 1038-1058
//   phase table ........... src/stage2e/scheduler.cuh:35-61
//   constants ............. src/stage2e/config.h
//
// The reference is not bit-deterministic (float atomics, a racy novelty
// update).  This restatement fixes one canonical semantics, shared with the
// CUDA path:
//   (1) Float sums into a neuron (input current from arrivals, NMDA current)
//       run over the neuron's incoming synapses in ascending reference
//       synapse id (pre-major CSR index); non-contributing synapses give +0.
//       Position k of that list goes to partial sum k mod 32; each partial
//       adds its terms in ascending order from +0; the 32 partials are then
//       reduced by the xor butterfly (offsets 16, 8, 4, 2, 1).
//   (2) Every exponential is snn_expf (include/snn_pmath.h); constant decay
//       factors are snn_expf of the same float argument the reference passes.
//   (3) Contraction: an expression `a*b + c` (or `c + a*b`) that the
//       reference writes in one statement is one fma(a, b, c); `a*b + c*d`
//       is fma(a, b, c*d); `a*b - c*d` is fma(a, b, -(c*d)).  Host-side
//       float arithmetic of the reference (scheduler / modulatory host code)
//       is not contracted.
//   (4) Thalamic novelty: every column reads the byte history before any
//       increment of this step, then history[b] += n_columns.
//   (5) Delay ring slots are unbounded; the number of events the reference
//       would drop at its 750,000-entry slot capacity is counted only.
//   (6) Working-memory slots, hippocampal replay, synaptic scaling (a no-op
//       launcher) and logging have no effect on the dynamics and are omitted.

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cmath>
#include <vector>
#include <algorithm>
#include "snn_pmath.h"
#ifdef _OPENMP
#include <omp.h>
#endif

#if defined(__x86_64__)
#include <xmmintrin.h>
#include <pmmintrin.h>
#endif

namespace {

// ---------------------------------------------------------------------------
// Parameters (topology generator + run knobs).  Field order is the ctypes ABI.
// ---------------------------------------------------------------------------
struct O2eParams {
    int32_t n_columns;        // 50 in the reference
    int32_t l4, l23, l5, l6;  // layer sizes per column: 200/350/200/250
    int32_t pf_groups;        // prefrontal groups (50)
    int32_t pf_group_size;    // 100
    int32_t deg_intra;        // 150
    int32_t deg_inter;        // 30 (L2/3 only)
    int32_t deg_l5_pf;        // 15 (L5 only)
    int32_t deg_pf_self;      // 100
    int32_t deg_pf_assoc;     // 50
    int64_t total_synapses;   // 10,700,000
    uint32_t seed;            // 42
    int32_t e0;               // E0 ablation
    int32_t phase_offset;     // added to the step for the phase-table lookup
    int32_t n_threads;        // OpenMP threads (0 = library default)
    int32_t preset;           // 0 reference constants, 1 the benchmark's AdEx / STP constants
};

struct Syn {  // mirrors the 80-byte BioSynapse (src/stage2e/types.h:66-101)
    int32_t pre, post;
    float weight, delay_f, last_pre, last_post, x_pre, x_post;
    float nmda, ampa, ca, R, elig, elig_slow, u, scaling;
    float autop, da_r, ach_r;
    uint8_t flags, ne_u8, ht5_u8, pad;
};
static_assert(sizeof(Syn) == 80, "Syn layout");

struct Neu {  // mirrors NeuronStateAdEx (src/stage2e/types.h:31-59)
    float V, s, nmda_cur, w;
    int32_t last;
    float fr;
    int32_t ref;
    float ca;
    uint8_t type, region, subtype, column;
    int16_t pf_group;
    uint16_t off;
    float wm, hf;
    int32_t r0, r1;
};
static_assert(sizeof(Neu) == 56, "Neu layout");

struct Gate { float gate, act_ema, nov_ema, l6_ema; };

enum { REG_L4 = 0, REG_L23 = 1, REG_L5 = 2, REG_L6 = 3, REG_PF = 4 };
const uint8_t FLAG_FF = 0x10;

// phase table, src/stage2e/scheduler.cuh:38-49
const float PH_GAIN[5] = {0.0f, 1.0f, 3.0f, 1.0f, 0.3f};
const float PH_PRUNE[5] = {0.0f, 0.0f, 0.0f, 0.05f, 0.02f};
const int PH_END[5] = {5000, 200000, 800000, 1500000, 3000000};
int phase_of(long long step) {
    for (int i = 0; i < 5; ++i) if (step < PH_END[i]) return i;
    return 4;
}

inline float fclampf(float x, float lo, float hi) {
    if (x < lo) x = lo;
    if (x > hi) x = hi;
    return x;
}

// canonical reduction (1): butterfly over 32 terms, lane 0's result
inline float tree32(float* v) {
    float t[32];
    for (int off = 16; off >= 1; off >>= 1) {
        for (int l = 0; l < 32; ++l) t[l] = pm_add(v[l], v[l ^ off]);
        memcpy(v, t, sizeof(t));
    }
    return v[0];
}

struct Oracle {
    O2eParams P;
    int N = 0, N_assoc = 0, NPC = 0;
    long long S = 0;
    // topology
    std::vector<int32_t> row_ptr;    // pre-major CSR, N+1
    std::vector<int32_t> col_idx;    // post per synapse
    std::vector<uint8_t> delay;      // raw delay per synapse
    std::vector<Syn> syn;
    std::vector<float> alpha, beta, xpre_mirror, camkii_act, e1, e2, ca_snap;
    std::vector<float> weights_cache;
    std::vector<int32_t> in_ptr, in_syn;  // post-major incoming lists
    // neurons
    std::vector<Neu> neu;
    std::vector<uint8_t> spike;
    std::vector<float> input, nmda_cur, inh;
    std::vector<float> da, ach, ne, ht5;
    // delay ring
    std::vector<std::vector<std::pair<int32_t, float>>> ring;
    int ring_idx = 0;
    // control state
    std::vector<Gate> gate;
    uint32_t byte_hist_nov[256];
    std::vector<int32_t> byte_histogram;   // spikes per byte
    std::vector<int32_t> neuron_byte_counts;
    std::vector<float> w_value, w_pred_diag, baseline_fr, pred_fr, sub_fr;
    std::vector<uint8_t> corpus;
    size_t corpus_pos = 0;
    // counters
    long long step_no = 0;
    long long total_steps = 0, total_spikes = 0, inject_spikes = 0;
    int last_spikes = 0;
    long long arrived_total = 0, dispatched_total = 0, dropped_total = 0;
    long long ltp_visits_total = 0;
    int last_arrived = 0, last_dispatched = 0;
    long long burst_spikes_total = 0;
    int last_byte = -1;
    float M_const_cache = 0.0f;
    // scratch
    std::vector<float> term_in, term_nmda;

    // constants (host computed exactly as the reference's constant folds)
    float dec_nmda, dec_ampa, dec_ca, dec_ca_ff, rec_ff_step, dec_xpre, dec_xpost;
    float fac_ff, rec_ff, fac_exc, rec_exc, fac_inh, rec_inh;
    float U_ff, U_exc, U_inh;              // STP utilisation by class
    float vt, dT, a_ad, b_ad;              // AdEx in the reference's normalised units
    float e1_dec, e2_dec, ca_n_dec, inv_taum, inv_tauw;
    float mod_dec[4];
    float ne_r, ht5_r;
};

// ---------------------------------------------------------------------------
// Topology: src/stage2e/network_init.cu:158-473, parameterised by column count
// ---------------------------------------------------------------------------
void build_topology(Oracle& o) {
    const O2eParams& P = o.P;
    const int NPC = P.l4 + P.l23 + P.l5 + P.l6;
    const int N_assoc = P.n_columns * NPC;
    const int N_pf = P.pf_groups * P.pf_group_size;
    const int N = N_assoc + N_pf;
    o.N = N; o.N_assoc = N_assoc; o.NPC = NPC;
    uint32_t rng = P.seed;
    auto next_rng = [&rng]() -> uint32_t {
        rng ^= rng << 13; rng ^= rng >> 17; rng ^= rng << 5; return rng;
    };
    auto randf = [&](float lo, float hi) -> float {
        float u = pm_div(pm_u2f(next_rng()), 4294967296.0f);
        return pm_add(lo, pm_mul(pm_sub(hi, lo), u));
    };
    auto randi = [&](int lo, int hi) -> int {
        return lo + (int)(next_rng() % (uint32_t)(hi - lo));
    };
    const float w_scale = pm_div(2.0f, sqrtf(200.0f));
    auto layer_of = [&](int off) {
        if (off < P.l4) return REG_L4;
        if (off < P.l4 + P.l23) return REG_L23;
        if (off < P.l4 + P.l23 + P.l5) return REG_L5;
        return REG_L6;
    };
    auto layer_off = [&](int L) {
        switch (L) {
            case REG_L4: return 0;
            case REG_L23: return P.l4;
            case REG_L5: return P.l4 + P.l23;
            case REG_L6: return P.l4 + P.l23 + P.l5;
        }
        return 0;
    };
    auto layer_sz = [&](int L) {
        switch (L) {
            case REG_L4: return P.l4;
            case REG_L23: return P.l23;
            case REG_L5: return P.l5;
            case REG_L6: return P.l6;
        }
        return 0;
    };
    std::vector<int> out_deg(N, 0);
    long long total = 0;
    for (int pre = 0; pre < N; ++pre) {
        int deg;
        if (pre < N_assoc) {
            int L = layer_of(pre % NPC);
            deg = P.deg_intra;
            if (L == REG_L23) deg += P.deg_inter;
            if (L == REG_L5) deg += P.deg_l5_pf;
        } else {
            deg = P.deg_pf_self + P.deg_pf_assoc;
        }
        out_deg[pre] = deg;
        total += deg;
    }
    while (total < P.total_synapses) { out_deg[randi(0, N_assoc)]++; total++; }
    while (total > P.total_synapses) {
        int pre = randi(0, N_assoc);
        if (out_deg[pre] > 50) { out_deg[pre]--; total--; }
    }
    const long long S = total;
    o.S = S;
    o.row_ptr.assign(N + 1, 0);
    for (int i = 0; i < N; ++i) o.row_ptr[i + 1] = o.row_ptr[i] + out_deg[i];
    o.col_idx.assign(S, 0);
    o.delay.assign(S, 0);
    o.syn.assign(S, Syn{});
    o.alpha.assign(S, 0.0f);
    o.beta.assign(S, 0.0f);
    o.weights_cache.assign(S, 0.0f);
    auto pick_layer = [&](int L) -> int {
        if (L == REG_L4) return REG_L23;
        if (L == REG_L23) return (next_rng() & 1) ? REG_L23 : REG_L5;
        if (L == REG_L5) return (next_rng() & 1) ? REG_L6 : REG_L23;
        if (L == REG_L6) return (next_rng() & 1) ? REG_L4 : REG_L6;
        return REG_PF;
    };
    auto init_syn = [&](long long idx, int pre, int post, float w, uint8_t d,
                        bool exc, bool ff) {
        Syn& s = o.syn[idx];
        s.pre = pre; s.post = post; s.weight = w; s.delay_f = pm_i2f(d);
        s.last_pre = -1000.0f; s.last_post = -1000.0f;
        s.x_pre = 0; s.x_post = 0; s.nmda = 0; s.ampa = 0; s.ca = 0; s.R = 1.0f;
        s.u = ff ? 0.02f : (exc ? 0.2f : 0.05f);
        s.elig = 0; s.elig_slow = 0; s.scaling = 1.0f; s.autop = 0;
        s.da_r = exc ? 0.5f : -0.3f; s.ach_r = 0.3f;
        uint8_t fl = exc ? 0x03 : 0x0C;
        if (ff) fl |= FLAG_FF;
        s.flags = fl;
        s.ne_u8 = (uint8_t)pm_mul(0.3f, 127.0f);
        s.ht5_u8 = (uint8_t)pm_mul(0.3f, 127.0f);
        s.pad = 0;
        float ratio = pm_div(fabsf(w), 1.5f);
        if (ratio > 0.999f) ratio = 0.999f;
        o.alpha[idx] = pm_mul(ratio, 0.1f);
        o.beta[idx] = pm_mul(pm_sub(1.0f, ratio), 0.1f);
        o.weights_cache[idx] = w;
        o.delay[idx] = d;
        o.col_idx[idx] = post;
    };
    for (int pre = 0; pre < N; ++pre) {
        long long start = o.row_ptr[pre];
        int deg = out_deg[pre];
        int nw = 0;
        bool is_pf = pre >= N_assoc;
        int pre_col = is_pf ? -1 : pre / NPC;
        int pre_off = is_pf ? 0 : pre % NPC;
        int L = is_pf ? REG_PF : layer_of(pre_off);
        int l_size, l_off;
        if (is_pf) { l_size = P.pf_group_size; l_off = (pre - N_assoc) % P.pf_group_size; }
        else { l_size = layer_sz(L); l_off = pre_off - layer_off(L); }
        int exc_count = (int)(pm_mul(pm_i2f(l_size), 0.8f));
        bool exc = l_off < exc_count;
        int n_intra = is_pf ? P.deg_pf_self : P.deg_intra;
        int n_inter = (L == REG_L23) ? P.deg_inter : 0;
        int n_pf = is_pf ? P.deg_pf_assoc : (L == REG_L5 ? P.deg_l5_pf : 0);
        auto intra_one = [&](bool pf_any) {
            int post; bool ff = false;
            if (is_pf) {
                if (pf_any) post = N_assoc + randi(0, N_pf);
                else {
                    int gb = N_assoc + ((pre - N_assoc) / P.pf_group_size) * P.pf_group_size;
                    post = gb + randi(0, P.pf_group_size);
                }
            } else {
                int cb = pre_col * NPC;
                int TL = pick_layer(L);
                post = cb + layer_off(TL) + randi(0, layer_sz(TL));
                ff = (L == REG_L4 && TL == REG_L23) || (L == REG_L23 && TL == REG_L5) ||
                     (L == REG_L5 && TL == REG_L6);
            }
            if (post == pre) post = (post + 1) % N;
            float wmin = ff ? 2.5f : 0.4f, wmax = ff ? 3.5f : 1.0f;
            float w = exc ? pm_mul(randf(wmin, wmax), w_scale)
                          : pm_mul(randf(-wmax, -wmin), w_scale);
            uint8_t d = (uint8_t)randi(1, 4);
            init_syn(start + nw, pre, post, w, d, exc, ff);
            nw++;
        };
        for (int k = 0; k < n_intra && nw < deg; ++k) intra_one(false);
        for (int k = 0; k < n_inter && nw < deg; ++k) {
            int tc = randi(0, P.n_columns);
            if (tc == pre_col) tc = (tc + 1) % P.n_columns;
            int post = tc * NPC + layer_off(REG_L23) + randi(0, P.l23);
            float w = exc ? pm_mul(randf(0.05f, 0.15f), w_scale)
                          : pm_mul(randf(-0.15f, -0.05f), w_scale);
            uint8_t d = (uint8_t)randi(5, 11);
            init_syn(start + nw, pre, post, w, d, exc, false);
            nw++;
        }
        for (int k = 0; k < n_pf && nw < deg; ++k) {
            int post; uint8_t d;
            if (is_pf) {
                post = randi(0, N_assoc);
                d = (uint8_t)randi(15, 21);
            } else {
                int g = randi(0, P.pf_groups);
                post = N_assoc + g * P.pf_group_size + randi(0, P.pf_group_size);
                d = (uint8_t)randi(15, 21);
            }
            float w = exc ? pm_mul(randf(0.6f, 1.2f), w_scale)
                          : pm_mul(randf(-1.2f, -0.6f), w_scale);
            init_syn(start + nw, pre, post, w, d, exc, false);
            nw++;
        }
        while (nw < deg) intra_one(true);
    }
}

// src/stage2e/network_init.cu:38-127
void init_neurons(Oracle& o) {
    const O2eParams& P = o.P;
    o.neu.assign(o.N, Neu{});
    for (int i = 0; i < o.N; ++i) {
        Neu& n = o.neu[i];
        n.V = 0; n.s = 0; n.nmda_cur = 0; n.w = 0; n.last = -1000; n.fr = 0;
        n.ref = 0; n.ca = 0; n.wm = 0; n.hf = 1.0f; n.off = 0; n.r0 = n.r1 = 0;
        if (i < o.N_assoc) {
            int col = i / o.NPC, off = i % o.NPC;
            n.column = (uint8_t)(col < 255 ? col : 254);  // reference stores uint8 (50 columns)
            n.pf_group = -1;
            int lo, ls;
            if (off < P.l4) { n.region = REG_L4; lo = off; ls = P.l4; }
            else if (off < P.l4 + P.l23) { n.region = REG_L23; lo = off - P.l4; ls = P.l23; }
            else if (off < P.l4 + P.l23 + P.l5) { n.region = REG_L5; lo = off - P.l4 - P.l23; ls = P.l5; }
            else { n.region = REG_L6; lo = off - P.l4 - P.l23 - P.l5; ls = P.l6; }
            int exc = (int)pm_mul(pm_i2f(ls), 0.8f);
            if (lo < exc) { n.type = 0; n.subtype = 0; }
            else {
                n.type = 1;
                float frac = pm_div(pm_i2f(lo - exc), pm_i2f(ls - exc));
                if (frac < 0.5f) n.subtype = 1;
                else if (frac < pm_add(0.5f, 0.3f)) n.subtype = 2;
                else n.subtype = 3;
            }
        } else {
            int pi = i - o.N_assoc;
            n.column = 255; n.region = REG_PF; n.pf_group = (int16_t)(pi / P.pf_group_size);
            int og = pi % P.pf_group_size;
            int exc = (int)pm_mul(pm_i2f(P.pf_group_size), 0.8f);
            if (og < exc) { n.type = 0; n.subtype = 0; } else { n.type = 1; n.subtype = 1; }
        }
    }
}

int column_of(const Oracle& o, int i) { return i < o.N_assoc ? i / o.NPC : -1; }

void setup(Oracle& o) {
    build_topology(o);
    init_neurons(o);
    const int N = o.N;
    const long long S = o.S;
    // post-major incoming lists, ascending synapse id
    o.in_ptr.assign(N + 1, 0);
    for (long long s = 0; s < S; ++s) o.in_ptr[o.col_idx[s] + 1]++;
    for (int i = 0; i < N; ++i) o.in_ptr[i + 1] += o.in_ptr[i];
    o.in_syn.assign(S, 0);
    {
        std::vector<int32_t> fill(o.in_ptr.begin(), o.in_ptr.end() - 1);
        for (long long s = 0; s < S; ++s) o.in_syn[fill[o.col_idx[s]]++] = (int32_t)s;
    }
    o.xpre_mirror.assign(S, 0.0f);
    o.camkii_act.assign(S, 0.0f);
    o.e1.assign(S, 0.0f);
    o.e2.assign(S, 0.0f);
    o.ca_snap.assign(S, 0.0f);
    o.term_in.assign(S, 0.0f);
    o.term_nmda.assign(S, 0.0f);
    o.spike.assign(N, 0);
    o.input.assign(N, 0.0f);
    o.nmda_cur.assign(N, 0.0f);
    o.inh.assign(N, 0.0f);
    o.da.assign(N, 0.0f); o.ach.assign(N, 0.0f); o.ne.assign(N, 0.0f); o.ht5.assign(N, 0.0f);
    o.ring.assign(20, {});
    o.gate.assign(o.P.n_columns, Gate{0.5f, 0.0f, 0.0f, 0.0f});
    memset(o.byte_hist_nov, 0, sizeof(o.byte_hist_nov));
    o.byte_histogram.assign(256, 0);
    o.neuron_byte_counts.assign((size_t)N * 256, 0);
    o.w_value.assign(200, 0.0f); o.w_pred_diag.assign(200, 0.0f);
    o.baseline_fr.assign(200, 0.0f); o.pred_fr.assign(200, 0.0f); o.sub_fr.assign(200, 0.0f);
    // constants (src/stage2e/synapse_kernels.cu:72-92,176-177,371-372,530-531;
    // neuron_kernels.cu:117-156; modulatory_kernels.cu:205-208)
    o.dec_nmda = snn_expf(pm_div(-1.0f, 150.0f));
    o.dec_ampa = snn_expf(pm_div(-1.0f, 5.0f));
    o.dec_ca = snn_expf(pm_div(-1.0f, 50.0f));
    o.dec_ca_ff = snn_expf(pm_div(-1.0f, 10.0f));
    o.rec_ff_step = pm_sub(1.0f, snn_expf(pm_div(-1.0f, 3.0f)));
    o.dec_xpre = snn_expf(pm_div(-1.0f, 20.0f));
    o.dec_xpost = snn_expf(pm_div(-1.0f, 20.0f));
    o.fac_ff = snn_expf(pm_div(-1.0f, 200.0f));
    o.rec_ff = pm_sub(1.0f, snn_expf(pm_div(-1.0f, 3.0f)));
    o.fac_exc = snn_expf(pm_div(-1.0f, 200.0f));
    o.rec_exc = pm_sub(1.0f, snn_expf(pm_div(-1.0f, 500.0f)));
    o.fac_inh = o.fac_exc;
    o.rec_inh = o.rec_exc;
    o.e1_dec = snn_expf(pm_div(-10.0f, 20.0f));
    o.e2_dec = snn_expf(pm_div(-10.0f, 200.0f));
    o.ca_n_dec = pm_sub(1.0f, pm_div(1.0f, 50.0f));
    o.inv_taum = pm_div(1.0f, 9.37f);
    o.inv_tauw = pm_div(1.0f, 144.0f);
    o.U_ff = 0.02f; o.U_exc = 0.2f; o.U_inh = 0.05f;
    o.vt = 0.8f; o.dT = 0.1f; o.a_ad = 0.0133f; o.b_ad = 0.0805f;
    if (o.P.preset == 1) {
        // benchmark constants (C 200 pF, gL 10 nS, EL -70 mV, VT -50 mV, dT 2 mV,
        // a 2 nS, b 0.08 nA, tau_w 100 ms, dt 1 ms) in the reference's units:
        // v = (V - EL) / 25 mV (VT -> 0.8, spike at 1), w in gL * 25 mV;
        // STP U 0.5, tau_d 200, tau_f 50 for every class (FF per-step recovery too)
        o.inv_taum = pm_div(1.0f, 20.0f);
        o.inv_tauw = pm_div(1.0f, 100.0f);
        o.vt = 0.8f; o.dT = 0.08f; o.a_ad = 0.2f; o.b_ad = 0.32f;
        o.U_ff = o.U_exc = o.U_inh = 0.5f;
        o.fac_ff = o.fac_exc = o.fac_inh = snn_expf(pm_div(-1.0f, 50.0f));
        o.rec_ff = o.rec_exc = o.rec_inh = pm_sub(1.0f, snn_expf(pm_div(-1.0f, 200.0f)));
        o.rec_ff_step = o.rec_ff;
        for (auto& sy : o.syn) sy.u = 0.5f;
    }
    o.mod_dec[0] = snn_expf(pm_div(-100.0f, 100.0f));
    o.mod_dec[1] = snn_expf(pm_div(-100.0f, 200.0f));
    o.mod_dec[2] = snn_expf(pm_div(-100.0f, 150.0f));
    o.mod_dec[3] = snn_expf(pm_div(-100.0f, 300.0f));
    o.ne_r = pm_div(pm_u2f(38u), 127.0f);
    o.ht5_r = o.ne_r;
}

// canonical sum (1) over the incoming list of post j: 32 strided partial sums
// (partial l adds incoming positions l, l+32, l+64, ... in ascending order,
// starting from +0), then the xor butterfly over the 32 partials
float canon_sum(const Oracle& o, int j, const std::vector<float>& term) {
    const int b = o.in_ptr[j], e = o.in_ptr[j + 1];
    float v[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int p = b + l; p < e; p += 32) acc = pm_add(acc, term[o.in_syn[p]]);
        v[l] = acc;
    }
    return tree32(v);
}

// M_ij = sigmoid(receptor . concentration), src/stage2e/synapse_kernels.cu:207-211
inline float m_ij(const Oracle& o, const Syn& s, int post) {
    float z = pm_mul(s.da_r, o.da[post]);
    z = pm_fma(s.ach_r, o.ach[post], z);
    z = pm_fma(pm_div(pm_u2f(s.ne_u8), 127.0f), o.ne[post], z);
    z = pm_fma(pm_div(pm_u2f(s.ht5_u8), 127.0f), o.ht5[post], z);
    return pm_div(1.0f, pm_add(1.0f, snn_expf(-z)));
}

inline float w_of(float a, float b, uint8_t flags) {
    float m = pm_div(pm_mul(1.5f, a), pm_add(a, b));
    return (flags & 0x03) ? m : -m;
}

uint8_t byte_for_step(Oracle& o, long long step) {
    if (!o.corpus.empty()) {
        uint8_t b = o.corpus[o.corpus_pos];
        o.corpus_pos = (o.corpus_pos + 1) % o.corpus.size();
        return b;
    }
    return (uint8_t)((step / 3) % 256);
}

void step(Oracle& o) {
    const int N = o.N;
    const long long S = o.S;
    const long long t = o.step_no;
    const int ncol = o.P.n_columns;
    const int ph = phase_of(t + o.P.phase_offset);
    const float gain = PH_GAIN[ph];
    const bool e0 = o.P.e0 != 0;

    // 1. delay inject (neuron_kernels.cu:234-260): input = canonical sum of arrivals
    std::vector<std::pair<int32_t, float>> arrived;
    arrived.swap(o.ring[o.ring_idx]);
    for (auto& a : arrived) o.term_in[a.first] = a.second;
#pragma omp parallel for schedule(static)
    for (int j = 0; j < N; ++j) o.input[j] = canon_sum(o, j, o.term_in);
    for (auto& a : arrived) o.term_in[a.first] = 0.0f;
    o.last_arrived = (int)arrived.size();
    o.arrived_total += (long long)arrived.size();

    // 1.5 column / L6 counts of the previous step + thalamic gate (scheduler.cu:501-523)
    std::vector<int> col_sp(ncol, 0), l6_sp(ncol, 0);
    for (int i = 0; i < o.N_assoc; ++i)
        if (o.spike[i]) {
            int c = i / o.NPC;
            col_sp[c]++;
            if (o.neu[i].region == REG_L6) l6_sp[c]++;
        }
    const bool inject = (t % 3) == 0;
    int byte = 0;
    if (inject) byte = byte_for_step(o, t);
    o.last_byte = inject ? byte : -1;
    {   // thalamic_gate.cu:53-142 with canonical novelty (4)
        uint32_t total_h = 0;
        for (int b = 0; b < 256; ++b) total_h += o.byte_hist_nov[b];
        uint32_t bc = o.byte_hist_nov[byte];
        for (int c = 0; c < ncol; ++c) {
            Gate& g = o.gate[c];
            float cur = pm_i2f(col_sp[c]);
            float den = g.act_ema > 1.0f ? g.act_ema : 1.0f;
            float an = fminf(1.0f, fmaxf(-1.0f, pm_div(pm_sub(g.act_ema, cur), den)));
            float l6c = pm_i2f(l6_sp[c]);
            float l6d = g.l6_ema > 1.0f ? g.l6_ema : 1.0f;
            float l6n = fminf(1.0f, fmaxf(-1.0f, pm_div(pm_sub(g.l6_ema, l6c), l6d)));
            float nov = 0.0f;
            if (inject) {
                uint32_t tm = total_h > 1u ? total_h : 1u;
                nov = pm_sub(1.0f, pm_div(pm_u2f(bc), pm_u2f(tm)));
                nov = fminf(1.0f, fmaxf(0.0f, nov));
            }
            const float one_m_99 = pm_sub(1.0f, 0.99f), one_m_95 = pm_sub(1.0f, 0.95f);
            g.act_ema = pm_fma(0.99f, g.act_ema, pm_mul(one_m_99, cur));
            g.l6_ema = pm_fma(0.99f, g.l6_ema, pm_mul(one_m_99, l6c));
            g.nov_ema = pm_fma(0.95f, g.nov_ema, pm_mul(one_m_95, nov));
            float tg = pm_fma(0.3f, an, 0.5f);
            tg = pm_fma(0.2f, g.nov_ema, tg);
            tg = pm_fma(0.15f, l6n, tg);
            tg = fminf(0.9f, fmaxf(0.1f, tg));
            g.gate = pm_fma(0.01f, pm_sub(tg, g.gate), g.gate);
            g.gate = fminf(1.0f, fmaxf(0.0f, g.gate));
        }
        if (inject) o.byte_hist_nov[byte] += (uint32_t)ncol;
    }

    // 2. population-coded input (input_encoding.cu:117-164)
    if (inject) {
        const int pref = 256 / ncol;
        for (int c = 0; c < ncol; ++c) {
            int ps = c * pref, pe = ps + pref;
            bool in_r = (byte >= ps && byte < pe);
            float g = in_r ? 2.0f : 0.03f;
            float v = pm_mul(pm_mul(80.0f, g), o.gate[c].gate);
            uint32_t h = (uint32_t)byte * 2654435761u + (uint32_t)c * 0x9E3779B9u;
            for (int k = 0; k < 100; ++k) {
                h ^= h << 13; h ^= h >> 17; h ^= h << 5;
                int n = c * o.NPC + (int)(h % (uint32_t)o.P.l4);
                o.input[n] = pm_add(o.input[n], v);
            }
        }
    }

    // 3. AdEx (neuron_kernels.cu:61-165)
    int burst = 0;
    for (int i = 0; i < N; ++i) {
        Neu& n = o.neu[i];
        if (n.ref > 0) {
            n.ref--; o.spike[i] = 0; n.fr = pm_mul(n.fr, 0.99f);
            continue;
        }
        n.s = pm_fma(n.s, 0.7f, pm_mul(o.input[i], 0.3f));
        float I = pm_sub(pm_add(n.s, o.nmda_cur[i]), o.inh[i]);
        float V = n.V, w = n.w;
        float ea = pm_div(pm_sub(V, o.vt), o.dT);
        if (ea > 10.0f) ea = 10.0f;
        if (ea < -10.0f) ea = -10.0f;
        float et = pm_mul(o.dT, snn_expf(ea));
        float dV = pm_mul(pm_add(pm_sub(pm_add(-V, et), w), I), o.inv_taum);
        float dw = pm_mul(pm_fma(o.a_ad, V, -w), o.inv_tauw);
        V = pm_add(V, dV);
        w = pm_add(w, dw);
        if (V < -0.5f) V = -0.5f;
        if (V > 1.5f) V = 1.5f;
        float theta = pm_add(1.0f, pm_div(pm_u2f(n.off), 256.0f));
        bool sp = V >= theta;
        o.spike[i] = sp;
        if (sp) {
            if (n.last >= 0 && t - n.last <= 5) burst++;
            n.last = (int32_t)t;
            n.ref = 2;
            V = 0.0f;
            w = pm_add(w, o.b_ad);
            n.ca = fminf(pm_add(n.ca, 0.2f), 1.0f);
            n.fr = pm_fma(n.fr, 0.9f, 0.1f);
            int no = (int)n.off + (int)pm_mul(0.001f, 256.0f);
            int mo = (int)pm_mul(0.3f, 256.0f);
            if (no > mo) no = mo;
            n.off = (uint16_t)no;
        } else {
            n.off = (uint16_t)pm_mul(pm_u2f(n.off), 0.999f);
            n.ca = pm_mul(n.ca, o.ca_n_dec);
            n.fr = pm_mul(n.fr, 0.995f);
        }
        n.V = V;
        n.w = w;
    }
    o.burst_spikes_total += burst;

    // byte statistics on inject steps (modulatory_kernels.cu:150-161, scheduler.cu:99-110)
    if (inject) {
        for (int i = 0; i < N; ++i)
            if (o.spike[i]) {
                o.byte_histogram[byte]++;
                o.neuron_byte_counts[(size_t)i * 256 + byte]++;
            }
    }

    // 4. arrival conductance + dense NMDA / Ca (synapse_kernels.cu:123-141, 45-121)
    for (auto& a : arrived) {
        Syn& s = o.syn[a.first];
        s.ampa = pm_fma(pm_mul(1.0f, s.R), s.u, s.ampa);
        if (s.flags & 0x02) s.nmda = pm_fma(pm_mul(0.5f, s.R), s.u, s.nmda);
    }
    std::vector<float> mg(N), Vn(N);
    for (int j = 0; j < N; ++j) {
        float V = o.neu[j].V;
        float Vb = pm_fma(50.0f, V, -70.0f);
        float e = snn_expf(pm_div(-Vb, 16.13f));
        mg[j] = pm_div(1.0f, pm_add(1.0f, pm_div(pm_mul(1.0f, e), 3.57f)));
        Vn[j] = V;
    }
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < S; ++i) {
        Syn& s = o.syn[i];
        const int post = s.post;
        const float m = mg[post];
        const bool ff = (s.flags & FLAG_FF) != 0;
        s.nmda = pm_mul(s.nmda, o.dec_nmda);
        s.ampa = pm_mul(s.ampa, o.dec_ampa);
        s.ca = pm_mul(s.ca, ff ? o.dec_ca_ff : o.dec_ca);
        if (ff) s.R = pm_fma(pm_sub(1.0f, s.R), o.rec_ff_step, s.R);
        float nm = pm_mul(s.nmda, m);
        s.ca = pm_fma(nm, 1000.0f, s.ca);
        float cmax = ff ? 0.12f : 1.0f;
        if (s.ca > cmax) s.ca = cmax;
        o.ca_snap[i] = s.ca;
        float term = 0.0f;
        if (s.flags & 0x02) {
            float I = pm_mul(pm_mul(nm, pm_sub(1.4f, Vn[post])), 0.05f);
            if (fabsf(I) > 1e-6f) term = I;
        }
        o.term_nmda[i] = term;
    }
#pragma omp parallel for schedule(static)
    for (int j = 0; j < N; ++j) o.nmda_cur[j] = canon_sum(o, j, o.term_nmda);

    // 5. dual-trace STDP, dense then arrivals (synapse_kernels.cu:153-329)
    long long ltp_visits = 0;
#pragma omp parallel for schedule(static) reduction(+ : ltp_visits)
    for (long long i = 0; i < S; ++i) {
        Syn& s = o.syn[i];
        const int post = s.post;
        const bool ps = o.spike[post] != 0;
        s.x_pre = pm_mul(s.x_pre, o.dec_xpre);
        s.x_post = pm_mul(s.x_post, o.dec_xpost);
        float dw = 0.0f;
        if (ps) { dw = pm_fma(s.x_pre, 0.03f, 0.0f); ltp_visits++; }
        if (ps) { s.x_post = pm_add(s.x_post, 0.03f); s.last_post = pm_ll2f(t); }
        const bool ff = (s.flags & FLAG_FF) != 0;
        const float eta = ff ? 2.0f : 20.0f;
        float M = 1.0f, pf = 1.0f;
        bool need = (dw > 0.0f) || (ps && s.ca > 0.15f);
        if (need && !e0) { M = m_ij(o, s, post); pf = pm_sub(1.0f, pm_mul(0.5f, s.autop)); }
        float& a = o.alpha[i];
        float& b = o.beta[i];
        if (dw > 0.0f) a = pm_fma(pm_mul(pm_mul(pm_mul(eta, dw), gain), M), pf, a);
        if (ps && s.ca > 0.15f) {
            float ex = pm_sub(s.ca, 0.15f);
            b = pm_fma(pm_mul(pm_mul(pm_mul(eta, ex), 0.5f), gain), M, b);
        }
        if (a < 1e-4f) a = 1e-4f;
        if (b < 1e-4f) b = 1e-4f;
        s.weight = w_of(a, b, s.flags);
        s.elig = pm_add(s.elig, dw);
        o.xpre_mirror[i] = s.x_pre;
    }
    o.ltp_visits_total += ltp_visits;
    for (auto& ar : arrived) {
        const long long i = ar.first;
        Syn& s = o.syn[i];
        const int post = s.post;
        float dw = pm_mul(-s.x_post, 0.03f);
        s.x_pre = pm_add(s.x_pre, 0.03f);
        s.last_pre = pm_ll2f(t);
        const bool ff = (s.flags & FLAG_FF) != 0;
        const float eta = ff ? 2.0f : 20.0f;
        float M = 1.0f, pf = 1.0f;
        if (dw != 0.0f && !e0) { M = m_ij(o, s, post); pf = pm_sub(1.0f, pm_mul(0.5f, s.autop)); }
        float& a = o.alpha[i];
        float& b = o.beta[i];
        if (dw > 0.0f) a = pm_fma(pm_mul(pm_mul(pm_mul(eta, dw), gain), M), pf, a);
        else if (dw < 0.0f) b = pm_fma(pm_mul(pm_mul(pm_mul(eta, -dw), gain), M), pf, b);
        if (a < 1e-4f) a = 1e-4f;
        if (b < 1e-4f) b = 1e-4f;
        s.weight = w_of(a, b, s.flags);
        s.elig = pm_add(s.elig, dw);
        o.xpre_mirror[i] = s.x_pre;
    }

    // 6. STP on arrivals (synapse_kernels.cu:334-387)
    for (auto& ar : arrived) {
        Syn& s = o.syn[ar.first];
        float U, fac, rec;
        if (s.flags & FLAG_FF) { U = o.U_ff; fac = o.fac_ff; rec = o.rec_ff; }
        else if (s.flags & 0x03) { U = o.U_exc; fac = o.fac_exc; rec = o.rec_exc; }
        else { U = o.U_inh; fac = o.fac_inh; rec = o.rec_inh; }
        s.R = pm_fma(pm_sub(1.0f, s.R), rec, s.R);
        s.u = pm_fma(pm_sub(s.u, U), fac, U);
        float un = pm_fma(U, pm_sub(1.0f, s.u), s.u);
        float rn = pm_mul(s.R, pm_sub(1.0f, un));
        s.u = un; s.R = rn;
        if (s.u > 1.0f) s.u = 1.0f;
        if (s.R < 0.0f) s.R = 0.0f;
    }

    // 7. dispatch (neuron_kernels.cu:170-209)
    int disp = 0;
    for (int pre = 0; pre < N; ++pre) {
        if (!o.spike[pre]) continue;
        for (int i = o.row_ptr[pre]; i < o.row_ptr[pre + 1]; ++i) {
            int d = o.delay[i];
            if (d < 1) d = 1;
            if (d >= 20) d = 19;
            int slot = (o.ring_idx + d) % 20;
            if (o.ring[slot].size() >= 750000) o.dropped_total++;  // reference would drop it
            o.ring[slot].push_back({i, pm_mul(o.syn[i].weight, o.syn[i].R)});
            disp++;
        }
    }
    o.last_dispatched = disp;
    o.dispatched_total += disp;
    // 8. inhibitory current cleared (scheduler.cu:569-571)
    std::fill(o.inh.begin(), o.inh.end(), 0.0f);

    int cur_spikes = 0;
    for (int i = 0; i < N; ++i) cur_spikes += o.spike[i];

    // 9. every 10 steps (scheduler.cu:576-582, 688-722)
    if (t % 10 == 0) {
        if (!e0) {
#pragma omp parallel for schedule(static)
            for (long long i = 0; i < S; ++i) {
                Syn& s = o.syn[i];
                float ca = s.ca, act = o.camkii_act[i], au = s.autop;
                float ca4 = pm_mul(pm_mul(pm_mul(ca, ca), ca), ca);
                float d_act = pm_fma(pm_mul(0.8f, ca4), pm_sub(1.0f, act),
                                     -pm_mul(pm_mul(0.1f, act), 0.5f));
                float d_au = pm_fma(pm_mul(pm_mul(0.5f, act), act), pm_sub(1.0f, au),
                                    -pm_mul(pm_mul(0.05f, au), 0.5f));
                act = pm_fma(d_act, 10.0f, act);
                au = pm_fma(d_au, 10.0f, au);
                act = fclampf(act, 0.0f, 1.0f);
                au = fclampf(au, 0.0f, 1.0f);
                o.camkii_act[i] = act;
                s.autop = au;
            }
#pragma omp parallel for schedule(static)
            for (long long i = 0; i < S; ++i) {
                Syn& s = o.syn[i];
                float a1 = pm_fma(o.e1[i], o.e1_dec, s.elig);
                float a2 = pm_fma(o.e2[i], o.e2_dec, a1);
                s.elig = 0.0f;
                o.e1[i] = a1;
                o.e2[i] = a2;
            }
        }
        float avg = o.total_steps > 0 ? pm_div(pm_ll2f(o.total_spikes), pm_ll2f(o.total_steps)) : 0.0f;
        float drive = pm_div(pm_i2f(o.last_spikes), pm_add(avg, 1.0f));
        drive = fclampf(drive, 0.0f, 2.0f);
        float gdrive = pm_mul(drive, 0.15f);
        for (int i = 0; i < N; ++i) {
            const Neu& n = o.neu[i];
            float sg = 1.0f;
            if (n.subtype == 0) sg = 1.40f;
            else if (n.subtype == 1) sg = 0.85f;
            else if (n.subtype == 2) sg = 1.10f;
            float rg = (n.region == REG_PF) ? 0.60f : 1.0f;
            float ld = pm_fma(n.fr, 2.0f, gdrive);
            float c = pm_mul(pm_mul(ld, sg), rg);
            if (n.type == 1) c = pm_mul(c, 0.35f);
            if (c > 2.0f) c = 2.0f;
            o.inh[i] = c;
        }
        std::vector<int> cs(ncol, 0);
        for (int i = 0; i < o.N_assoc; ++i) if (o.spike[i]) cs[i / o.NPC]++;
        float apc = pm_div(avg, pm_i2f(ncol));
        int k = (int)pm_mul(apc, 0.5f);
        if (k < 3) k = 3;
        if (k > 5) k = 5;
        int width = k * 8;
        if (width < 1) width = 1;
        if (width > o.NPC) width = o.NPC;
        for (int i = 0; i < o.N_assoc; ++i) {
            int col = i / o.NPC;
            int sp = cs[col];
            if (sp <= 0) continue;
            int rank = (i + col * 37) % o.NPC;
            if (sp > k && rank >= width) {
                float pr = pm_div(pm_i2f(sp - k), pm_i2f(k + 1));
                float ex = pm_mul(0.35f, pr);
                if (ex > 2.0f) ex = 2.0f;
                o.inh[i] = pm_add(o.inh[i], ex);
            }
        }
    }

    // 10. every 100 steps: modulators + TD value function (scheduler.cu:724-751)
    if (t % 100 == 0 && !e0) {
        float avg = o.total_steps > 0 ? pm_div(pm_ll2f(o.total_spikes), pm_ll2f(o.total_steps)) : 0.0f;
        float cur = pm_i2f(o.last_spikes);
        float nov = avg > 0.0f ? pm_div(fabsf(pm_sub(cur, avg)), pm_add(avg, 1.0f)) : 0.0f;
        if (nov > 1.0f) nov = 1.0f;
        float pred = (cur > 10.0f && cur < 1000.0f) ? 0.5f : 0.1f;
        float reward = pm_add(pm_mul(0.5f, nov), pm_mul(0.3f, pred));
        const int per = N / 200;
        for (int sc = 0; sc < 200; ++sc) {
            int st = sc * per, en = st + per;
            if (en > N) en = N;
            int cnt = 0;
            for (int i = st; i < en; ++i) cnt += o.spike[i];
            o.sub_fr[sc] = pm_div(pm_i2f(cnt), pm_i2f(per));
        }
        float vs = 0.0f;
        for (int k = 0; k < 200; ++k) vs = pm_fma(o.w_value[k], o.sub_fr[k], vs);
        const float one_m_99 = pm_sub(1.0f, 0.99f);
        for (int k = 0; k < 200; ++k) {
            o.baseline_fr[k] = pm_fma(0.99f, o.baseline_fr[k], pm_mul(one_m_99, o.sub_fr[k]));
            o.pred_fr[k] = pm_mul(o.w_pred_diag[k], o.sub_fr[k]);
        }
        float vsp = 0.0f;
        for (int k = 0; k < 200; ++k) vsp = pm_fma(o.w_value[k], o.pred_fr[k], vsp);
        float delta = pm_sub(pm_add(reward, pm_mul(0.9f, vsp)), vs);
        for (int k = 0; k < 200; ++k) {
            float wv = pm_fma(pm_mul(0.001f, delta), o.sub_fr[k], o.w_value[k]);
            wv = fclampf(wv, -1.0f, 1.0f);
            o.w_value[k] = wv;
            float pe = pm_sub(o.sub_fr[k], o.baseline_fr[k]);
            o.w_pred_diag[k] = pm_fma(pm_mul(0.001f, pe), o.sub_fr[k], o.w_pred_diag[k]);
        }
        float da_sig = pm_add(0.1f, delta > 0.0f ? delta : pm_mul(0.3f, delta));
        if (da_sig < 0.0f) da_sig = 0.0f;
        float ach_sig = pm_add(pm_add(0.2f, pm_mul(0.3f, nov)), pm_mul(0.1f, pred));
        float ne_sig = 0.05f;
        float ht_sig = 0.1f;
        if (delta < -0.5f) ht_sig = pm_add(ht_sig, pm_mul(0.3f, fabsf(delta)));
        for (int i = 0; i < N; ++i) {
            o.da[i] = fclampf(pm_fma(o.da[i], o.mod_dec[0], da_sig), 0.0f, 2.0f);
            o.ach[i] = fclampf(pm_fma(o.ach[i], o.mod_dec[1], ach_sig), 0.0f, 2.0f);
            o.ne[i] = fclampf(pm_fma(o.ne[i], o.mod_dec[2], ne_sig), 0.0f, 2.0f);
            o.ht5[i] = fclampf(pm_fma(o.ht5[i], o.mod_dec[3], ht_sig), 0.0f, 2.0f);
        }
    }

    // 11. every 1000 steps: PSW evidence decay (scheduler.cu:55-86, 1038-1058)
    if (t % 1000 == 0) {
        const float thr = PH_PRUNE[ph];
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < S; ++i) {
            float a = pm_mul(o.alpha[i], 0.95f), b = pm_mul(o.beta[i], 0.95f);
            if (a < 1e-4f) a = 1e-4f;
            if (b < 1e-4f) b = 1e-4f;
            if (pm_add(a, b) < thr) { a = 0.05f; b = 0.05f; }
            o.alpha[i] = a; o.beta[i] = b;
            o.syn[i].weight = w_of(a, b, o.syn[i].flags);
        }
    }

    // 12. ring advance + statistics (scheduler.cu:622-670)
    o.ring_idx = (o.ring_idx + 1) % 20;
    o.total_steps++;
    o.total_spikes += cur_spikes;
    if (inject) o.inject_spikes += cur_spikes;
    o.last_spikes = cur_spikes;
    o.step_no++;
}

}  // namespace

// ---------------------------------------------------------------------------
// C API for the test harness (ctypes)
// ---------------------------------------------------------------------------
extern "C" {

struct O2eCounters {
    int64_t step, total_spikes, arrived, dispatched, dropped, ltp_visits, burst_spikes;
    int32_t last_spikes, last_arrived, last_dispatched, last_byte;
    int32_t n_neurons, ring_idx;
    int64_t n_synapses;
};

static void fp_env_strict() {
#if defined(__x86_64__)
    _MM_SET_FLUSH_ZERO_MODE(_MM_FLUSH_ZERO_OFF);
    _MM_SET_DENORMALS_ZERO_MODE(_MM_DENORMALS_ZERO_OFF);
#endif
}

void* o2e_create(const O2eParams* p) {
    fp_env_strict();
    Oracle* o = new Oracle();
    o->P = *p;
    setup(*o);
    return o;
}
void o2e_destroy(void* h) { delete (Oracle*)h; }
void o2e_set_corpus(void* h, const uint8_t* b, int64_t n) {
    Oracle* o = (Oracle*)h;
    o->corpus.assign(b, b + n);
    o->corpus_pos = 0;
}
void o2e_run(void* h, int32_t n_steps) {
    fp_env_strict();
    Oracle* o = (Oracle*)h;
#ifdef _OPENMP
    if (o->P.n_threads > 0) omp_set_num_threads(o->P.n_threads);
#endif
    for (int k = 0; k < n_steps; ++k) step(*o);
}
void o2e_counters(void* h, O2eCounters* c) {
    Oracle* o = (Oracle*)h;
    c->step = o->step_no; c->total_spikes = o->total_spikes;
    c->arrived = o->arrived_total; c->dispatched = o->dispatched_total;
    c->dropped = o->dropped_total; c->ltp_visits = o->ltp_visits_total;
    c->burst_spikes = o->burst_spikes_total;
    c->last_spikes = o->last_spikes; c->last_arrived = o->last_arrived;
    c->last_dispatched = o->last_dispatched; c->last_byte = o->last_byte;
    c->n_neurons = o->N; c->ring_idx = o->ring_idx; c->n_synapses = o->S;
}
// topology export (pre-major): row_ptr[N+1], post[S], delay[S], flags[S]
void o2e_topology(void* h, int32_t* row_ptr, int32_t* post, uint8_t* delay, uint8_t* flags) {
    Oracle* o = (Oracle*)h;
    if (row_ptr) memcpy(row_ptr, o->row_ptr.data(), sizeof(int32_t) * (o->N + 1));
    for (long long s = 0; s < o->S; ++s) {
        if (post) post[s] = o->col_idx[s];
        if (delay) delay[s] = o->delay[s];
        if (flags) flags[s] = o->syn[s].flags;
    }
}
// neuron field export; which: 0 V, 1 s, 2 w, 3 fr, 4 ca, 5 x (input), 6 nmda_cur, 7 inh,
// 8 spike (as float), 9 last (as float), 10 ref (as float)
void o2e_neuron_f32(void* h, int32_t which, float* out) {
    Oracle* o = (Oracle*)h;
    for (int i = 0; i < o->N; ++i) {
        const Neu& n = o->neu[i];
        float v = 0;
        switch (which) {
            case 0: v = n.V; break;
            case 1: v = n.s; break;
            case 2: v = n.w; break;
            case 3: v = n.fr; break;
            case 4: v = n.ca; break;
            case 5: v = o->input[i]; break;
            case 6: v = o->nmda_cur[i]; break;
            case 7: v = o->inh[i]; break;
            case 8: v = o->spike[i] ? 1.0f : 0.0f; break;
            case 9: v = (float)n.last; break;
            case 10: v = (float)n.ref; break;
        }
        out[i] = v;
    }
}
// arrival sum that the next step will start from (ring slot of the next step)
void o2e_next_input(void* h, float* out) {
    Oracle* o = (Oracle*)h;
    for (auto& a : o->ring[o->ring_idx]) o->term_in[a.first] = a.second;
    for (int j = 0; j < o->N; ++j) out[j] = canon_sum(*o, j, o->term_in);
    for (auto& a : o->ring[o->ring_idx]) o->term_in[a.first] = 0.0f;
}
void o2e_spikes(void* h, uint8_t* out) {
    Oracle* o = (Oracle*)h;
    memcpy(out, o->spike.data(), o->N);
}
// synapse field export, pre-major order; which: 0 alpha, 1 beta, 2 weight, 3 x_pre,
// 4 x_post, 5 nmda, 6 ca, 7 R, 8 u, 9 elig, 10 camkii_act, 11 autophos, 12 e1, 13 e2,
// 14 ampa, 15 last_pre
void o2e_synapse_f32(void* h, int32_t which, float* out) {
    Oracle* o = (Oracle*)h;
    for (long long i = 0; i < o->S; ++i) {
        const Syn& s = o->syn[i];
        float v = 0;
        switch (which) {
            case 0: v = o->alpha[i]; break;
            case 1: v = o->beta[i]; break;
            case 2: v = s.weight; break;
            case 3: v = s.x_pre; break;
            case 4: v = s.x_post; break;
            case 5: v = s.nmda; break;
            case 6: v = s.ca; break;
            case 7: v = s.R; break;
            case 8: v = s.u; break;
            case 9: v = s.elig; break;
            case 10: v = o->camkii_act[i]; break;
            case 11: v = s.autop; break;
            case 12: v = o->e1[i]; break;
            case 13: v = o->e2[i]; break;
            case 14: v = s.ampa; break;
            case 15: v = s.last_pre; break;
        }
        out[i] = v;
    }
}
// SCKP v2 file as BioMechanismScheduler::save_checkpoint writes it
// (src/stage2e/scheduler.cu:411-483): u32 magic 0x53434B50, u32 version 2,
// u32 step, u32 n_syn, u32 n_neu, BioSynapse[n_syn] (80 B each, the Syn
// layout above), i32 neuron_byte_counts[n_neu * 256], f32 alpha[n_syn],
// f32 beta[n_syn].  Returns 0, or 2 when the file cannot be written.
int o2e_save_sckp(void* h, const char* path, int32_t step) {
    Oracle* o = (Oracle*)h;
    FILE* fp = fopen(path, "wb");
    if (!fp) return 2;
    const uint32_t hdr[5] = {0x53434B50u, 2u, (uint32_t)step, (uint32_t)o->S, (uint32_t)o->N};
    fwrite(hdr, sizeof(uint32_t), 5, fp);
    fwrite(o->syn.data(), sizeof(Syn), (size_t)o->S, fp);
    fwrite(o->neuron_byte_counts.data(), sizeof(int32_t), (size_t)o->N * 256, fp);
    fwrite(o->alpha.data(), sizeof(float), (size_t)o->S, fp);
    fwrite(o->beta.data(), sizeof(float), (size_t)o->S, fp);
    return fclose(fp) == 0 ? 0 : 2;
}

// control-state export: gates[4*n_columns], modulators[4], byte_histogram[256]
void o2e_control(void* h, float* gates, float* mods, int32_t* byte_hist) {
    Oracle* o = (Oracle*)h;
    if (gates)
        for (int c = 0; c < o->P.n_columns; ++c) {
            gates[4 * c] = o->gate[c].gate; gates[4 * c + 1] = o->gate[c].act_ema;
            gates[4 * c + 2] = o->gate[c].nov_ema; gates[4 * c + 3] = o->gate[c].l6_ema;
        }
    if (mods) { mods[0] = o->da[0]; mods[1] = o->ach[0]; mods[2] = o->ne[0]; mods[3] = o->ht5[0]; }
    if (byte_hist) memcpy(byte_hist, o->byte_histogram.data(), 256 * sizeof(int32_t));
}
void o2e_neuron_byte_counts(void* h, int32_t* out) {
    Oracle* o = (Oracle*)h;
    memcpy(out, o->neuron_byte_counts.data(), o->neuron_byte_counts.size() * sizeof(int32_t));
}
// initial alpha/beta/weights_cache straight from the generator (before any step)
void o2e_init_weights(void* h, float* w, float* a, float* b) {
    Oracle* o = (Oracle*)h;
    if (w) memcpy(w, o->weights_cache.data(), o->S * sizeof(float));
    if (a) memcpy(a, o->alpha.data(), o->S * sizeof(float));
    if (b) memcpy(b, o->beta.data(), o->S * sizeof(float));
}
float o2e_expf(float x) { return snn_expf(x); }
void o2e_expf_array(const float* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = snn_expf(x[i]);
}
uint64_t o2e_fnv64(const void* p, int64_t n) {
    const unsigned char* b = (const unsigned char*)p;
    uint64_t h = 1469598103934665603ull;
    for (int64_t i = 0; i < n; ++i) { h ^= b[i]; h *= 1099511628211ull; }
    return h;
}

}  // extern "C"
