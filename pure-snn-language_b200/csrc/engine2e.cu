// engine2e.cu - Stage 2e engine on sm_100a: AdEx neurons, NMDA/Ca synapses,
// Tsodyks-Markram STP, dual-trace PSW STDP, CaMKII / eligibility, axonal
// delays, thalamic gate, modulators and inhibition, one step = 2 kernels
// (+ the all-gather and the mirror-group kernels between them on column shards):
//
//   k_neurons   (N threads) start of step t (byte, phase gain, M_ij, thalamic
//                           gates), population-coded input, inhibition, AdEx update,
//                           spike history / raster / counters, Mg block and
//                           post trace of the neuron, then the update of the
//                           neuron's outgoing synapse groups (NMDA g, pre
//                           trace, STP) and their per-step view
//   k_synapses  (warp/post) post-major pass over every neuron's incoming
//                           synapses: Ca / NMDA current, LTP (post spike),
//                           LTD (arrival), dispatch value capture, input
//                           current for the next step, CaMKII / eligibility
//                           fold every 10 steps, PSW decay every 1000 steps;
//                           CTA 0 first runs the end of step t (inhibition
//                           drive, modulators / TD value function, statistics,
//                           hand-over of byte history and counters to t + 1)
//
// Semantics follow src/stage2e/scheduler.cu:485-676 step for step; the CPU
// oracle (oracle/oracle2e.cpp) states the same semantics with per-synapse
// state, so bit equality with it also checks the exact invariants used here:
//   - x_post and last_post depend only on the post neuron (one per neuron);
//   - R, u, NMDA g and x_pre depend only on (pre, effective delay, FF flag):
//     one "group" per such triple, updated once per step by the pre's thread;
//   - the weight is 1.5*alpha/(alpha+beta) with the pre's sign, derived when
//     needed instead of stored; inhibitory synapses keep Ca, NMDA g and
//     CaMKII at exactly 0 and are skipped by those updates;
//   - modulator concentrations are identical for every neuron, so M_ij takes
//     one of two values (excitatory / inhibitory pre) per step.
// Delivery is pulled: synapse s of neuron j receives at step T iff its pre
// spiked at T - d_s (32-step spike history per neuron).  The value delivered
// is w*R captured at dispatch; synapses with d >= 2 keep it in an 8-slot
// ring indexed by floor(t_dispatch / 3) mod 8 (the 2-step refractory period
// makes dispatches of one synapse >= 3 steps apart, and d <= 19 keeps at most
// 7 in flight, so slots never collide).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <limits>
#include <memory>
#include <type_traits>
#include <nccl.h>
#include "nccl_dl.h"
#include "ckpt.h"
#include "common.h"
#include "net2e.h"
#include "snn_pmath.h"

namespace snn2e {

constexpr int NCLASS = 3;  // STP classes: 0 feed-forward, 1 excitatory, 2 inhibitory
constexpr int VAL_SLOTS = 8;
constexpr int TD_DIM = 200;

// group view flag bits (view.w holds them as raw bits)
constexpr uint32_t GV_D_MASK = 0x1f, GV_FF = 1u << 5, GV_EXC = 1u << 6, GV_ARR = 1u << 7,
                   GV_NEXT = 1u << 8, GV_DISP = 1u << 9,
                   GV_EV = 1u << 10;  // arrival, dispatch or a ring read for the next step
constexpr int NEU_BLOCK = 128;  // neurons per k_neurons CTA; groups carry their pre's index in it
constexpr int NEU_THREADS = 256;  // k_neurons CTA size: the first NEU_BLOCK threads own a neuron, all update groups
#ifndef NEU_GU
#define NEU_GU 4   // groups per thread in flight in k_neurons
#endif
// packed static group word: d_eff | ff << 5 | exc << 6 | size << 8 | (pre % NEU_BLOCK) << 24
__host__ __device__ inline unsigned gw_size(unsigned m) { return (m >> 8) & 0xffffu; }
__host__ __device__ inline unsigned gw_lpre(unsigned m) { return m >> 24; }

struct Consts {
    // neuron (normalised AdEx, src/stage2e/neuron_kernels.cu:85-165)
    float syn_keep, syn_in, vt, dT, inv_taum, a_ad, inv_tauw, b_ad, vmin, vmax;
    float ca_n_inc, ca_n_dec, fr_refr, fr_spk_keep, fr_spk_add, fr_quiet, off_decay;
    int refr_steps, off_add, off_max;
    // synapse
    float dec_nmda, dec_ampa, dec_ca, dec_ca_ff, ca_max, ca_max_ff, rec_ff_step, dec_xpre, dec_xpost;
    float g_nmda, ca_gain, e_rev, i_gain, i_min;
    float U[NCLASS], fac[NCLASS], rec[NCLASS];
    float a_plus, a_minus, w_max, eta, eta_ff, reb_thr, reb_gain, ab_min, ab_reset, psw_decay;
    float e1_dec, e2_dec;
    float ck_k1, ck_k2, ck_k3, ck_k4, ck_pp1, ck_dt;
    // modulators
    float mod_dec[4], rec_da[2], rec_ach, rec_ne, rec_ht5;
    // input
    float pop_gain, gain_in, gain_out;
    int pop_k, pref_range, inject_interval;
};

struct Ctrl {
    long long next_t, t;
    int inject, byte;
    float gain, prune_thr, M[2];
    float gdrive;
    int kwta_k, inh_active;
    int learn, byte_override, e0, phase_offset;
    long long total_steps, total_spikes, inject_spikes;
    int last_spikes;
    float conc[4];
    long long corpus_len, corpus_pos;
    unsigned long long arrivals, dispatched, ltp_visits, burst, dropped_ref;
    int step_spikes[2];
    unsigned long long step_arrivals[2];
    long long raster_base;  // step whose raster is in row 0
    unsigned hist_total;    // sum of the byte history (novelty denominator)
    int error;              // set by a kernel whose bounded wait ran out
};

struct Dev {
    // neurons
    float *V, *wad, *s, *fr, *can, *xpost, *mg, *input, *nmda_cur;
    int *last, *ref;
    unsigned short* off;
    unsigned* info;  // type | region<<1 | subtype<<4 | column<<8 (0xffffff = PF)
    unsigned* hist;
    int *gbeg, *in_ptr;
    // groups
    unsigned* gmeta;
    int* gsize;
    int* gpre;
    float4* gstate;  // R, u, nmda, xpre
    float2* gview;   // hot view of step t: nmda, flags (as bits)
    float2* gcold;   // cold view of step t: xpre before the arrival jump, R after STP
    float2* gextra;  // AMPA conductance, step of the last arrival (checkpoint fields)
    // synapses (post-major)
    unsigned* gid;
    float* ca;
    float4* ev;      // alpha, beta, autophosphorylation, eligibility
    float *act, *e1, *e2;
    float* val;      // VAL_SLOTS per synapse
    // control
    Ctrl* ctrl;
    float4* gates;   // [2][ncol] gate, act_ema, nov_ema, l6_ema after even / odd steps
    int *col_sp, *l6_sp, *sub_sp;  // [2][ncol], [2][ncol], [2][TD_DIM]
    unsigned* byte_hist_nov;
    int* byte_histogram;
    int* neuron_byte_counts;
    float *w_value, *w_pred, *baseline;
    const unsigned char* corpus;
    unsigned* raster;
    int raster_cap, words;
    int N, N_assoc, NPC, ncol, l4, per_sub;
    int tile_cap;           // staged elements per stream per buffer (>= any aligned in-list)
    int queue_cap;          // per-warp event queue entries (>= max in-degree)
    // column sharding: local neuron j is global a0 + j for j < n_a, else
    // pf0 + (j - n_a).  With sharded != 0 the step's spike words, spike count
    // and TD sub-population counts go to `send`, every rank's payload arrives
    // in `recv` (an all-gather between k_neurons and k_mirror_hist), and the
    // groups of remote pres ("mirror" groups, after the local ones) are
    // updated by k_mirror_groups from the gathered bits.
    int n_a, a0, pf0, sharded, world;
    int c0, c1;             // this rank's columns
    unsigned* send;
    const unsigned* recv;
    int pw, words_max;      // payload words per rank; count word index
    int M;                  // mirror pres
    const int* mbeg;        // M + 1 group ranges
    const unsigned* mbit;   // bit of each mirror pre in recv
    unsigned* mhist;        // 32-step spike history of each mirror pre
    long long G_local, GM;  // groups of local pres; mirror groups (after them)
    const int* gmir;        // mirror pre of each mirror group
};

// Exponentials on the simulation path.  The canonical build uses snn_expf
// (shared bit for bit with the CPU oracle); the refmath build
// (-DSNN_REFMATH, compiled with the compiler's default contraction) uses CUDA's
// expf as the reference's kernels do, for agreement with the reference binary
// instead of with the oracle.
#ifdef SNN_REFMATH
__device__ __forceinline__ float k_exp(float x) { return expf(x); }
__global__ void k_exp_one(float x, float* out) { *out = expf(x); }
#else
__device__ __forceinline__ float k_exp(float x) { return snn_expf(x); }
#endif

// a constant decay exp(x), computed like the kernels compute theirs
inline float const_exp(float x) {
#ifdef SNN_REFMATH
    float* d = nullptr;
    float h = 0.0f;
    SNN_CUDA(cudaMalloc((void**)&d, sizeof(float)));
    k_exp_one<<<1, 1>>>(x, d);
    const cudaError_t e = cudaMemcpy(&h, d, sizeof(float), cudaMemcpyDeviceToHost);
    cudaFree(d);
    SNN_CUDA(e);
    return h;
#else
    return snn_expf(x);
#endif
}

__device__ __forceinline__ int phase_of(long long step) {
    return step < 5000 ? 0 : step < 200000 ? 1 : step < 800000 ? 2 : step < 1500000 ? 3 : 4;
}
__constant__ float c_phase_gain[5] = {0.0f, 1.0f, 3.0f, 1.0f, 0.3f};
__constant__ float c_phase_prune[5] = {0.0f, 0.0f, 0.0f, 0.05f, 0.02f};

__device__ __forceinline__ float clampf(float x, float lo, float hi) {
    if (x < lo) x = lo;
    if (x > hi) x = hi;
    return x;
}

// ---------------------------------------------------------------------------
// Start of step t (src/stage2e/scheduler.cu:485-540, synapse_kernels.cu:
// 207-211, thalamic_gate.cu:53-142), computed at the top of k_neurons: every
// CTA derives t, the injection flag and the byte itself (the same function of
// the control block, which nothing modifies until the step's epilogue), CTA 0
// also publishes phase gain, pruning threshold and M_ij for the synapse pass,
// and the thalamic gates are stepped by the CTAs that hold L4 neurons of a
// column (each computes the same value from the gate state of step t-1; the
// CTA holding the column's first neuron stores it).
// ---------------------------------------------------------------------------
struct StepIn {
    long long t;
    int inject, byte;
};

__device__ __forceinline__ StepIn step_inputs(const Dev& d, const Consts& k) {
    const Ctrl* c = d.ctrl;
    StepIn s;
    s.t = c->next_t;
    s.inject = (s.t % k.inject_interval) == 0;
    s.byte = 0;
    if (s.inject) {
        const int bo = c->byte_override;
        const long long clen = c->corpus_len;
        if (bo >= 0) s.byte = bo;
        else if (clen > 0) s.byte = d.corpus[c->corpus_pos];
        else s.byte = (int)((s.t / k.inject_interval) % 256);
    }
    return s;
}

// CTA 0: per-step scalars of the synapse pass and the epilogue
__device__ void publish_step(const Dev& d, const Consts& k, const StepIn& s) {
    Ctrl* c = d.ctrl;
    const int ph = phase_of(s.t + c->phase_offset);
    const int learn = c->learn, e0 = c->e0;
    const float c0 = c->conc[0], c1 = c->conc[1], c2 = c->conc[2], c3 = c->conc[3];
    float M[2];
    for (int e = 0; e < 2; ++e) {
        if (e0) { M[e] = 1.0f; continue; }
        float z = pm_mul(k.rec_da[e], c0);
        z = pm_fma(k.rec_ach, c1, z);
        z = pm_fma(k.rec_ne, c2, z);
        z = pm_fma(k.rec_ht5, c3, z);
        M[e] = pm_div(1.0f, pm_add(1.0f, k_exp(-z)));
    }
    c->t = s.t;
    c->gain = learn ? c_phase_gain[ph] : 0.0f;
    c->prune_thr = c_phase_prune[ph];
    c->inject = s.inject;
    c->byte = s.inject ? s.byte : -1;
    c->M[0] = M[0];
    c->M[1] = M[1];
}

// thalamic gate of column `col` after step t (double-buffered by t & 1)
__device__ float4 gate_step(const Dev& d, int col, const StepIn& s) {
    const long long t = s.t;
    float4 g = d.gates[((t + 1) & 1) * d.ncol + col];
    const bool prev_ok = t > 0;
    const float cur = prev_ok ? pm_i2f(d.col_sp[((t - 1) & 1) * d.ncol + col]) : 0.0f;
    const float l6c = prev_ok ? pm_i2f(d.l6_sp[((t - 1) & 1) * d.ncol + col]) : 0.0f;
    const float den = g.y > 1.0f ? g.y : 1.0f;
    const float an = fminf(1.0f, fmaxf(-1.0f, pm_div(pm_sub(g.y, cur), den)));
    const float l6d = g.w > 1.0f ? g.w : 1.0f;
    const float l6n = fminf(1.0f, fmaxf(-1.0f, pm_div(pm_sub(g.w, l6c), l6d)));
    float nov = 0.0f;
    if (s.inject) {
        const unsigned htot = d.ctrl->hist_total, bc = d.byte_hist_nov[s.byte];
        const unsigned tm = htot > 1u ? htot : 1u;
        nov = pm_sub(1.0f, pm_div(pm_u2f(bc), pm_u2f(tm)));
        nov = fminf(1.0f, fmaxf(0.0f, nov));
    }
    const float om99 = pm_sub(1.0f, 0.99f), om95 = pm_sub(1.0f, 0.95f);
    g.y = pm_fma(0.99f, g.y, pm_mul(om99, cur));
    g.w = pm_fma(0.99f, g.w, pm_mul(om99, l6c));
    g.z = pm_fma(0.95f, g.z, pm_mul(om95, nov));
    float tg = pm_fma(0.3f, an, 0.5f);
    tg = pm_fma(0.2f, g.z, tg);
    tg = pm_fma(0.15f, l6n, tg);
    tg = fminf(0.9f, fmaxf(0.1f, tg));
    g.x = pm_fma(0.01f, pm_sub(tg, g.x), g.x);
    g.x = fminf(1.0f, fmaxf(0.0f, g.x));
    return g;
}

// ---------------------------------------------------------------------------
// end of step t: the host-side work the reference does after the dispatch of
// step t (src/stage2e/scheduler.cu:576-670): inhibition drive / kWTA size for
// step t+1 (:688-722), modulators + TD value function (:724-751,
// modulatory_kernels.cu:176-254), statistics.  Runs in one thread at the
// start of k_synapses (all of step t's neuron counters are final by then).
// ---------------------------------------------------------------------------
__device__ void step_epilogue(const Dev& d, const Consts& k) {
    Ctrl* c = d.ctrl;
    const long long t = c->t;
    const int sp = c->step_spikes[t & 1];
    const float avg = c->total_steps > 0
                          ? pm_div(pm_ll2f(c->total_spikes), pm_ll2f(c->total_steps))
                          : 0.0f;
    c->inh_active = 0;
    if (t % 10 == 0) {
        float drive = pm_div(pm_i2f(c->last_spikes), pm_add(avg, 1.0f));
        drive = clampf(drive, 0.0f, 2.0f);
        c->gdrive = pm_mul(drive, 0.15f);
        const int kk = (int)pm_mul(pm_div(avg, pm_i2f(d.ncol)), 0.5f);
        c->kwta_k = kk < 3 ? 3 : (kk > 5 ? 5 : kk);
        c->inh_active = 1;
    }
    if (t % 100 == 0 && !c->e0) {
        const float cur = pm_i2f(c->last_spikes);
        float nov = avg > 0.0f ? pm_div(fabsf(pm_sub(cur, avg)), pm_add(avg, 1.0f)) : 0.0f;
        if (nov > 1.0f) nov = 1.0f;
        const float pred = (cur > 10.0f && cur < 1000.0f) ? 0.5f : 0.1f;
        const float reward = pm_add(pm_mul(0.5f, nov), pm_mul(0.3f, pred));
        const int* sub = d.sub_sp + (t & 1) * TD_DIM;
        const float per = pm_i2f(d.per_sub);
        float vs = 0.0f;
        for (int q = 0; q < TD_DIM; ++q) vs = pm_fma(d.w_value[q], pm_div(pm_i2f(sub[q]), per), vs);
        const float om = pm_sub(1.0f, 0.99f);
        float vsp = 0.0f;
        for (int q = 0; q < TD_DIM; ++q) {
            const float f = pm_div(pm_i2f(sub[q]), per);
            d.baseline[q] = pm_fma(0.99f, d.baseline[q], pm_mul(om, f));
            vsp = pm_fma(d.w_value[q], pm_mul(d.w_pred[q], f), vsp);
        }
        const float delta = pm_sub(pm_add(reward, pm_mul(0.9f, vsp)), vs);
        for (int q = 0; q < TD_DIM; ++q) {
            const float f = pm_div(pm_i2f(sub[q]), per);
            d.w_value[q] = clampf(pm_fma(pm_mul(0.001f, delta), f, d.w_value[q]), -1.0f, 1.0f);
            const float pe = pm_sub(f, d.baseline[q]);
            d.w_pred[q] = pm_fma(pm_mul(0.001f, pe), f, d.w_pred[q]);
        }
        float sig[4];
        sig[0] = pm_add(0.1f, delta > 0.0f ? delta : pm_mul(0.3f, delta));
        if (sig[0] < 0.0f) sig[0] = 0.0f;
        sig[1] = pm_add(pm_add(0.2f, pm_mul(0.3f, nov)), pm_mul(0.1f, pred));
        sig[2] = 0.05f;
        sig[3] = 0.1f;
        if (delta < -0.5f) sig[3] = pm_add(sig[3], pm_mul(0.3f, fabsf(delta)));
        for (int m = 0; m < 4; ++m)
            c->conc[m] = clampf(pm_fma(c->conc[m], k.mod_dec[m], sig[m]), 0.0f, 2.0f);
    }
    c->total_steps += 1;
    c->total_spikes += sp;
    if (t % k.inject_interval == 0) c->inject_spikes += sp;
    c->last_spikes = sp;
    const unsigned long long arr = c->step_arrivals[t & 1];
    if (arr > 750000ull) c->dropped_ref += arr - 750000ull;
    // hand-over to step t + 1: what must follow every CTA of step t's k_neurons
    if (c->inject) {
        d.byte_hist_nov[c->byte] += (unsigned)d.ncol;
        c->hist_total += (unsigned)d.ncol;
        const long long clen = c->corpus_len;
        if (c->byte_override < 0 && clen > 0) c->corpus_pos = (c->corpus_pos + 1) % clen;
    }
    c->byte_override = -1;
    c->step_spikes[(t + 1) & 1] = 0;
    c->step_arrivals[(t + 1) & 1] = 0ull;
    c->next_t = t + 1;
}

// STP / NMDA / pre-trace update of group g at step t from its pre's spike
// history h (bit 0 = spike at t, bit d = spike at t - d) and its per-step
// view for the synapse pass
// (ex = the group's AMPA conductance and last arrival step, loaded by the
// caller together with meta and st)
__device__ __forceinline__ void update_group(const Dev& d, const Consts& k, int g, unsigned meta, float4 st,
                                             float2 ex, unsigned h, long long t,
                                             unsigned long long& arr_cnt, unsigned long long& disp_cnt) {
    const int dd = meta & GV_D_MASK;
    const bool ff = meta & GV_FF, exc = meta & GV_EXC;
    const bool arr = (h >> dd) & 1u;
    const bool nxt = (h >> (dd - 1)) & 1u;
    const bool disp = h & 1u;
    if (arr) {
        ex.x = pm_fma(pm_mul(1.0f, st.x), st.y, ex.x);
        ex.y = pm_ll2f(t);
    }
    ex.x = pm_mul(ex.x, k.dec_ampa);
    d.gextra[g] = ex;
    if (arr && exc) st.z = pm_fma(pm_mul(k.g_nmda, st.x), st.y, st.z);
    st.z = pm_mul(st.z, k.dec_nmda);
    if (ff) st.x = pm_fma(pm_sub(1.0f, st.x), k.rec_ff_step, st.x);
    st.w = pm_mul(st.w, k.dec_xpre);
    const float x_ltp = st.w;
    if (arr) {
        st.w = pm_add(st.w, k.a_plus);
        const int cl = ff ? 0 : (exc ? 1 : 2);
        const float U = k.U[cl];
        st.x = pm_fma(pm_sub(1.0f, st.x), k.rec[cl], st.x);
        st.y = pm_fma(pm_sub(st.y, U), k.fac[cl], U);
        const float un = pm_fma(U, pm_sub(1.0f, st.y), st.y);
        const float rn = pm_mul(st.x, pm_sub(1.0f, un));
        st.y = un > 1.0f ? 1.0f : un;
        st.x = rn < 0.0f ? 0.0f : rn;
        arr_cnt += gw_size(meta);
    }
    if (disp) disp_cnt += gw_size(meta);
    d.gstate[g] = st;
    const bool ring = nxt && dd >= 2;
    const unsigned fl = (meta & (GV_D_MASK | GV_FF | GV_EXC)) | (arr ? GV_ARR : 0u) |
                        (nxt ? GV_NEXT : 0u) | (disp ? GV_DISP : 0u) |
                        ((arr || disp || ring) ? GV_EV : 0u);
    d.gview[g] = make_float2(st.z, __uint_as_float(fl));
    d.gcold[g] = make_float2(x_ltp, st.x);
}

// ---------------------------------------------------------------------------
// k_neurons: one thread per neuron, then the CTA's outgoing synapse groups.
//   input .......... input_encoding.cu:117-164 (hashes recomputed per L4 neuron,
//                    duplicates added in hash order)
//   inhibition ..... scheduler.cu:112-133 + 234-265 (computed at step t from
//                    fire rates / column counts of step t-1, as the reference
//                    writes it after step t-1 for the step-t update)
//   AdEx ........... neuron_kernels.cu:61-165
//   groups ......... synapse_kernels.cu:123-141 (arrival conductance), :84-94
//                    (decays, FF recovery), :176-194 / :282 (pre trace),
//                    :334-387 (STP); one thread per group of the CTA's neurons
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NEU_THREADS) k_neurons(Dev d, Consts k) {
    __shared__ unsigned s_hist[NEU_BLOCK];
    __shared__ StepIn s_in;
    __shared__ float s_gate[NEU_BLOCK];  // gate of column s_colA + q
    __shared__ int s_colA;
    const Ctrl* c = d.ctrl;
    const int i0 = blockIdx.x * NEU_BLOCK;
    const int i1 = min(i0 + NEU_BLOCK, d.N);
    const int i = i0 + (int)threadIdx.x;
    const int gi = i < d.n_a ? d.a0 + i : d.pf0 + (i - d.n_a);  // global neuron id
    const bool valid = threadIdx.x < NEU_BLOCK && i < d.N;
    // the neuron's state is loaded first: its latency overlaps the step
    // inputs and gates below
    struct NeuIn {
        unsigned info, hist;
        float input, fr, V, s, nmda, wad, can, xpost;
        int ref, last;
        unsigned short off;
    } nu{};
    if (valid) {
        nu.info = d.info[i]; nu.input = d.input[i]; nu.ref = d.ref[i]; nu.fr = d.fr[i];
        nu.V = d.V[i]; nu.off = d.off[i]; nu.s = d.s[i]; nu.nmda = d.nmda_cur[i];
        nu.wad = d.wad[i]; nu.can = d.can[i]; nu.xpost = d.xpost[i]; nu.hist = d.hist[i];
        nu.last = d.last[i];
    }
    // the CTA's group range and the inhibition scalars (written by the
    // previous step's epilogue, not modified in this kernel)
    const int g0 = d.gbeg[i0], g1 = d.gbeg[i1];
    // the first NEU_GU groups of every thread are loaded now: their latency
    // overlaps the step inputs, the gates and the neuron update
    unsigned m0[NEU_GU];
    float4 st0[NEU_GU];
    float2 ex0[NEU_GU];
#pragma unroll
    for (int u = 0; u < NEU_GU; ++u) {
        const int gu = g0 + (int)threadIdx.x + u * NEU_THREADS;
        m0[u] = gu < g1 ? d.gmeta[gu] : 0u;
        st0[u] = gu < g1 ? d.gstate[gu] : make_float4(0, 0, 0, 0);
        ex0[u] = gu < g1 ? d.gextra[gu] : make_float2(0, 0);
    }
    const int inh_active = c->inh_active, kwta_k = c->kwta_k;
    const float gdrive = c->gdrive;
    if (threadIdx.x == 0) {
        s_in = step_inputs(d, k);
        if (blockIdx.x == 0) publish_step(d, k, s_in);
    }
    __syncthreads();
    const long long t = s_in.t;
    {   // thalamic gates of the columns whose L4 neurons this CTA holds
        const int la = min(i1, d.n_a);  // local column neurons are [0, n_a)
        const int colA = i0 < la ? (d.a0 + i0) / d.NPC : 0;
        const int colB = i0 < la ? (d.a0 + la - 1) / d.NPC : -1;
        if (threadIdx.x == 0) s_colA = colA;
        const int col = colA + (int)threadIdx.x;
        if (col <= colB) {
            const int l4_lo = col * d.NPC, l4_hi = l4_lo + d.l4;  // global L4 range
            const int g_lo = d.a0 + i0, g_hi = d.a0 + la;        // this CTA's column neurons
            if (l4_lo < g_hi && l4_hi > g_lo) {
                const float4 g = gate_step(d, col, s_in);
                s_gate[threadIdx.x] = g.x;
                if (l4_lo >= g_lo) d.gates[(t & 1) * d.ncol + col] = g;  // holds the column's first neuron
            }
        }
        __syncthreads();
    }
    unsigned spike = 0;
    unsigned hist = 0;
    if (valid) {
        const unsigned info = nu.info;
        const int type = info & 1, region = (info >> 1) & 7, subtype = (info >> 4) & 3;
        const int col = (region != PF) ? (int)(info >> 8) : -1;
        float input = nu.input;
        if (s_in.inject && region == L4) {
            const int off = gi - col * d.NPC;
            const int b = s_in.byte;
            const int ps = col * k.pref_range;
            const bool in_r = b >= ps && b < ps + k.pref_range;
            const float v = pm_mul(pm_mul(k.pop_gain, in_r ? k.gain_in : k.gain_out), s_gate[col - s_colA]);
            unsigned h = (unsigned)b * 2654435761u + (unsigned)col * 0x9E3779B9u;
            for (int q = 0; q < k.pop_k; ++q) {
                h ^= h << 13; h ^= h >> 17; h ^= h << 5;
                if ((int)(h % (unsigned)d.l4) == off) input = pm_add(input, v);
            }
        }
        float inh = 0.0f;
        if (inh_active) {
            const float sg = subtype == 0 ? 1.40f : subtype == 1 ? 0.85f : subtype == 2 ? 1.10f : 1.0f;
            const float rg = region == PF ? 0.60f : 1.0f;
            float cur = pm_mul(pm_mul(pm_fma(nu.fr, 2.0f, gdrive), sg), rg);
            if (type == 1) cur = pm_mul(cur, 0.35f);
            if (cur > 2.0f) cur = 2.0f;
            inh = cur;
            if (col >= 0) {
                const int sp = d.col_sp[((t - 1) & 1) * d.ncol + col];
                const int kk = kwta_k;
                int width = kk * 8;
                width = width < 1 ? 1 : (width > d.NPC ? d.NPC : width);
                const int rank = (gi + col * 37) % d.NPC;
                if (sp > 0 && sp > kk && rank >= width) {
                    float ex = pm_mul(0.35f, pm_div(pm_i2f(sp - kk), pm_i2f(kk + 1)));
                    if (ex > 2.0f) ex = 2.0f;
                    inh = pm_add(inh, ex);
                }
            }
        }
        int ref = nu.ref;
        float fr = nu.fr;
        float V = nu.V;
        unsigned short off = nu.off;
        if (ref > 0) {
            d.ref[i] = ref - 1;
            d.fr[i] = pm_mul(fr, k.fr_refr);
        } else {
            const float s = pm_fma(nu.s, k.syn_keep, pm_mul(input, k.syn_in));
            const float I = pm_sub(pm_add(s, nu.nmda), inh);
            float w = nu.wad;
            float ea = pm_div(pm_sub(V, k.vt), k.dT);
            if (ea > 10.0f) ea = 10.0f;
            if (ea < -10.0f) ea = -10.0f;
            const float et = pm_mul(k.dT, k_exp(ea));
            const float dV = pm_mul(pm_add(pm_sub(pm_add(-V, et), w), I), k.inv_taum);
            const float dw = pm_mul(pm_fma(k.a_ad, V, -w), k.inv_tauw);
            V = pm_add(V, dV);
            w = pm_add(w, dw);
            V = clampf(V, k.vmin, k.vmax);
            const float theta = pm_add(1.0f, pm_div(pm_u2f(off), 256.0f));
            float can = nu.can;
            if (V >= theta) {
                spike = 1;
                const int last = nu.last;
                if (last >= 0 && t - last <= 5) atomicAdd(&d.ctrl->burst, 1ull);
                d.last[i] = (int)t;
                ref = k.refr_steps;
                V = 0.0f;
                w = pm_add(w, k.b_ad);
                can = fminf(pm_add(can, k.ca_n_inc), 1.0f);
                fr = pm_fma(fr, k.fr_spk_keep, k.fr_spk_add);
                int no = (int)off + k.off_add;
                if (no > k.off_max) no = k.off_max;
                off = (unsigned short)no;
            } else {
                off = (unsigned short)pm_mul(pm_u2f(off), k.off_decay);
                can = pm_mul(can, k.ca_n_dec);
                fr = pm_mul(fr, k.fr_quiet);
            }
            d.s[i] = s;
            d.wad[i] = w;
            d.V[i] = V;
            d.can[i] = can;
            d.fr[i] = fr;
            d.ref[i] = ref;
            d.off[i] = off;
        }
        // Mg block and post trace of neuron i for this step's synapse pass
        const float Vb = pm_fma(50.0f, V, -70.0f);
        const float e = k_exp(pm_div(-Vb, 16.13f));
        d.mg[i] = pm_div(1.0f, pm_add(1.0f, pm_div(pm_mul(1.0f, e), 3.57f)));
        float xp = pm_mul(nu.xpost, k.dec_xpost);
        if (spike) xp = pm_add(xp, k.a_minus);
        d.xpost[i] = xp;
        hist = (nu.hist << 1) | spike;
        d.hist[i] = hist;
        if (spike) {
            const int sub = gi / d.per_sub;
            if (d.sharded) {  // global counts are summed over the ranks by k_mirror_hist
                atomicAdd(&d.send[d.words_max], 1u);
                if (sub < TD_DIM) atomicAdd(&d.send[d.words_max + 1 + sub], 1u);
            } else {
                atomicAdd(&d.ctrl->step_spikes[t & 1], 1);
                if (sub < TD_DIM) atomicAdd(&d.sub_sp[(t & 1) * TD_DIM + sub], 1);
            }
            if (col >= 0) {
                atomicAdd(&d.col_sp[(t & 1) * d.ncol + col], 1);
                if (region == L6) atomicAdd(&d.l6_sp[(t & 1) * d.ncol + col], 1);
            }
            if (s_in.inject) {
                atomicAdd(&d.byte_histogram[s_in.byte], 1);
                atomicAdd(&d.neuron_byte_counts[(long long)i * 256 + s_in.byte], 1);
            }
            atomicAdd(&d.ctrl->ltp_visits, (unsigned long long)(d.in_ptr[i + 1] - d.in_ptr[i]));
        }
    }
    if (threadIdx.x < NEU_BLOCK) s_hist[threadIdx.x] = hist;
    const unsigned word = __ballot_sync(0xffffffffu, spike != 0);
    if (threadIdx.x < NEU_BLOCK && (threadIdx.x & 31) == 0 && (i >> 5) < d.words) {
        const long long row = (t - c->raster_base) % d.raster_cap;
        d.raster[row * d.words + (i >> 5)] = word;
        if (d.sharded) d.send[i >> 5] = word;
    }
    __syncthreads();
    // outgoing synapse groups of this CTA's neurons, one thread per group
    unsigned long long arr_cnt = 0, disp_cnt = 0;
#pragma unroll
    for (int u = 0; u < NEU_GU; ++u) {
        const int gu = g0 + (int)threadIdx.x + u * NEU_THREADS;
        if (gu < g1) update_group(d, k, gu, m0[u], st0[u], ex0[u], s_hist[gw_lpre(m0[u])], t, arr_cnt, disp_cnt);
    }
    // the rest (CTAs with more than NEU_GU * NEU_THREADS groups), NEU_GU per
    // iteration: every load of the iteration is issued before the first
    // group's stores
    const int stride = NEU_GU * NEU_THREADS;
    for (int g = g0 + stride + (int)threadIdx.x; g < g1; g += stride) {
        unsigned m[NEU_GU];
        float4 st[NEU_GU];
        float2 ex[NEU_GU];
#pragma unroll
        for (int u = 0; u < NEU_GU; ++u) {
            const int gu = g + u * NEU_THREADS;
            m[u] = gu < g1 ? d.gmeta[gu] : 0u;
            st[u] = gu < g1 ? d.gstate[gu] : make_float4(0, 0, 0, 0);
            ex[u] = gu < g1 ? d.gextra[gu] : make_float2(0, 0);
        }
#pragma unroll
        for (int u = 0; u < NEU_GU; ++u) {
            const int gu = g + u * NEU_THREADS;
            if (gu < g1)
                update_group(d, k, gu, m[u], st[u], ex[u], s_hist[gw_lpre(m[u])], t, arr_cnt, disp_cnt);
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        arr_cnt += __shfl_xor_sync(0xffffffffu, arr_cnt, o);
        disp_cnt += __shfl_xor_sync(0xffffffffu, disp_cnt, o);
    }
    if ((threadIdx.x & 31) == 0) {
        if (arr_cnt) {
            atomicAdd(&d.ctrl->arrivals, arr_cnt);
            atomicAdd(&d.ctrl->step_arrivals[t & 1], arr_cnt);
        }
        if (disp_cnt) atomicAdd(&d.ctrl->dispatched, disp_cnt);
    }
}

// ---------------------------------------------------------------------------
// Sharded runs.  A mirror group (the groups of a remote pre with synapses onto
// this rank) is updated in two parts, which together give exactly the update
// the owning rank's k_neurons gives a local pre's groups:
//   k_mirror_groups  one thread per mirror group, before step t's exchange
//                    (on a side stream, overlapping k_neurons and the
//                    all-gather): the update from the pre's spikes up to
//                    t - 1, i.e. with bit 0 (a spike at t) still clear.  Only
//                    the dispatch flag and, for delay 1, the next-step flag
//                    depend on bit 0.
//   k_mirror_hist    after the all-gather of step t's payloads: block 0 sums
//                    the global spike count and TD sub-population counts of
//                    step t; one thread per mirror pre shifts the gathered bit
//                    of step t into its 32-step history and, if the pre spiked,
//                    sets the dispatch (and delay-1 next-step) flags of its
//                    mirror groups and counts their dispatches.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_mirror_hist(Dev d) {
    const long long t = d.ctrl->t;
    if (blockIdx.x == 0) {
        if (threadIdx.x == 0) {
            long long cnt = 0;
            for (int r = 0; r < d.world; ++r) cnt += d.recv[(size_t)r * d.pw + d.words_max];
            d.ctrl->step_spikes[t & 1] = (int)cnt;
        }
        for (int q = threadIdx.x; q < TD_DIM; q += blockDim.x) {
            int sc = 0;
            for (int r = 0; r < d.world; ++r) sc += (int)d.recv[(size_t)r * d.pw + d.words_max + 1 + q];
            d.sub_sp[(t & 1) * TD_DIM + q] = sc;
        }
    }
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    unsigned long long disp_cnt = 0;
    if (m < d.M) {
        const unsigned b = d.mbit[m];
        const unsigned spk = (d.recv[b >> 5] >> (b & 31)) & 1u;
        d.mhist[m] = (d.mhist[m] << 1) | spk;
        if (spk)  // the pre's mirror groups are [mbeg[m], mbeg[m + 1]) (group indices)
            for (int g = d.mbeg[m]; g < d.mbeg[m + 1]; ++g) {
                const unsigned meta = d.gmeta[g];
                float2 v = d.gview[g];
                const unsigned add = GV_DISP | GV_EV | ((meta & GV_D_MASK) == 1u ? GV_NEXT : 0u);
                v.y = __uint_as_float(__float_as_uint(v.y) | add);
                d.gview[g] = v;
                disp_cnt += gw_size(meta);
            }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) disp_cnt += __shfl_xor_sync(0xffffffffu, disp_cnt, o);
    if ((threadIdx.x & 31) == 0 && disp_cnt) atomicAdd(&d.ctrl->dispatched, disp_cnt);
}

__global__ void __launch_bounds__(256) k_mirror_groups(Dev d, Consts k) {
    // step t = next_t: k_neurons of the same step may be running, and it
    // publishes ctrl->t only for the synapse pass
    const long long t = d.ctrl->next_t;
    const long long x = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    unsigned long long arr_cnt = 0, disp_cnt = 0;
    if (x < d.GM) {
        const int g = (int)(d.G_local + x);
        update_group(d, k, g, d.gmeta[g], d.gstate[g], d.gextra[g], d.mhist[d.gmir[x]] << 1, t, arr_cnt,
                     disp_cnt);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) arr_cnt += __shfl_xor_sync(0xffffffffu, arr_cnt, o);
    if ((threadIdx.x & 31) == 0 && arr_cnt) {
        atomicAdd(&d.ctrl->arrivals, arr_cnt);
        atomicAdd(&d.ctrl->step_arrivals[t & 1], arr_cnt);
    }
}

// ---------------------------------------------------------------------------
// k_synapses: one warp per post-synaptic neuron, post-major.
//   Ca / NMDA ....... synapse_kernels.cu:45-121
//   LTP (post) ...... synapse_kernels.cu:153-255
//   LTD (arrival) ... synapse_kernels.cu:257-329
//   dispatch value .. neuron_kernels.cu:204-206 (w * R after this step's STP)
//   input of t+1 .... neuron_kernels.cu:37-56 (delivery of the arrivals)
//   CaMKII / elig ... synapse_kernels.cu:469-543 (every 10 steps)
//   PSW decay ....... scheduler.cu:55-86 (every 1000 steps)
// Both sums use the canonical order: 32-synapse chunks in ascending
// reference synapse id, xor butterfly inside a chunk, chunks added in order.
// Each lane carries two chunks at once (independent loads in flight).
// ---------------------------------------------------------------------------
// --- bulk async copy (1D TMA) helpers -------------------------------------
__device__ __forceinline__ unsigned smem_u32(const void* p) {
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
// global -> shared bulk copy completing on `bar` (16-byte aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes,
                                         unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

#ifndef SYN_FOLD_U
#define SYN_FOLD_U 3   // chunks whose loads the periodic phase issues together
#endif
#ifndef SYN_MIN_BLOCKS
#define SYN_MIN_BLOCKS 4
#endif
#ifndef SYN_THREADS_CFG
#define SYN_THREADS_CFG 224
#endif
#ifndef SYN_GRAB_RUN
#define SYN_GRAB_RUN 2   // consecutive posts per unit of a CTA's post list
#endif
// 7 warps per CTA (4 CTAs per SM at 72 registers), each an independent pipeline
constexpr int SYN_THREADS = SYN_THREADS_CFG;
constexpr int SYN_WARPS = SYN_THREADS / 32;
constexpr unsigned WAIT_LIMIT = 1u << 24;  // bounded spin (~seconds) before flagging an error

struct PostCtx {
    long long t;
    float gain, prune, Mexc, Minh, mgj, xpost, one_m_V;
    bool post_spk, e0, do10, do1000;
    int slot_now;
};

// Plasticity / dispatch / periodic work of one queued synapse p (every
// synapse of a spiking post, arrivals, dispatches, ring reads, and all
// synapses on the 10- / 1000-step schedule).  Returns the synapse's term of
// the next step's input current (0 if none).
// Plasticity / dispatch / periodic work of one queued synapse, split into a
// load stage (all independent loads issued) and a compute stage, so that a
// warp can keep two batches of 32 queued synapses in flight.
struct EvIn {
    unsigned gw, fl;
    int p;
    float ca, ring;
    float2 cold;
    float4 q;
};

__device__ __forceinline__ void ev_load(const Dev& d, const PostCtx& pc, int p, unsigned gw,
                                        unsigned fl, float ca, EvIn& x) {
    x.gw = gw; x.fl = fl; x.p = p; x.ca = ca;
    const int dd = fl & GV_D_MASK;
    const bool plast = pc.post_spk || (fl & (GV_ARR | GV_DISP)) || pc.do1000;
    x.ring = 0.0f;
    if ((fl & GV_NEXT) && dd >= 2)
        x.ring = d.val[(long long)p * VAL_SLOTS + (int)(((pc.t + 1 - dd) / 3) & (VAL_SLOTS - 1))];
    x.cold = make_float2(0.0f, 0.0f);
    x.q = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (plast) {
        x.cold = d.gcold[gw & 0x3fffffffu];  // x_pre before the arrival jump, R after STP
        x.q = d.ev[p];                       // alpha, beta, auto, elig
    }
}

// returns the synapse's term of the next step's input current (0 if none)
__device__ __forceinline__ float ev_compute(const Dev& d, const Consts& k, const PostCtx& pc,
                                            EvIn& x) {
    const unsigned fl = x.fl;
    const bool ff = x.gw & (1u << 30), exc = x.gw >> 31;
    const int dd = fl & GV_D_MASK;
    const bool arr = fl & GV_ARR, disp = fl & GV_DISP;
    const bool plast = pc.post_spk || arr || disp || pc.do1000;
    float term_in = x.ring;
    if (!plast) return term_in;
    float4 q = x.q;
    const float ca = x.ca;
    const int p = x.p;
    const float eta = ff ? k.eta_ff : k.eta;
    const float M = pc.e0 ? 1.0f : (exc ? pc.Mexc : pc.Minh);
    const float pf = pc.e0 ? 1.0f : pm_sub(1.0f, pm_mul(0.5f, q.z));
    if (pc.post_spk) {  // LTP from the pre trace (post spiked); selects, not branches
        const float dw = pm_fma(x.cold.x, k.a_plus, 0.0f);
        const float nx = pm_fma(pm_mul(pm_mul(pm_mul(eta, dw), pc.gain), M), pf, q.x);
        q.x = dw > 0.0f ? nx : q.x;
        const float ex = pm_sub(ca, k.reb_thr);
        const float ny = pm_fma(pm_mul(pm_mul(pm_mul(eta, ex), k.reb_gain), pc.gain), M, q.y);
        q.y = ca > k.reb_thr ? ny : q.y;
        q.w = pm_add(q.w, dw);
    }
    {   // LTD at arrival from the post trace, computed for every lane
        const float dw = pm_mul(-pc.xpost, k.a_minus);
        const float ny = pm_fma(pm_mul(pm_mul(pm_mul(eta, -dw), pc.gain), M), pf, q.y);
        q.y = (arr && dw < 0.0f) ? ny : q.y;
        const float nw = pm_add(q.w, dw);
        q.w = arr ? nw : q.w;
    }
    if (disp) {  // value this dispatch delivers d steps later
        const float wm = pm_div(pm_mul(k.w_max, q.x), pm_add(q.x, q.y));
        const float val = pm_mul(exc ? wm : -wm, x.cold.y);
        if (dd == 1) term_in = val;
        else d.val[(long long)p * VAL_SLOTS + pc.slot_now] = val;
    }
    if (pc.do1000) {
        float a = pm_mul(q.x, k.psw_decay), bb = pm_mul(q.y, k.psw_decay);
        if (a < k.ab_min) a = k.ab_min;
        if (bb < k.ab_min) bb = k.ab_min;
        if (pm_add(a, bb) < pc.prune) { a = k.ab_reset; bb = k.ab_reset; }
        q.x = a;
        q.y = bb;
    }
    if (pc.post_spk || arr || pc.do1000) d.ev[p] = q;
    return term_in;
}

// CaMKII every 10 steps (synapse_kernels.cu:469-515) of an excitatory synapse
// from this step's Ca
__device__ __forceinline__ void camkii(const Consts& k, float ca, float& act, float& au) {
    const float ca4 = pm_mul(pm_mul(pm_mul(ca, ca), ca), ca);
    const float da = pm_fma(pm_mul(k.ck_k1, ca4), pm_sub(1.0f, act),
                            -pm_mul(pm_mul(k.ck_k2, act), k.ck_pp1));
    const float du = pm_fma(pm_mul(pm_mul(k.ck_k3, act), act), pm_sub(1.0f, au),
                            -pm_mul(pm_mul(k.ck_k4, au), k.ck_pp1));
    act = clampf(pm_fma(da, k.ck_dt, act), 0.0f, 1.0f);
    au = clampf(pm_fma(du, k.ck_dt, au), 0.0f, 1.0f);
}

__device__ __forceinline__ void prefetch_l2(const void* ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

// ---------------------------------------------------------------------------
// k_synapses: persistent; every warp is an independent pipeline over the
// post-synaptic neurons it takes from its CTA's list (runs of 2 consecutive
// posts, the CTAs' runs interleaved over the network).  Lane 0 stages the
// group ids of the warp's next neuron into the warp's own shared-memory
// buffer with cp.async.bulk (mbarrier per buffer, two buffers), and prefetches
// its Ca values into L2, while the warp works on the current one.  Per neuron:
//   dense phase ..... Ca / NMDA (synapse_kernels.cu:45-121) for every incoming
//                     synapse (four 32-synapse chunks per iteration); synapses
//                     that also need plasticity, dispatch or ring work go to a
//                     per-warp queue
//   event phase ..... the queue, 32 synapses at a time: LTP (post spike,
//                     synapse_kernels.cu:153-255), LTD (arrival, :257-329),
//                     dispatch capture (neuron_kernels.cu:204-206), ring read
//                     (delivery at t+1, neuron_kernels.cu:37-56), CaMKII /
//                     eligibility (t % 10, synapse_kernels.cu:469-543), PSW
//                     decay (t % 1000, scheduler.cu:55-86)
// Sums (NMDA current, next-step input) follow the canonical order: lane l
// keeps the partial of positions l, l+32, ... in ascending order (zero terms
// skipped, which is exact), then one xor butterfly.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(SYN_THREADS, SYN_MIN_BLOCKS) k_synapses(Dev d, Consts k) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) unsigned long long bars[SYN_WARPS][2];
    __shared__ int s_grab;  // next index of this CTA's post list to hand out
    if (threadIdx.x == 0) s_grab = 0;
    __syncthreads();
    if (blockIdx.x == 0) {
        if (threadIdx.x == 0) step_epilogue(d, k);
        // zero the count buffers of step t + 1 (the other parity)
        const int nb = (int)((d.ctrl->t + 1) & 1);
        for (int q = d.c0 + threadIdx.x; q < d.c1; q += blockDim.x) {
            d.col_sp[nb * d.ncol + q] = 0;
            d.l6_sp[nb * d.ncol + q] = 0;
        }
        for (int q = threadIdx.x; q < TD_DIM; q += blockDim.x) d.sub_sp[nb * TD_DIM + q] = 0;
        if (d.sharded)
            for (int q = threadIdx.x; q < 1 + TD_DIM; q += blockDim.x) d.send[d.words_max + q] = 0u;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned lt_mask = (1u << lane) - 1u;
    const int cap = d.tile_cap;  // staged elements per stream per buffer
    // per-warp shared memory: [buf0 gid | buf1 gid | queue]; Ca is read and
    // written in global memory (its row is prefetched into L2 with the staging
    // copy), which leaves the rest of the SM's on-chip memory to L1
    unsigned* const wbase = reinterpret_cast<unsigned*>(smem_raw) + (size_t)warp * (2 * cap + d.queue_cap);
    unsigned* const queue = wbase + 2 * cap;  // position | flags << 16
    unsigned long long* const bar = bars[warp];
    if (lane == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    const Ctrl* c = d.ctrl;
    PostCtx pc;
    pc.t = c->t;
    pc.gain = c->gain;
    pc.prune = c->prune_thr;
    pc.Mexc = c->M[1];
    pc.Minh = c->M[0];
    pc.e0 = c->e0 != 0;
    pc.do10 = (pc.t % 10 == 0) && !pc.e0;
    pc.do1000 = (pc.t % 1000 == 0);
    pc.slot_now = (int)((pc.t / 3) & (VAL_SLOTS - 1));
    const bool all_events = pc.do1000;
    // CTA c owns the runs of R consecutive posts that start at R (c + G i)
    // (G the grid size); its warps take the posts in order from a
    // shared-memory counter, each warp taking the post after next while it
    // stages the next one, so that the warps of a CTA work on neighbouring
    // posts and finish together (a static share of ~15 posts per warp left
    // a tail of slow warps; global counters cost more than they save)
    const int G = gridDim.x;
    constexpr int R = SYN_GRAB_RUN;
    auto grab = [&]() -> int {  // lane 0 only; increasing, d.N once past the end
        const int n = atomicAdd(&s_grab, 1);
        const long long jj = ((long long)blockIdx.x + (long long)(n / R) * G) * R + n % R;
        return jj < d.N ? (int)jj : d.N;
    };
    auto issue = [&](int rb, int re, int buf) {  // lane 0 only: the row [rb, re)
        const int a0 = rb & ~3, a1 = (re + 3) & ~3;
        const unsigned bytes = (unsigned)(a1 - a0) * 4u;
        unsigned* dst = wbase + cap * buf;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&bar[buf], bytes);
        if (bytes > 0) {
            bulk_g2s(dst, d.gid + a0, bytes, &bar[buf]);
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(d.ca + a0), "r"(bytes) : "memory");
        }
    };
    unsigned phases = 0u;  // bit s = parity of the next wait on buffer s
    int it = 0;
    // lane 0 loads the row bounds of the post after next one iteration ahead,
    // so that issuing a staging copy never waits for them
    int nb_b = 0, nb_e = 0;
    int j = d.N, jn = d.N;  // this warp's current post (all lanes) / next post (lane 0)
    if (lane == 0) {
        j = grab();
        if (j < d.N) {
            issue(d.in_ptr[j], d.in_ptr[j + 1], 0);
            jn = grab();
            if (jn < d.N) { nb_b = d.in_ptr[jn]; nb_e = d.in_ptr[jn + 1]; }
        }
    }
    j = __shfl_sync(0xffffffffu, j, 0);
    for (; j < d.N; ++it) {
        const int buf = it & 1;
        const bool has_next = __shfl_sync(0xffffffffu, jn, 0) < d.N;
        int jnn = d.N;
        if (lane == 0 && jn < d.N) {
            issue(nb_b, nb_e, buf ^ 1);
            jnn = grab();
            if (jnn < d.N) { nb_b = d.in_ptr[jnn]; nb_e = d.in_ptr[jnn + 1]; }
        }
        // this neuron's row bounds and scalars, issued before the wait so that
        // their latency overlaps the staging copy
        const int b = d.in_ptr[j], e = d.in_ptr[j + 1];
        pc.mgj = d.mg[j];
        const unsigned hist_j = d.hist[j];
        pc.xpost = d.xpost[j];
        const float V_j = d.V[j];
        bool ok = false;
        for (unsigned spin = 0; spin < WAIT_LIMIT; ++spin) {
            if (mbar_try_wait(&bar[buf], (phases >> buf) & 1u)) { ok = true; break; }
        }
        phases ^= 1u << buf;
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) {
                atomicOr(&d.ctrl->error, 1);
                if (has_next)  // drain the copy already issued (bounded) before exiting
                    for (unsigned spin = 0; spin < WAIT_LIMIT; ++spin)
                        if (mbar_try_wait(&bar[buf ^ 1], (phases >> (buf ^ 1)) & 1u)) break;
            }
            return;
        }
        const int a0 = b & ~3;
        const unsigned* sg = wbase + cap * buf;
        pc.post_spk = hist_j & 1u;
        pc.one_m_V = pm_sub(k.e_rev, V_j);
        const bool all = all_events || pc.post_spk;
        float part_nmda = 0.0f, part_in = 0.0f;
        int qn = 0;
        // dense phase: four chunks per iteration, all loads issued first; the
        // row's last 1-3 chunks go through a body of exactly that many chunks
        // (rows hold 6.6 chunks on average: padding them to a multiple of four
        // left a quarter of the dense phase's lanes idle)
        auto dense = [&](auto u_const, int base) {
            constexpr int U = decltype(u_const)::value;
            unsigned gw[U];
            float2 hv[U];
            float cav[U];
#pragma unroll
            for (int h = 0; h < U; ++h) {
                const int p = base + 32 * h + lane;
                gw[h] = p < e ? sg[p - a0] : 0u;
                cav[h] = p < e ? __ldcg(d.ca + p) : 0.0f;
            }
#pragma unroll
            for (int h = 0; h < U; ++h) {
                const int p = base + 32 * h + lane;
                hv[h] = p < e ? d.gview[gw[h] & 0x3fffffffu] : make_float2(0.0f, 0.0f);
            }
#pragma unroll
            for (int h = 0; h < U; ++h) {
                const int p = base + 32 * h + lane;
                const bool v = p < e;
                const unsigned fl = __float_as_uint(hv[h].y);
                const bool need = v && (all || (fl & GV_EV));
                {   // excitatory: Ca and NMDA current, computed for every lane
                    // (an inhibitory group's NMDA conductance is 0) and kept
                    // by predicated stores / selects
                    const bool ex = v && (gw[h] >> 31);
                    const bool ff = gw[h] & (1u << 30);
                    float ca = pm_mul(cav[h], ff ? k.dec_ca_ff : k.dec_ca);
                    const float nm = pm_mul(hv[h].x, pc.mgj);
                    ca = pm_fma(nm, k.ca_gain, ca);
                    const float cmax = ff ? k.ca_max_ff : k.ca_max;
                    ca = ca > cmax ? cmax : ca;
                    if (ex) d.ca[p] = ca;
                    const float I = pm_mul(pm_mul(nm, pc.one_m_V), k.i_gain);
                    const float sum = pm_add(part_nmda, I);
                    part_nmda = (ex && fabsf(I) > k.i_min) ? sum : part_nmda;
                }
                const unsigned m = __ballot_sync(0xffffffffu, need);
                if (need) queue[qn + __popc(m & lt_mask)] = (unsigned)(p - b) | (fl << 16);
                qn += __popc(m);
            }
        };
        {
            const int chunks = (e - b + 31) >> 5;
            int base = b;
            for (int q = 0; q + 4 <= chunks; q += 4, base += 128) dense(std::integral_constant<int, 4>{}, base);
            switch (chunks & 3) {
                case 3: dense(std::integral_constant<int, 3>{}, base); break;
                case 2: dense(std::integral_constant<int, 2>{}, base); break;
                case 1: dense(std::integral_constant<int, 1>{}, base); break;
                default: break;
            }
        }
        __syncwarp();
        // event phase: two batches of 32 queued synapses in flight, ascending
        auto accumulate = [&](float term, int off) {
            unsigned m = __ballot_sync(0xffffffffu, term != 0.0f);
            while (m) {
                const int src = __ffs(m) - 1;
                m &= m - 1;
                const int o = __shfl_sync(0xffffffffu, off, src);
                const float tv = __shfl_sync(0xffffffffu, term, src);
                if ((o & 31) == lane) part_in = pm_add(part_in, tv);
            }
        };
        for (int q0 = 0; q0 < qn; q0 += 64) {
            const int qa = q0 + lane, qb = q0 + 32 + lane;
            EvIn xa, xb;
            int offa = 0, offb = 0;
            if (qa < qn) {
                const unsigned ent = queue[qa];
                offa = (int)(ent & 0xffffu);
                const int p = b + offa;
                ev_load(d, pc, p, sg[p - a0], ent >> 16, __ldcg(d.ca + p), xa);
            }
            if (qb < qn) {
                const unsigned ent = queue[qb];
                offb = (int)(ent & 0xffffu);
                const int p = b + offb;
                ev_load(d, pc, p, sg[p - a0], ent >> 16, __ldcg(d.ca + p), xb);
            }
            const float ta = qa < qn ? ev_compute(d, k, pc, xa) : 0.0f;
            const float tb = qb < qn ? ev_compute(d, k, pc, xb) : 0.0f;
            accumulate(ta, offa);
            if (q0 + 32 < qn) accumulate(tb, offb);
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            part_nmda = pm_add(part_nmda, __shfl_xor_sync(0xffffffffu, part_nmda, o));
            part_in = pm_add(part_in, __shfl_xor_sync(0xffffffffu, part_in, o));
        }
        if (lane == 0) {
            d.nmda_cur[j] = part_nmda;
            d.input[j] = part_in;
        }
        // periodic phase (t % 10, synapse_kernels.cu:469-543), after this
        // step's LTP / LTD of every synapse of the row: CaMKII of the
        // excitatory synapses from this step's Ca, then the eligibility fold
        // e1 = e1 d1 + elig, e2 = e2 d2 + e1, elig = 0; streamed over the row
        // SYN_FOLD_U chunks at a time (coalesced), not through the event queue
        if (pc.do10) {
            __syncwarp();  // the event phase's record stores are visible to every lane
            for (int base = b; base < e; base += 32 * SYN_FOLD_U) {
                float4 q[SYN_FOLD_U];
                float t1[SYN_FOLD_U], t2[SYN_FOLD_U], av[SYN_FOLD_U], cv[SYN_FOLD_U];
#pragma unroll
                for (int h = 0; h < SYN_FOLD_U; ++h) {
                    const int p = base + 32 * h + lane;
                    q[h] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    t1[h] = t2[h] = av[h] = cv[h] = 0.0f;
                    if (p < e) {
                        q[h] = d.ev[p];
                        t1[h] = d.e1[p];
                        t2[h] = d.e2[p];
                        if (sg[p - a0] >> 31) {
                            av[h] = d.act[p];
                            cv[h] = __ldcg(d.ca + p);
                        }
                    }
                }
#pragma unroll
                for (int h = 0; h < SYN_FOLD_U; ++h) {
                    const int p = base + 32 * h + lane;
                    if (p < e) {
                        if (sg[p - a0] >> 31) {
                            camkii(k, cv[h], av[h], q[h].z);
                            d.act[p] = av[h];
                        }
                        const float a1 = pm_fma(t1[h], k.e1_dec, q[h].w);
                        d.e1[p] = a1;
                        d.e2[p] = pm_fma(t2[h], k.e2_dec, a1);
                        q[h].w = 0.0f;
                        d.ev[p] = q[h];
                    }
                }
            }
        }
        // the whole warp is done with this buffer before lane 0 refills it
        __syncwarp();
        j = __shfl_sync(0xffffffffu, jn, 0);
        jn = jnn;
    }
}

// ---------------------------------------------------------------------------
// semantic evaluation (src/stage2e/scheduler.cu:294-310 and :195-231): the
// columns' byte responses, one CTA per column, thread b adding byte b over
// the column's contiguous neurons (exact int sums); each neuron's spike total
// and chi-squared against the uniform expectation, in float, in the
// reference's order of operations
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_column_bytes(const int* __restrict__ nbc, int npc, int* __restrict__ out) {
    const int c = blockIdx.x, b = threadIdx.x;
    const int* src = nbc + (size_t)c * npc * 256 + b;
    int sum = 0;
    for (int i = 0; i < npc; ++i) sum += src[(size_t)i * 256];
    out[(size_t)c * 256 + b] = sum;
}

__global__ void __launch_bounds__(256) k_neuron_chi2(const int* __restrict__ nbc, int N, float* __restrict__ chi2,
                                                     int* __restrict__ total) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N) return;
    const int4* row = reinterpret_cast<const int4*>(nbc + (size_t)i * 256);
    int rt = 0;
    for (int q = 0; q < 64; ++q) {
        const int4 v = row[q];
        rt += v.x + v.y + v.z + v.w;
    }
    const float expected = pm_mul(pm_i2f(rt), 1.0f / 256.0f);
    float x = 0.0f;
    if (!(expected < 1e-10f))
        for (int q = 0; q < 64; ++q) {
            const int4 v = row[q];
            const int c4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float diff = pm_sub(pm_i2f(c4[u]), expected);
                x = pm_add(x, pm_div(pm_mul(diff, diff), expected));
            }
        }
    chi2[i] = x;
    total[i] = rt;
}

// Jensen-Shannon divergence of two distributions over `dim` bins, natural log
// (src/stage2e/scheduler.cu:31-40)
static double js_div(const double* P, const double* Q, int dim) {
    double js = 0.0;
    for (int b = 0; b < dim; ++b) {
        const double pi = P[b], pj = Q[b];
        const double m = 0.5 * (pi + pj);
        if (pi > 1e-12 && m > 1e-12) js += 0.5 * pi * std::log(pi / m);
        if (pj > 1e-12 && m > 1e-12) js += 0.5 * pj * std::log(pj / m);
    }
    return js < 0.0 ? 0.0 : js;
}

// ---------------------------------------------------------------------------
// host engine
// ---------------------------------------------------------------------------
struct Engine2e : snnb::Engine {
    snn_config cfg;
    cudaStream_t stream = nullptr;
    HostNet net;
    Layout lay;
    Consts K{};
    Dev D{};
    bool built = false;
    long long steps = 0;
    int raster_cap = 1024;
    long long raster_base_host = 0;  // first step of the current raster rows
    // step graphs by length (kernels read the step from device memory, so a
    // graph of n steps serves any n consecutive steps), most recently used last
    struct StepGraph {
        int n;
        cudaGraph_t g;
        cudaGraphExec_t x;
    };
    std::vector<StepGraph> graphs;
    static constexpr size_t kMaxGraphs = 4;
    // profiling: level 1 = events around every kernel of every step; level 2
    // = one event pair around each run call (no event inside the steps)
    bool profiling = false;
    int prof_level = 0;
    cudaEvent_t run_ev[2] = {nullptr, nullptr};
    std::vector<cudaEvent_t> pev;
    snn_profile prof{};
    // device buffers
    snnb::DevBuf<float> V, wad, s, fr, can, xpost, mg, input, nmda_cur, ca, act, e1, e2, val;
    snnb::DevBuf<int> last, ref, gbeg, in_ptr, gsize, gpre, col_sp, l6_sp, sub_sp, byte_histogram,
        neuron_byte_counts;
    snnb::DevBuf<unsigned short> off;
    snnb::DevBuf<unsigned> info, hist, gmeta, gid, byte_hist_nov, raster;
    snnb::DevBuf<float4> gstate, ev, gates;
    snnb::DevBuf<float2> gview, gcold, gextra;
    snnb::DevBuf<float> w_value, w_pred, baseline;
    snnb::DevBuf<Ctrl> ctrl;
    snnb::DevBuf<unsigned char> corpus;
    snnb::DevBuf<int> counts_tmp;
    int tile_cap = 0, syn_grid = 1, queue_cap = 0;
    size_t syn_smem = 0;
    // column sharding (world > 1): NCCL communicator, this rank's ranges,
    // payload buffers and the mirror groups of remote pres
    int rank = 0, world = 1;
    ncclComm_t comm = nullptr;
    // sharded runs: the mirror-group update runs on a side stream, forked at
    // the start of each step and joined before the exchange's fix-up
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    Shard sh;
    std::vector<int64_t> new_of_old;  // layout group id -> device group id
    snnb::DevBuf<unsigned> send, recv, mbit, mhist;
    snnb::DevBuf<int> mbeg, gmir;
    int64_t G_local = 0;              // groups of local pres (the rest mirror remote pres)

    explicit Engine2e(const snn_config& c) : cfg(c) {
        if (cfg.raster_steps > 0) raster_cap = cfg.raster_steps;
        SNN_CUDA(cudaSetDevice(cfg.device));
        SNN_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        set_consts();
    }
    ~Engine2e() override {
        for (auto e : pev) cudaEventDestroy(e);
        if (ev_fork) cudaEventDestroy(ev_fork);
        if (ev_join) cudaEventDestroy(ev_join);
        for (auto e : run_ev)
            if (e) cudaEventDestroy(e);
        // graphs holding NCCL calls go before the communicator
        for (auto& sg : graphs) {
            cudaGraphExecDestroy(sg.x);
            cudaGraphDestroy(sg.g);
        }
        graphs.clear();
        if (stream) cudaStreamSynchronize(stream);
        if (comm) snnb::nccl().CommDestroy(comm);
        if (side) {
            cudaStreamSynchronize(side);
            cudaStreamDestroy(side);
        }
        if (stream) {
            cudaStreamDestroy(stream);
        }
    }

    void set_consts() {
        Consts& k = K;
        // ref preset: literals of src/stage2e/neuron_kernels.cu:92-160 and
        // src/stage2e/config.h:100-303
        k.syn_keep = 0.7f; k.syn_in = 0.3f; k.vt = 0.8f; k.dT = 0.1f;
        k.inv_taum = pm_div(1.0f, 9.37f); k.a_ad = 0.0133f; k.inv_tauw = pm_div(1.0f, 144.0f);
        k.b_ad = 0.0805f; k.vmin = -0.5f; k.vmax = 1.5f;
        k.ca_n_inc = 0.2f; k.ca_n_dec = pm_sub(1.0f, pm_div(1.0f, 50.0f));
        k.fr_refr = 0.99f; k.fr_spk_keep = 0.9f; k.fr_spk_add = 0.1f; k.fr_quiet = 0.995f;
        k.off_decay = 0.999f; k.refr_steps = 2;
        k.off_add = (int)pm_mul(0.001f, 256.0f); k.off_max = (int)pm_mul(0.3f, 256.0f);
        k.dec_nmda = const_exp(pm_div(-1.0f, 150.0f));
        k.dec_ampa = const_exp(pm_div(-1.0f, 5.0f));
        k.dec_ca = const_exp(pm_div(-1.0f, 50.0f));
        k.dec_ca_ff = const_exp(pm_div(-1.0f, 10.0f));
        k.ca_max = 1.0f; k.ca_max_ff = 0.12f;
        k.rec_ff_step = pm_sub(1.0f, const_exp(pm_div(-1.0f, 3.0f)));
        k.dec_xpre = const_exp(pm_div(-1.0f, 20.0f));
        k.dec_xpost = const_exp(pm_div(-1.0f, 20.0f));
        k.g_nmda = 0.5f; k.ca_gain = 1000.0f; k.e_rev = 1.4f; k.i_gain = 0.05f; k.i_min = 1e-6f;
        const float taus_f[NCLASS] = {200.0f, 200.0f, 200.0f}, taus_r[NCLASS] = {3.0f, 500.0f, 500.0f};
        const float Us[NCLASS] = {0.02f, 0.2f, 0.05f};
        for (int q = 0; q < NCLASS; ++q) {
            k.U[q] = Us[q];
            k.fac[q] = const_exp(pm_div(-1.0f, taus_f[q]));
            k.rec[q] = pm_sub(1.0f, const_exp(pm_div(-1.0f, taus_r[q])));
        }
        k.a_plus = 0.03f; k.a_minus = 0.03f; k.w_max = 1.5f; k.eta = 20.0f; k.eta_ff = 2.0f;
        k.reb_thr = 0.15f; k.reb_gain = 0.5f; k.ab_min = 1e-4f; k.ab_reset = 0.05f; k.psw_decay = 0.95f;
        k.e1_dec = const_exp(pm_div(-10.0f, 20.0f));
        k.e2_dec = const_exp(pm_div(-10.0f, 200.0f));
        k.ck_k1 = 0.8f; k.ck_k2 = 0.1f; k.ck_k3 = 0.5f; k.ck_k4 = 0.05f; k.ck_pp1 = 0.5f; k.ck_dt = 10.0f;
        k.mod_dec[0] = const_exp(pm_div(-100.0f, 100.0f));
        k.mod_dec[1] = const_exp(pm_div(-100.0f, 200.0f));
        k.mod_dec[2] = const_exp(pm_div(-100.0f, 150.0f));
        k.mod_dec[3] = const_exp(pm_div(-100.0f, 300.0f));
        k.rec_da[0] = -0.3f; k.rec_da[1] = 0.5f;  // [0] inhibitory pre, [1] excitatory pre
        k.rec_ach = 0.3f;
        k.rec_ne = pm_div(pm_u2f((unsigned)pm_mul(0.3f, 127.0f)), 127.0f);
        k.rec_ht5 = k.rec_ne;
        k.pop_gain = 80.0f; k.gain_in = 2.0f; k.gain_out = 0.03f; k.pop_k = 100; k.inject_interval = 3;
        if (cfg.preset == SNN_PRESET_BASELINE) {
            // the benchmark's constants (C 200 pF, gL 10 nS, EL -70 mV, VT -50 mV,
            // dT 2 mV, a 2 nS, b 0.08 nA, tau_w 100 ms, dt 1 ms) in the reference's
            // normalised units: v = (V - EL) / 25 mV (VT -> 0.8, spike at 1), w in
            // gL * 25 mV; STP U 0.5, tau_d 200, tau_f 50 for every synapse class,
            // the feed-forward per-step recovery included
            k.inv_taum = pm_div(1.0f, 20.0f);
            k.inv_tauw = pm_div(1.0f, 100.0f);
            k.vt = 0.8f; k.dT = 0.08f; k.a_ad = 0.2f; k.b_ad = 0.32f;
            for (int q = 0; q < NCLASS; ++q) {
                k.U[q] = 0.5f;
                k.fac[q] = const_exp(pm_div(-1.0f, 50.0f));
                k.rec[q] = pm_sub(1.0f, const_exp(pm_div(-1.0f, 200.0f)));
            }
            k.rec_ff_step = k.rec[0];
        }
    }

    void set_shard(int32_t r, int32_t w, const void* uid) override {
        SNN_REQUIRE(!built, SNN_ERR_STATE, "shard before building the network");
        SNN_REQUIRE(w >= 1 && r >= 0 && r < w, SNN_ERR_ARG, "bad rank / world size");
        SNN_REQUIRE(comm == nullptr, SNN_ERR_STATE, "the network is sharded already");
        rank = r;
        world = w;
        if (w > 1) {
            SNN_REQUIRE(uid, SNN_ERR_ARG, "null NCCL unique id");
            ncclUniqueId id;
            memcpy(&id, uid, sizeof(id));
            SNN_CUDA(cudaSetDevice(cfg.device));
            const snnb::NcclApi& nc = snnb::nccl();
            ncclResult_t nr = nc.CommInitRank(&comm, w, id, r);
            SNN_REQUIRE(nr == ncclSuccess, SNN_ERR_CUDA,
                        std::string("ncclCommInitRank: ") + nc.GetErrorString(nr));
            SNN_CUDA(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking));
            SNN_CUDA(cudaEventCreateWithFlags(&ev_fork, cudaEventDisableTiming));
            SNN_CUDA(cudaEventCreateWithFlags(&ev_join, cudaEventDisableTiming));
        }
    }

    void build(const snn_topology_spec& spec) override {
        SNN_REQUIRE(!built, SNN_ERR_STATE, "network already built");
        SNN_REQUIRE(spec.rule == 0, SNN_ERR_UNSUPPORTED, "stage2e supports the reference rule only");
        sh = make_shard(spec, rank, world);
        generate_reference(spec, net, &sh);
        build_layout(net, lay);
        K.pref_range = 256 / net.ncol;
        const int NG = net.N;          // all neurons
        const int N = sh.n_local();    // this rank's neurons
        const int64_t S = net.S, G = lay.G;
        D.N = N; D.N_assoc = net.N_assoc; D.NPC = net.NPC; D.ncol = net.ncol; D.l4 = net.l4;
        D.per_sub = NG / TD_DIM;
        SNN_REQUIRE(D.per_sub > 0, SNN_ERR_ARG, "network too small for the 200-dim value function");
        D.n_a = sh.a1 - sh.a0; D.a0 = sh.a0; D.pf0 = sh.pf0; D.c0 = sh.c0; D.c1 = sh.c1;
        D.sharded = world > 1 ? 1 : 0;
        D.world = world;
        D.words = (N + 31) / 32;
        D.raster_cap = raster_cap;
        // neurons
        V.alloc(N); wad.alloc(N); s.alloc(N); fr.alloc(N); can.alloc(N); xpost.alloc(N); mg.alloc(N);
        input.alloc(N); nmda_cur.alloc(N); last.alloc(N); ref.alloc(N); off.alloc(N); info.alloc(N);
        hist.alloc(N); gbeg.alloc(N + 1); in_ptr.alloc(N + 1);
        for (auto* b : {&V, &wad, &s, &fr, &can, &xpost, &mg, &input, &nmda_cur}) b->zero(stream);
        ref.zero(stream); off.zero(stream); hist.zero(stream);
        std::vector<int> h_last(N, -1000);
        last.upload(h_last.data(), N, stream);
        std::vector<unsigned> h_info(N);
        std::vector<int> h_in(N + 1);
        for (int i = 0; i < N; ++i) {
            const int gi = sh.global_of(i);
            unsigned colf = net.column[gi] < 0 ? 0xffffffu : (unsigned)net.column[gi];
            h_info[i] = (unsigned)net.type[gi] | ((unsigned)net.region[gi] << 1) |
                        ((unsigned)net.subtype[gi] << 4) | (colf << 8);
            h_in[i] = lay.in_ptr[gi];  // only local neurons have incoming synapses here
        }
        h_in[N] = lay.in_ptr[NG];
        info.upload(h_info.data(), N, stream);
        in_ptr.upload(h_in.data(), N + 1, stream);
        // groups: those of local pres in local order, then the mirror groups
        // of remote pres (ascending global id)
        new_of_old.assign(G, -1);
        std::vector<int64_t> order;
        order.reserve(G);
        std::vector<int> h_gbeg(N + 1), h_mbeg;
        std::vector<unsigned> h_mbit;
        for (int i = 0; i < N; ++i) {
            const int gi = sh.global_of(i);
            h_gbeg[i] = (int)order.size();
            for (int g = lay.gbeg[gi]; g < lay.gbeg[gi + 1]; ++g) order.push_back(g);
        }
        h_gbeg[N] = (int)order.size();
        G_local = (int64_t)order.size();
        std::vector<Shard> all(world);
        for (int r = 0; r < world; ++r) all[r] = make_shard(spec, r, world);
        int words_max = 0;
        for (int r = 0; r < world; ++r) words_max = std::max(words_max, (all[r].n_local() + 31) / 32);
        const int pw = words_max + 1 + TD_DIM;
        for (int gi = 0; gi < NG; ++gi) {
            if (sh.owns(gi) || lay.gbeg[gi] == lay.gbeg[gi + 1]) continue;
            int owner = -1;
            for (int r = 0; r < world && owner < 0; ++r)
                if (all[r].owns(gi)) owner = r;
            SNN_REQUIRE(owner >= 0, SNN_ERR_STATE, "neuron without an owning shard");
            h_mbeg.push_back((int)order.size());
            h_mbit.push_back((unsigned)((int64_t)owner * pw * 32 + all[owner].local_of(gi)));
            for (int g = lay.gbeg[gi]; g < lay.gbeg[gi + 1]; ++g) order.push_back(g);
        }
        h_mbeg.push_back((int)order.size());
        SNN_REQUIRE((int64_t)order.size() == G, SNN_ERR_STATE, "group reordering lost groups");
        SNN_REQUIRE((int64_t)world * pw * 32 < (1ll << 32), SNN_ERR_ARG, "exchange payload too large");
        for (int64_t x = 0; x < G; ++x) new_of_old[order[x]] = x;
        D.M = (int)h_mbit.size();
        D.pw = pw;
        D.words_max = words_max;
        gbeg.upload(h_gbeg.data(), N + 1, stream);
        gmeta.alloc(G); gsize.alloc(G); gstate.alloc(G); gview.alloc(G); gcold.alloc(G); gextra.alloc(G);
        {
            std::vector<float2> h_ex(G, make_float2(0.0f, -1000.0f));
            gextra.upload(h_ex.data(), G, stream);
            SNN_CUDA(cudaStreamSynchronize(stream));
        }
        {
            std::vector<unsigned> packed(G);
            std::vector<int> h_gsize(G), h_gpre(G);
            std::vector<float4> h_gs(G);
            for (int64_t x = 0; x < G; ++x) {
                const int64_t g = order[x];
                SNN_REQUIRE(lay.gsize[g] < 65536, SNN_ERR_ARG, "synapse group too large");
                const unsigned lpre = x < G_local ? (unsigned)(sh.local_of(lay.gpre[g]) % NEU_BLOCK) : 0u;
                packed[x] = (lay.gmeta[g] & 0x7fu) | ((unsigned)lay.gsize[g] << 8) | (lpre << 24);
                h_gsize[x] = lay.gsize[g];
                h_gpre[x] = lay.gpre[g];
                h_gs[x] = make_float4(1.0f, cfg.preset == SNN_PRESET_BASELINE ? 0.5f : lay.gu0[g], 0.0f, 0.0f);
            }
            gmeta.upload(packed.data(), G, stream);
            gsize.upload(h_gsize.data(), G, stream);
            gpre.alloc(G);
            gpre.upload(h_gpre.data(), G, stream);
            gstate.upload(h_gs.data(), G, stream);
            SNN_CUDA(cudaStreamSynchronize(stream));
        }
        gview.zero(stream);
        gcold.zero(stream);
        mbeg.alloc(h_mbeg.size());
        mbeg.upload(h_mbeg.data(), h_mbeg.size(), stream);
        mbit.alloc(std::max<size_t>(h_mbit.size(), 1));
        if (!h_mbit.empty()) mbit.upload(h_mbit.data(), h_mbit.size(), stream);
        mhist.alloc(std::max<size_t>(h_mbit.size(), 1));
        mhist.zero(stream);
        {   // mirror pre of every mirror group
            std::vector<int> h_gmir((size_t)std::max<int64_t>(G - G_local, 1), 0);
            for (size_t m = 0; m + 1 < h_mbeg.size(); ++m)
                for (int g = h_mbeg[m]; g < h_mbeg[m + 1]; ++g) h_gmir[(size_t)(g - G_local)] = (int)m;
            gmir.alloc(h_gmir.size());
            gmir.upload(h_gmir.data(), h_gmir.size(), stream);
            SNN_CUDA(cudaStreamSynchronize(stream));
        }
        D.G_local = G_local;
        D.GM = G - G_local;
        if (world > 1) {
            send.alloc(pw);
            send.zero(stream);
            recv.alloc((size_t)world * pw);
            recv.zero(stream);
        }
        // synapses, post-major
        // gid / ca are streamed in 16-byte aligned tiles: pad by 4 elements
        gid.alloc(S + 4); ca.alloc(S + 4); ev.alloc(S); act.alloc(S); e1.alloc(S); e2.alloc(S);
        val.alloc((size_t)S * VAL_SLOTS);
        gid.zero(stream);
        for (int64_t p = 0; p < S; ++p) {  // layout group ids -> device group ids
            const uint32_t v = lay.gid_pm[p];
            lay.gid_pm[p] = (uint32_t)new_of_old[v & 0x3fffffffu] | (v & 0xc0000000u);
        }
        gid.upload(lay.gid_pm.data(), S, stream);
        SNN_CUDA(cudaStreamSynchronize(stream));
        {   // plasticity records {alpha, beta, auto, elig}, post-major
            std::vector<float4> h_ev(S);
            for (int64_t p = 0; p < S; ++p) {
                const int32_t sid = lay.perm[p];
                h_ev[p] = make_float4(net.alpha[sid], net.beta[sid], 0.0f, 0.0f);
            }
            ev.upload(h_ev.data(), S, stream);
            SNN_CUDA(cudaStreamSynchronize(stream));
        }
        // synapse pass: per-warp staging buffers sized by the largest in-degree
        {
            int max_in = 0;
            for (int j = 0; j < N; ++j) max_in = std::max(max_in, h_in[j + 1] - h_in[j]);
            SNN_REQUIRE(max_in < 65536, SNN_ERR_ARG, "in-degree above 65535");
            tile_cap = ((max_in + 6) + 3) & ~3;   // aligned range of any neuron's list
            queue_cap = (max_in + 31) & ~31;
            const size_t smem = (size_t)SYN_WARPS * (2 * (size_t)tile_cap + queue_cap) * sizeof(unsigned);
            SNN_REQUIRE(smem <= 200 * 1024, SNN_ERR_ARG, "in-degree too large for the staging buffers");
            SNN_CUDA(cudaFuncSetAttribute(k_synapses, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
            int sms = 0, per_sm = 0;
            SNN_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cfg.device));
            SNN_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_synapses, SYN_THREADS, smem));
            per_sm = std::max(per_sm, 1);
            syn_grid = std::max(1, std::min((N + SYN_WARPS - 1) / SYN_WARPS, per_sm * sms));
            syn_smem = smem;
        }
        ca.zero(stream); act.zero(stream); e1.zero(stream); e2.zero(stream); val.zero(stream);
        // control
        ctrl.alloc(1);
        Ctrl h{};
        h.byte_override = -1;
        h.learn = 1;
        h.e0 = cfg.e0;
        h.phase_offset = cfg.phase_offset;
        ctrl.upload(&h, 1, stream);
        gates.alloc(2 * (size_t)net.ncol);  // state after even / odd steps
        std::vector<float4> h_g(2 * (size_t)net.ncol, make_float4(0.5f, 0.0f, 0.0f, 0.0f));
        gates.upload(h_g.data(), 2 * (size_t)net.ncol, stream);
        col_sp.alloc(2 * net.ncol); l6_sp.alloc(2 * net.ncol); sub_sp.alloc(2 * TD_DIM);
        col_sp.zero(stream); l6_sp.zero(stream); sub_sp.zero(stream);
        byte_hist_nov.alloc(256); byte_hist_nov.zero(stream);
        byte_histogram.alloc(256); byte_histogram.zero(stream);
        neuron_byte_counts.alloc((size_t)N * 256); neuron_byte_counts.zero(stream);
        w_value.alloc(TD_DIM); w_pred.alloc(TD_DIM); baseline.alloc(TD_DIM);
        w_value.zero(stream); w_pred.zero(stream); baseline.zero(stream);
        raster.alloc((size_t)raster_cap * D.words); raster.zero(stream);
        corpus.alloc(1);
        counts_tmp.alloc(1);
        fill_dev();
        SNN_CUDA(cudaStreamSynchronize(stream));
        built = true;
    }

    void fill_dev() {
        D.V = V.p; D.wad = wad.p; D.s = s.p; D.fr = fr.p; D.can = can.p; D.xpost = xpost.p; D.mg = mg.p;
        D.input = input.p; D.nmda_cur = nmda_cur.p; D.last = last.p; D.ref = ref.p; D.off = off.p;
        D.info = info.p; D.hist = hist.p; D.gbeg = gbeg.p; D.in_ptr = in_ptr.p;
        D.gmeta = gmeta.p; D.gsize = gsize.p; D.gpre = gpre.p; D.gstate = gstate.p; D.gview = gview.p; D.gcold = gcold.p; D.gextra = gextra.p;
        D.tile_cap = tile_cap; D.queue_cap = queue_cap;
        D.gid = gid.p; D.ca = ca.p; D.ev = ev.p; D.act = act.p; D.e1 = e1.p; D.e2 = e2.p; D.val = val.p;
        D.ctrl = ctrl.p; D.gates = gates.p; D.col_sp = col_sp.p; D.l6_sp = l6_sp.p; D.sub_sp = sub_sp.p;
        D.byte_hist_nov = byte_hist_nov.p; D.byte_histogram = byte_histogram.p;
        D.neuron_byte_counts = neuron_byte_counts.p; D.w_value = w_value.p; D.w_pred = w_pred.p;
        D.baseline = baseline.p; D.corpus = corpus.p; D.raster = raster.p;
        D.send = send.p; D.recv = recv.p; D.mbeg = mbeg.p; D.mbit = mbit.p; D.mhist = mhist.p;
        D.gmir = gmir.p;
    }

    void set_corpus(const uint8_t* b, int64_t n) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_REQUIRE(n >= 0 && (n == 0 || b), SNN_ERR_ARG, "bad corpus");
        if ((size_t)n > corpus.n) {
            SNN_CUDA(cudaStreamSynchronize(stream));
            corpus.alloc(n);
            D.corpus = corpus.p;
            drop_graph();
        }
        if (n > 0) corpus.upload(b, n, stream);
        long long len = n, pos = 0;
        SNN_CUDA(cudaMemcpyAsync((char*)ctrl.p + offsetof(Ctrl, corpus_len), &len, sizeof(len),
                                 cudaMemcpyHostToDevice, stream));
        SNN_CUDA(cudaMemcpyAsync((char*)ctrl.p + offsetof(Ctrl, corpus_pos), &pos, sizeof(pos),
                                 cudaMemcpyHostToDevice, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
    }

    // callers synchronize the stream first
    void drop_graph() {
        for (auto& sg : graphs) {
            cudaGraphExecDestroy(sg.x);
            cudaGraphDestroy(sg.g);
        }
        graphs.clear();
    }

    // kernels (timing slots) per step: control, neurons, [exchange + mirror
    // groups when sharded], synapses
    int nslot() const { return world > 1 ? 3 : 2; }

    // one step; with profiling, events ev[0..nslot] bracket the slots
    // (inside a stream capture the records must be "external" so that they
    // become event-record nodes that time the graph's kernels)
    void launch_step(cudaStream_t st, cudaEvent_t* ev = nullptr, bool capturing = false) {
        const int nb = (D.N + NEU_BLOCK - 1) / NEU_BLOCK;
        const unsigned fl = capturing ? cudaEventRecordExternal : cudaEventRecordDefault;
        int e = 0;
        if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[e++], st, fl));
        if (world > 1) {  // mirror groups from spikes up to t - 1, beside k_neurons and the exchange
            SNN_CUDA(cudaEventRecord(ev_fork, st));
            SNN_CUDA(cudaStreamWaitEvent(side, ev_fork, 0));
            k_mirror_groups<<<(unsigned)std::max(1ll, (D.GM + 255) / 256), 256, 0, side>>>(D, K);
            SNN_CUDA(cudaEventRecord(ev_join, side));
        }
        k_neurons<<<nb, NEU_THREADS, 0, st>>>(D, K);
        if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[e++], st, fl));
        if (world > 1) {
            const snnb::NcclApi& nc = snnb::nccl();
            const ncclResult_t nr = nc.AllGather(send.p, recv.p, (size_t)D.pw, ncclUint32, comm, st);
            SNN_REQUIRE(nr == ncclSuccess, SNN_ERR_CUDA, std::string("ncclAllGather: ") + nc.GetErrorString(nr));
            SNN_CUDA(cudaStreamWaitEvent(st, ev_join, 0));
            k_mirror_hist<<<std::max(1, (D.M + 255) / 256), 256, 0, st>>>(D);
            if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[e++], st, fl));
        }
        k_synapses<<<syn_grid, SYN_THREADS, syn_smem, st>>>(D, K);
        if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[e++], st, fl));
    }

    void ensure_events(int n_steps) {
        size_t need = (size_t)n_steps * (nslot() + 1);
        while (pev.size() < need) {
            cudaEvent_t e;
            SNN_CUDA(cudaEventCreate(&e));
            pev.push_back(e);
        }
    }

    // accumulate the profile of n steps whose events are pev[0 .. 3n]
    // accumulate the profile of n steps starting at step t0; slot 3 also
    // collects the synapse pass of steps with t % 10 == 0 (CaMKII /
    // eligibility schedule), which move most bytes
    void harvest(int n, long long t0) {
        SNN_CUDA(cudaStreamSynchronize(stream));
        const int ns = nslot();
        for (int q = 0; q < n; ++q) {
            for (int kk = 0; kk < ns; ++kk) {
                float ms = 0.0f;
                SNN_CUDA(cudaEventElapsedTime(&ms, pev[ns * q + kk], pev[ns * q + kk + 1]));
                prof.kernel_ms[kk] += ms;
                prof.launches[kk] += 1;
                prof.step_ms += ms;
                if (kk == ns - 1 && (t0 + q) % 10 == 0) {
                    prof.kernel_ms[ns] += ms;
                    prof.launches[ns] += 1;
                }
            }
        }
        prof.steps += n;
    }

    // the graph of `n` steps, captured on first use; the least recently used
    // of more than kMaxGraphs lengths is released (after the stream drains)
    cudaGraphExec_t graph_for(int n) {
        for (size_t i = 0; i < graphs.size(); ++i)
            if (graphs[i].n == n) {
                const StepGraph sg = graphs[i];
                graphs.erase(graphs.begin() + (long)i);
                graphs.push_back(sg);
                return sg.x;
            }
        if (graphs.size() >= kMaxGraphs) {
            SNN_CUDA(cudaStreamSynchronize(stream));
            cudaGraphExecDestroy(graphs.front().x);
            cudaGraphDestroy(graphs.front().g);
            graphs.erase(graphs.begin());
        }
        if (profiling) ensure_events(n);
        StepGraph sg{n, nullptr, nullptr};
        SNN_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
        for (int q = 0; q < n; ++q) launch_step(stream, profiling ? &pev[(size_t)nslot() * q] : nullptr, true);
        SNN_CUDA(cudaStreamEndCapture(stream, &sg.g));
        const cudaError_t ie = cudaGraphInstantiate(&sg.x, sg.g, 0);
        if (ie != cudaSuccess) cudaGraphDestroy(sg.g);
        SNN_CUDA(ie);
        graphs.push_back(sg);
        return sg.x;
    }

    void set_profiling(int32_t en) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_REQUIRE(en >= 0 && en <= 2, SNN_ERR_ARG, "profiling level must be 0, 1 or 2");
        SNN_CUDA(cudaStreamSynchronize(stream));
        prof_level = en;
        profiling = en == 1;
        if (en == 2 && !run_ev[0]) {
            SNN_CUDA(cudaEventCreate(&run_ev[0]));
            SNN_CUDA(cudaEventCreate(&run_ev[1]));
        }
        drop_graph();
        memset(&prof, 0, sizeof(prof));
        int q = 0;
        strcpy(prof.names[q++], "k_neurons");
        if (world > 1) strcpy(prof.names[q++], "allgather+mirror");
        strcpy(prof.names[q++], "k_synapses");
        strcpy(prof.names[q++], "k_synapses@t%10==0");
        prof.n_kernels = q;
    }

    void get_profile(snn_profile* o) override { *o = prof; }

    void set_ctrl_field(size_t off_b, const void* v, size_t n) {
        SNN_CUDA(cudaMemcpyAsync((char*)ctrl.p + off_b, v, n, cudaMemcpyHostToDevice, stream));
    }

    void run(int32_t n_steps, int32_t byte_override, int32_t learn, uint32_t* raster_out,
             int32_t* counts_out) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_REQUIRE(n_steps >= 0, SNN_ERR_ARG, "negative step count");
        if (n_steps == 0) return;
        int lr = learn ? 1 : 0;
        set_ctrl_field(offsetof(Ctrl, learn), &lr, sizeof(int));
        long long rb = steps;
        raster_base_host = rb;
        set_ctrl_field(offsetof(Ctrl, raster_base), &rb, sizeof(rb));
        if (byte_override >= 0) {
            SNN_REQUIRE(byte_override < 256, SNN_ERR_ARG, "byte out of range");
            set_ctrl_field(offsetof(Ctrl, byte_override), &byte_override, sizeof(int));
        }
        int done = 0;
        const int chunk = 50;
        // raster rows wrap every raster_cap steps: the run is cut into spans
        // that end at a wrap, each span into graphs of `chunk` steps and one
        // of the remainder
        auto span_at = [&](int d0) { return std::min(n_steps - d0, raster_cap - (d0 % raster_cap)); };
        if (prof_level == 2) {  // every graph built before the first event: no host work timed
            for (int d0 = 0; d0 < n_steps; d0 += span_at(d0)) {
                const int sp = span_at(d0);
                if (sp >= chunk) graph_for(chunk);
                if (sp % chunk) graph_for(sp % chunk);
            }
            SNN_CUDA(cudaEventRecord(run_ev[0], stream));
        }
        while (done < n_steps) {
            const int span = span_at(done);  // rows drained before they are overwritten
            int q = 0;
            while (q < span) {
                const int m = std::min(chunk, span - q);
                SNN_CUDA(cudaGraphLaunch(graph_for(m), stream));
                if (profiling) harvest(m, steps + done + q);
                q += m;
            }
            if (raster_out || counts_out) {
                const long long row0 = (done % raster_cap);
                if (raster_out)
                    SNN_CUDA(cudaMemcpyAsync(raster_out + (size_t)done * D.words,
                                             raster.p + row0 * D.words,
                                             (size_t)span * D.words * sizeof(unsigned),
                                             cudaMemcpyDeviceToHost, stream));
                if (counts_out) {
                    // counted from the caller's copy of the rows when there is
                    // one, else from a copy of our own
                    std::vector<unsigned> tmp;
                    const uint32_t* rows = raster_out ? raster_out + (size_t)done * D.words : nullptr;
                    if (!rows) {
                        tmp.resize((size_t)span * D.words);
                        SNN_CUDA(cudaMemcpyAsync(tmp.data(), raster.p + row0 * D.words,
                                                 tmp.size() * sizeof(unsigned), cudaMemcpyDeviceToHost,
                                                 stream));
                        rows = tmp.data();
                    }
                    SNN_CUDA(cudaStreamSynchronize(stream));
                    for (int r = 0; r < span; ++r) {
                        int cnt = 0;
                        for (int w = 0; w < D.words; ++w) cnt += __builtin_popcount(rows[(size_t)r * D.words + w]);
                        counts_out[done + r] = cnt;
                    }
                }
                SNN_CUDA(cudaStreamSynchronize(stream));
            }
            done += span;
        }
        if (prof_level == 2) {
            SNN_CUDA(cudaEventRecord(run_ev[1], stream));
            SNN_CUDA(cudaEventSynchronize(run_ev[1]));
            float ms = 0.0f;
            SNN_CUDA(cudaEventElapsedTime(&ms, run_ev[0], run_ev[1]));
            prof.step_ms += ms;
            prof.steps += n_steps;
        }
        steps += n_steps;
        SNN_CUDA(cudaGetLastError());
    }

    void check_device_error() {
        int err = 0;
        SNN_CUDA(cudaMemcpyAsync(&err, (char*)ctrl.p + offsetof(Ctrl, error), sizeof(int),
                                 cudaMemcpyDeviceToHost, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
        SNN_REQUIRE(err == 0, SNN_ERR_CUDA, "a kernel's bounded wait for its staged data ran out");
    }
    void sync() override {
        SNN_CUDA(cudaStreamSynchronize(stream));
        check_device_error();
    }
    int64_t steps_done() const override { return steps; }

    void counters(snn_counters* o) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        Ctrl h;
        SNN_CUDA(cudaMemcpyAsync(&h, ctrl.p, sizeof(Ctrl), cudaMemcpyDeviceToHost, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
        SNN_REQUIRE(h.error == 0, SNN_ERR_CUDA, "a kernel's bounded wait for its staged data ran out");
        memset(o, 0, sizeof(*o));
        o->step = steps;
        o->total_spikes = h.total_spikes;
        o->arrivals = (int64_t)h.arrivals;
        o->dispatched = (int64_t)h.dispatched;
        o->dropped_ref = (int64_t)h.dropped_ref;
        o->ltp_visits = (int64_t)h.ltp_visits;
        o->burst_spikes = (int64_t)h.burst;
        o->n_neurons = D.N;   // this rank's neurons (all of them unsharded)
        o->n_synapses = net.S;
        o->n_groups = lay.G;
        o->last_spikes = steps > 0 ? h.step_spikes[(steps - 1) & 1] : 0;
        o->last_byte = steps > 0 ? h.byte : -1;
        o->modeled_bytes = modeled_bytes(steps, (double)h.arrivals, (double)h.dispatched,
                                         (double)h.ltp_visits);
    }

    // Algorithmic HBM bytes of the synapse pass over the first `n` steps
    // (the traffic its semantics require under this layout): every step the
    // group id of every synapse (4 B) and the Ca of every excitatory synapse
    // (read + write, 8 B); per dispatched edge 12 B (alpha, beta read; value
    // write); per arrival 36 B (value read; plasticity record read + write);
    // per LTP visit 32 B (plasticity record read + write); every 10 steps
    // eligibility (8 B) and e1 / e2 (16 B) of every synapse plus CaMKII act /
    // autophosphorylation (16 B) of every excitatory one, read + write; every
    // 1000 steps alpha / beta (16 B) of every synapse.
    double modeled_bytes(long long n, double arr, double disp, double ltp) const {
        double s_exc = 0;
        for (int64_t g = 0; g < lay.G; ++g)
            if (lay.gmeta[g] & GV_EXC) s_exc += lay.gsize[g];
        const double S = (double)net.S;
        const double dense = n * (4.0 * S + 8.0 * s_exc);
        const double periodic = (double)((n + 9) / 10) * (24.0 * S + 16.0 * s_exc) +
                                (double)((n + 999) / 1000) * 16.0 * S;
        const double events = disp * 12.0 + arr * 36.0 + ltp * 32.0;
        return dense + periodic + events;
    }

    void get_spikes(uint32_t* words, int64_t n_words) override {
        SNN_REQUIRE(built && steps > 0, SNN_ERR_STATE, "no step executed yet");
        SNN_REQUIRE(n_words >= D.words, SNN_ERR_ARG, "bitmask buffer too small");
        const long long row = (steps - 1 - raster_base_host) % raster_cap;
        SNN_CUDA(cudaMemcpyAsync(words, raster.p + row * D.words, D.words * sizeof(unsigned),
                                 cudaMemcpyDeviceToHost, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
    }

    // device group of every kept synapse, in the reference (pre-major) order
    std::vector<uint32_t> sid_group_cache;
    const std::vector<uint32_t>& sid_groups() {
        if (!sid_group_cache.empty() || net.S == 0) return sid_group_cache;
        sid_group_cache.resize(net.S);
        for (int pre = 0; pre < net.N; ++pre) {
            for (int32_t sid = net.row_ptr[pre]; sid < net.row_ptr[pre + 1]; ++sid) {
                const int key = eff_delay(net.delay[sid]) * 2 + ((net.flags[sid] & RF_FF) ? 1 : 0);
                int g = lay.gbeg[pre];
                while (g < lay.gbeg[pre + 1]) {
                    const uint32_t m = lay.gmeta[g];
                    if ((int)((m & GV_D_MASK) * 2 + ((m & GV_FF) ? 1 : 0)) == key) break;
                    ++g;
                }
                sid_group_cache[sid] = (uint32_t)new_of_old[g];
            }
        }
        return sid_group_cache;
    }

    template <typename T>
    std::vector<T> fetch(const snnb::DevBuf<T>& b, size_t n) {
        std::vector<T> h(n);
        b.download(h.data(), n, stream);
        SNN_CUDA(cudaStreamSynchronize(stream));
        return h;
    }

    // BioMechanismScheduler::launch_semantic_eval (src/stage2e/scheduler.cu:785-1036)
    void semantic_eval(int64_t step, snn_semantic* o, int32_t* assign_out, int64_t n_assign) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_REQUIRE(world == 1, SNN_ERR_UNSUPPORTED, "semantic evaluation of a sharded network is not available");
        const int NC = net.ncol, NB = 256, N = D.N;
        SNN_REQUIRE(NC >= 1, SNN_ERR_STATE, "the network has no columns");
        SNN_REQUIRE(!assign_out || n_assign >= NC, SNN_ERR_ARG, "cluster buffer smaller than the column count");
        snnb::DevBuf<int> d_col, d_tot;
        snnb::DevBuf<float> d_chi;
        d_col.alloc((size_t)NC * NB);
        d_tot.alloc(N);
        d_chi.alloc(N);
        k_column_bytes<<<NC, NB, 0, stream>>>(neuron_byte_counts.p, D.NPC, d_col.p);
        k_neuron_chi2<<<(N + 255) / 256, 256, 0, stream>>>(neuron_byte_counts.p, N, d_chi.p, d_tot.p);
        SNN_CUDA(cudaGetLastError());
        const std::vector<int> resp = fetch(d_col, (size_t)NC * NB);
        const std::vector<int> tot = fetch(d_tot, N);
        const std::vector<float> chi = fetch(d_chi, N);
        const std::vector<int> lst = fetch(last, N);
        memset(o, 0, sizeof(*o));
        o->n_columns = NC;
        // column distributions (an empty column counts as uniform)
        std::vector<double> P((size_t)NC * NB), col_total(NC, 0.0);
        double grand = 0.0;
        for (int c = 0; c < NC; ++c) {
            double sum = 0.0;
            for (int b = 0; b < NB; ++b) sum += resp[(size_t)c * NB + b];
            col_total[c] = sum;
            grand += sum;
            for (int b = 0; b < NB; ++b)
                P[(size_t)c * NB + b] = sum < 1e-10 ? 1.0 / NB : resp[(size_t)c * NB + b] / sum;
        }
        o->grand_total = grand;
        // pairwise JS
        std::vector<double> js((size_t)NC * NC, 0.0);
        double js_sum = 0.0, js_max = 0.0;
        long long js_n = 0;
        for (int i = 0; i < NC; ++i)
            for (int j = i + 1; j < NC; ++j) {
                const double v = js_div(&P[(size_t)i * NB], &P[(size_t)j * NB], NB);
                js[(size_t)i * NC + j] = js[(size_t)j * NC + i] = v;
                js_sum += v;
                if (v > js_max) js_max = v;
                ++js_n;
            }
        o->js_mean = js_n > 0 ? js_sum / js_n : 0.0;
        o->js_max = js_max;
        // k-means, k 5, JS distance, round-robin start
        const int K = 5;
        std::vector<int> asg(NC);
        for (int i = 0; i < NC; ++i) asg[i] = i % K;
        std::vector<double> cen((size_t)K * NB);
        for (int iter = 0; iter < 20; ++iter) {
            std::vector<int> cnt(K, 0);
            std::vector<double> sp((size_t)K * NB, 0.0);
            for (int i = 0; i < NC; ++i) {
                cnt[asg[i]]++;
                for (int b = 0; b < NB; ++b) sp[(size_t)asg[i] * NB + b] += P[(size_t)i * NB + b];
            }
            for (int k = 0; k < K; ++k) {
                double* ck = &cen[(size_t)k * NB];
                if (cnt[k] > 0) {
                    double sum = 0.0;
                    for (int b = 0; b < NB; ++b) {
                        ck[b] = sp[(size_t)k * NB + b] / cnt[k];
                        sum += ck[b];
                    }
                    for (int b = 0; b < NB; ++b) ck[b] = sum < 1e-12 ? 1.0 / NB : ck[b] / sum;
                } else {
                    for (int b = 0; b < NB; ++b) ck[b] = 1.0 / NB;
                }
            }
            bool changed = false;
            for (int i = 0; i < NC; ++i) {
                double best = std::numeric_limits<double>::max();
                int bk = 0;
                for (int k = 0; k < K; ++k) {
                    const double dd = js_div(&P[(size_t)i * NB], &cen[(size_t)k * NB], NB);
                    if (dd < best) { best = dd; bk = k; }
                }
                if (bk != asg[i]) { asg[i] = bk; changed = true; }
            }
            if (!changed) break;
        }
        // silhouette on the JS matrix
        double sil = 0.0;
        int sil_n = 0;
        for (int i = 0; i < NC; ++i) {
            double a = 0.0, bmin = std::numeric_limits<double>::max();
            int an = 0;
            for (int k = 0; k < K; ++k) {
                if (k == asg[i]) {
                    for (int j = 0; j < NC; ++j)
                        if (j != i && asg[j] == k) { a += js[(size_t)i * NC + j]; ++an; }
                    if (an > 0) a /= an;
                } else {
                    double ds = 0.0;
                    int dn = 0;
                    for (int j = 0; j < NC; ++j)
                        if (asg[j] == k) { ds += js[(size_t)i * NC + j]; ++dn; }
                    if (dn > 0 && ds / dn < bmin) bmin = ds / dn;
                }
            }
            if (an > 0 && bmin < std::numeric_limits<double>::max()) {
                const double den = a > bmin ? a : bmin;
                sil += den > 1e-12 ? (bmin - a) / den : 0.0;
                ++sil_n;
            }
        }
        o->silhouette = sil_n > 0 ? sil / sil_n : 0.0;
        // column ratio over the non-zero columns
        double cmin = std::numeric_limits<double>::max(), cmax = 0.0;
        int nz = 0;
        for (int c = 0; c < NC; ++c)
            if (col_total[c] > 0.0) {
                cmin = std::min(cmin, col_total[c]);
                cmax = std::max(cmax, col_total[c]);
                ++nz;
            }
        o->nonzero_columns = nz;
        o->column_ratio = (nz >= 2 && cmin > 0.0) ? cmax / cmin : 0.0;
        // per layer: mean spike delay after the last injection step before
        // `step`, and chi-squared selectivity (float sums in neuron order)
        long long li = ((step - 1) / 3) * 3;
        if (li < 0) li = 0;
        double dsum[5] = {0, 0, 0, 0, 0};
        float csum[5] = {0, 0, 0, 0, 0};
        for (int i = 0; i < N; ++i) {
            const int r = net.region[i];
            if (r > 4) continue;
            if (lst[i] >= li) {
                dsum[r] += (double)(lst[i] - li);
                o->layer_delay_n[r]++;
            }
            if (tot[i] >= 10) {
                o->layer_act[r]++;
                csum[r] = pm_add(csum[r], chi[i]);
                if (chi[i] > 293.2f) o->layer_sig[r]++;
            }
        }
        for (int r = 0; r < 5; ++r) {
            o->layer_delay[r] = o->layer_delay_n[r] > 0 ? dsum[r] / o->layer_delay_n[r] : -1.0;
            o->layer_chi2_mean[r] = o->layer_act[r] > 0 ? (double)csum[r] / (double)o->layer_act[r] : 0.0;
        }
        if (assign_out)
            for (int i = 0; i < NC; ++i) assign_out[i] = asg[i];
    }

    void get_state(int32_t which, void* buf, int64_t nbytes) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        const int N = D.N;    // this rank's neurons
        const int NG = net.N; // pres of the kept synapses' row pointer
        const int64_t S = net.S;
        auto need = [&](int64_t bytes) {
            SNN_REQUIRE(nbytes >= bytes, SNN_ERR_ARG, "state buffer too small");
        };
        auto neuron_f = [&](const snnb::DevBuf<float>& b) {
            need((int64_t)N * 4);
            b.download((float*)buf, N, stream);
            SNN_CUDA(cudaStreamSynchronize(stream));
        };
        auto neuron_i = [&](const snnb::DevBuf<int>& b) {
            need((int64_t)N * 4);
            b.download((int*)buf, N, stream);
            SNN_CUDA(cudaStreamSynchronize(stream));
        };
        // post-major synapse array -> reference (pre-major) order
        auto syn_pm = [&](const std::vector<float>& pm) {
            need(S * 4);
            float* o = (float*)buf;
            for (int64_t p = 0; p < S; ++p) o[lay.perm[p]] = pm[p];
        };
        // group state -> per synapse (pre-major)
        (void)NG;
        auto syn_group = [&](int comp) {
            need(S * 4);
            auto gs = fetch(gstate, lay.G);
            const auto& sg = sid_groups();
            float* o = (float*)buf;
            for (int64_t sid = 0; sid < S; ++sid) {
                const float4 v = gs[sg[sid]];
                o[sid] = comp == 0 ? v.x : comp == 1 ? v.y : comp == 2 ? v.z : v.w;
            }
        };
        auto syn_extra = [&](int comp) {
            need(S * 4);
            auto gx = fetch(gextra, lay.G);
            const auto& sg = sid_groups();
            float* o = (float*)buf;
            for (int64_t sid = 0; sid < S; ++sid) o[sid] = comp == 0 ? gx[sg[sid]].x : gx[sg[sid]].y;
        };
        auto ev_comp = [&](int comp) {
            auto h = fetch(ev, S);
            std::vector<float> pm(S);
            for (int64_t p = 0; p < S; ++p) {
                const float4 v = h[p];
                pm[p] = comp == 0 ? v.x : comp == 1 ? v.y : comp == 2 ? v.z : v.w;
            }
            syn_pm(pm);
        };
        switch (which) {
            case SNN_STATE_V: neuron_f(V); break;
            case SNN_STATE_W_ADAPT: neuron_f(wad); break;
            case SNN_STATE_SYN_CURRENT: neuron_f(s); break;
            case SNN_STATE_FIRE_RATE: neuron_f(fr); break;
            case SNN_STATE_CA_NEURON: neuron_f(can); break;
            case SNN_STATE_INPUT: neuron_f(input); break;
            case SNN_STATE_NMDA_CUR: neuron_f(nmda_cur); break;
            case SNN_STATE_LAST_SPIKE: neuron_i(last); break;
            case SNN_STATE_REFRACTORY: neuron_i(ref); break;
            case SNN_STATE_X_POST: neuron_f(xpost); break;
            case SNN_STATE_THRESH_OFF: {
                need((int64_t)N * 4);
                auto h = fetch(off, N);
                for (int i = 0; i < N; ++i) ((int*)buf)[i] = h[i];
                break;
            }
            case SNN_STATE_ALPHA: ev_comp(0); break;
            case SNN_STATE_BETA: ev_comp(1); break;
            case SNN_STATE_CAMKII_AUTO: ev_comp(2); break;
            case SNN_STATE_ELIG: ev_comp(3); break;
            case SNN_STATE_WEIGHT: {
                auto h = fetch(ev, S);
                std::vector<float> pm(S);
                for (int64_t p = 0; p < S; ++p) {
                    float m = pm_div(pm_mul(1.5f, h[p].x), pm_add(h[p].x, h[p].y));
                    pm[p] = (net.flags[lay.perm[p]] & (RF_AMPA | RF_NMDA)) ? m : -m;
                }
                syn_pm(pm);
                break;
            }
            case SNN_STATE_CA: syn_pm(fetch(ca, S)); break;
            case SNN_STATE_CAMKII_ACT: syn_pm(fetch(act, S)); break;
            case SNN_STATE_E1: syn_pm(fetch(e1, S)); break;
            case SNN_STATE_E2: syn_pm(fetch(e2, S)); break;
            case SNN_STATE_RESOURCE: syn_group(0); break;
            case SNN_STATE_UTIL: syn_group(1); break;
            case SNN_STATE_NMDA_G: syn_group(2); break;
            case SNN_STATE_X_PRE: syn_group(3); break;
            case SNN_STATE_AMPA: syn_extra(0); break;
            case SNN_STATE_LAST_PRE: syn_extra(1); break;
            case SNN_STATE_POST: need(S * 4); memcpy(buf, net.post.data(), S * 4); break;
            case SNN_STATE_DELAY: need(S); memcpy(buf, net.delay.data(), S); break;
            case SNN_STATE_FLAGS: need(S); memcpy(buf, net.flags.data(), S); break;
            case SNN_STATE_ROW_PTR: need((int64_t)(NG + 1) * 4); memcpy(buf, net.row_ptr.data(), (NG + 1) * 4); break;
            case SNN_STATE_GATES: {
                need((int64_t)net.ncol * 16);
                const size_t half = steps > 0 ? (size_t)((steps - 1) & 1) : 1;  // after the last step
                SNN_CUDA(cudaMemcpyAsync(buf, gates.p + half * net.ncol, (size_t)net.ncol * sizeof(float4),
                                         cudaMemcpyDeviceToHost, stream));
                SNN_CUDA(cudaStreamSynchronize(stream));
                break;
            }
            case SNN_STATE_MODULATORS: {
                need(16);
                Ctrl h;
                ctrl.download(&h, 1, stream);
                SNN_CUDA(cudaStreamSynchronize(stream));
                memcpy(buf, h.conc, 16);
                break;
            }
            case SNN_STATE_BYTE_HIST: {
                need(256 * 4);
                byte_histogram.download((int*)buf, 256, stream);
                SNN_CUDA(cudaStreamSynchronize(stream));
                break;
            }
            case SNN_STATE_NEURON_BYTE_COUNTS: {
                need((int64_t)N * 256 * 4);
                neuron_byte_counts.download((int*)buf, (size_t)N * 256, stream);
                SNN_CUDA(cudaStreamSynchronize(stream));
                break;
            }
            default: throw snnb::Error(SNN_ERR_ARG, "unknown state field");
        }
    }

    void set_e0(int32_t en) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        int v = en ? 1 : 0;
        set_ctrl_field(offsetof(Ctrl, e0), &v, sizeof(int));
        SNN_CUDA(cudaStreamSynchronize(stream));
    }

    // ---- checkpoints ------------------------------------------------------
    struct NativeBlob {  // host-side state + a fingerprint of the network
        int64_t steps, raster_base, N, S, G, M;
        int32_t rank, world, ncol, raster_cap;
    };
    std::vector<snnb::DevSection> native_sections() {
        std::vector<snnb::DevSection> v;
        auto add = [&](const char* n, auto& b) { v.push_back({n, (void*)b.p, b.bytes()}); };
        add("V", V); add("wad", wad); add("s", s); add("fr", fr); add("can", can);
        add("xpost", xpost); add("mg", mg); add("input", input); add("nmda_cur", nmda_cur);
        add("last", last); add("ref", ref); add("off", off); add("hist", hist);
        add("gstate", gstate); add("gview", gview); add("gcold", gcold); add("gextra", gextra);
        add("ca", ca); add("ev", ev); add("act", act); add("e1", e1); add("e2", e2); add("val", val);
        add("ctrl", ctrl); add("gates", gates); add("col_sp", col_sp); add("l6_sp", l6_sp);
        add("sub_sp", sub_sp); add("byte_hist_nov", byte_hist_nov); add("byte_histogram", byte_histogram);
        add("neuron_byte_counts", neuron_byte_counts); add("w_value", w_value); add("w_pred", w_pred);
        add("baseline", baseline); add("raster", raster); add("mhist", mhist);
        return v;
    }
    NativeBlob blob() const {
        NativeBlob b{};
        b.steps = steps; b.raster_base = raster_base_host; b.N = D.N; b.S = net.S; b.G = lay.G; b.M = D.M;
        b.rank = rank; b.world = world; b.ncol = net.ncol; b.raster_cap = raster_cap;
        return b;
    }

    // SCKP v2 (src/stage2e/scheduler.cu:411-483): this rank's synapses as the
    // reference's 80-byte BioSynapse records in reference synapse order, the
    // neuron x byte counts, alpha, beta; `step` = steps executed
    struct BioSyn {
        int32_t pre, post;
        float weight, delay_steps, last_pre, last_post, x_pre, x_post;
        float nmda, ampa, ca, resource, elig, elig_slow, util, scaling;
        float autoph, da_r, ach_r;
        uint8_t flags, ne_u8, ht5_u8, pad;
    };
    static_assert(sizeof(BioSyn) == 80, "BioSynapse record");
    void write_sckp(const char* path) {
        const int64_t S = net.S;
        SNN_REQUIRE(S < (1ll << 32) && D.N >= 0, SNN_ERR_ARG, "too many synapses for SCKP v2");
        auto gs = fetch(gstate, lay.G);
        auto gx = fetch(gextra, lay.G);
        auto evh = fetch(ev, S);
        auto cah = fetch(ca, S);
        auto xp = fetch(xpost, D.N);
        auto lst = fetch(last, D.N);
        const auto& sg = sid_groups();
        std::vector<BioSyn> aos(S);
        std::vector<float> al(S), be(S);
        const uint8_t r38 = (uint8_t)pm_mul(0.3f, 127.0f);
        for (int pre = 0; pre < net.N; ++pre) {
            for (int32_t sid = net.row_ptr[pre]; sid < net.row_ptr[pre + 1]; ++sid) {
                BioSyn& b = aos[sid];
                memset(&b, 0, sizeof(b));
                const int post = net.post[sid];
                const int lp = sh.local_of(post);
                const bool exc = net.flags[sid] & (RF_AMPA | RF_NMDA);
                const float4 g = gs[sg[sid]];
                const float2 x = gx[sg[sid]];
                b.pre = pre; b.post = post;
                b.delay_steps = pm_i2f(net.delay[sid]);
                b.last_pre = x.y; b.last_post = pm_i2f(lst[lp]);
                b.x_pre = g.w; b.x_post = xp[lp];
                b.nmda = g.z; b.ampa = x.x; b.resource = g.x; b.util = g.y;
                b.elig_slow = 0.0f; b.scaling = 1.0f;
                b.da_r = exc ? 0.5f : -0.3f; b.ach_r = 0.3f;
                b.flags = net.flags[sid]; b.ne_u8 = r38; b.ht5_u8 = r38;
            }
        }
        for (int64_t p = 0; p < S; ++p) {
            const int32_t sid = lay.perm[p];
            BioSyn& b = aos[sid];
            const float4 e = evh[p];
            const float m = pm_div(pm_mul(1.5f, e.x), pm_add(e.x, e.y));
            b.weight = (b.flags & (RF_AMPA | RF_NMDA)) ? m : -m;
            b.ca = cah[p]; b.elig = e.w; b.autoph = e.z;
            al[sid] = e.x; be[sid] = e.y;
        }
        auto nbc = fetch(neuron_byte_counts, (size_t)D.N * 256);
        snnb::BinFile f(path, true);
        const uint32_t hdr[5] = {0x53434B50u, 2u, (uint32_t)steps, (uint32_t)S, (uint32_t)D.N};
        f.put(hdr, sizeof(hdr));
        f.put(aos.data(), sizeof(BioSyn) * (size_t)S);
        f.put(nbc.data(), sizeof(int) * nbc.size());
        f.put(al.data(), 4 * (size_t)S);
        f.put(be.data(), 4 * (size_t)S);
        f.close();
    }

    void save(const char* path, int32_t fmt) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_CUDA(cudaStreamSynchronize(stream));
        if (fmt == SNN_FMT_NATIVE) {
            const NativeBlob b = blob();
            snnb::save_native(path, SNN_MODEL_STAGE2E, &b, sizeof(b), native_sections(), stream);
        } else if (fmt == SNN_FMT_SCKP_V2) {
            write_sckp(path);
        } else if (fmt == SNN_FMT_RAW_F32) {  // weights in reference synapse order
            std::vector<float> w(net.S);
            get_state(SNN_STATE_WEIGHT, w.data(), (int64_t)w.size() * 4);
            snnb::BinFile f(path, true);
            f.put(w.data(), w.size() * 4);
            f.close();
        } else {
            throw snnb::Error(SNN_ERR_UNSUPPORTED, "Stage 2e writes the native, SCKP v2 and raw formats");
        }
    }
    void load(const char* path, int32_t fmt) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_REQUIRE(fmt == SNN_FMT_NATIVE, SNN_ERR_UNSUPPORTED,
                    "Stage 2e resumes from the native format (SCKP v2 has no reader in the reference)");
        const NativeBlob want = blob();
        NativeBlob got{};
        snnb::load_native(path, SNN_MODEL_STAGE2E, &got, sizeof(got), native_sections(), stream,
                          [&](const void* p) {
                              NativeBlob f;
                              memcpy(&f, p, sizeof(f));
                              SNN_REQUIRE(f.N == want.N && f.S == want.S && f.G == want.G && f.M == want.M &&
                                              f.rank == want.rank && f.world == want.world &&
                                              f.ncol == want.ncol && f.raster_cap == want.raster_cap,
                                          SNN_ERR_IO, "checkpoint of another network or shard");
                          });
        steps = got.steps;
        raster_base_host = got.raster_base;
    }
};

}  // namespace snn2e

namespace snnb {
Engine* make_engine_stage2e(const snn_config& cfg) { return new snn2e::Engine2e(cfg); }
}  // namespace snnb
