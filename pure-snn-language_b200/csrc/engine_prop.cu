// engine_prop.cu - propagation microbench (SNN_MODEL_PROP) and the standalone
// push entry point snn_propagate.
//
// One step t is three kernels (two without STDP), captured 50 steps per CUDA
// graph:
//   k4_push  warp-per-(spiking neuron, 512-synapse segment) push over the
//            pre-major SoA streams int32 post[S] / f32 w[S]: 16-byte streaming
//            loads, one int32 red.add per synapse into the L2-resident
//            accumulator (exact, so order-free); LTD fused on the same
//            registers (w rewritten with 16-byte streaming stores).
//   k4_push_b (bucketed form, chosen at higher rates) CTA per (post bucket,
//            part of the spikers): shared-memory accumulation of the CTA's
//            row segments, stored to its row of per-part sums
//   k4_lif   thread per neuron: LIF on the accumulator (zeroing it) or on the
//            sum of the per-part rows of the bucketed push, raster
//            word by ballot, list of LIF spikes (STDP), and the forced spikes
//            of step t+1 with their Tsodyks-Markram release (warp-aggregated
//            appends to the double-buffered pre-spike list; step t+1's push
//            commits the spike time and STP state).
//   k4_ltp   warp per LIF spike: LTP over its incoming synapses through the
//            reverse CSR (synapse ids), reading the pre's last spike before t.
// The step index lives in device memory (t_base + the step's offset in the
// graph), advanced by a one-thread kernel at the end of each launch.
#include <algorithm>
#include <mutex>
#include "ckpt.h"
#include "common.h"
#include "snn_prop_rules.h"

namespace {

constexpr int P_THREADS = 256;
constexpr int P_UNROLL = 4;                 // 16-byte vectors per lane per segment
constexpr int P_SEG4 = 32 * P_UNROLL;       // vectors per segment (512 synapses)
constexpr float Q_SCALE_INV = 5.9604644775390625e-8f;  // 2^-24

struct PCtrl {
    int t_base;
    int learn;
    float lr;                 // dopamine * w_max
    int pad0;
    unsigned n_pre[2];        // forced spikes of steps with parity 0 / 1
    unsigned n_post;          // LIF spikes of the current step (STDP list)
    unsigned pad1;
    unsigned long long events, pre_spikes, post_spikes, ltp_visits;
    long long raster_base;
};

struct PDev {
    int N, F, n_exc, words, raster_cap;
    uint32_t thr;
    uint64_t key;
    float w_max;
    const int32_t* post;
    float* w;
    const uint32_t* in_ptr;
    const uint32_t* rev;
    int32_t* acc;
    float *V, *I, *u, *R;
    int8_t* ref;
    int32_t *last_post, *tA, *tB;  // last / previous forced spike (committed by k4_push)
    int32_t* pre_list;        // [2][N]
    float *rel_list, *un_list, *rn_list;  // [2][N]: release and the STP state after it
    int32_t* post_list;       // [N]
    uint32_t* raster;
    const float* exp_tab;
    PCtrl* ctrl;
    const uint16_t* boff;     // [N][nb + 1] start of each post bucket in the (sorted) row
    int nb, bw, parts;        // nb buckets of bw posts; CTAs per bucket in k4_push_b
    int32_t* part;            // [parts][N] sums of the bucketed push, one writer per slot
    int lif_parts;            // > 0: k4_lif sums part[0 .. lif_parts) instead of acc
    // post range of this rank: buckets [b0, b0 + nb_loc), neurons [lo, hi)
    // (one GPU: the whole network); `sharded` counts events per local segment
    int b0, nb_loc, lo, hi, sharded;
    int ltp_chunks;           // LTP work items per spiking post (LTP_CHUNK incoming synapses each)
};

__device__ __forceinline__ float e20(const PDev& D, int dt) {
    return dt <= SNN_PROP_EXP_STEPS ? __ldg(D.exp_tab + dt) : 0.0f;
}

// LTD of one excitatory out-synapse whose post last spiked at lp (strictly
// before t; lp < 0: never)
__device__ __forceinline__ float ltd_lp(const PDev& D, float w, int lp, int t, float lr) {
    if (lp < 0) return w;
    const float dw = pm_mul(-0.05f, e20(D, t - lp));
    return pm_min(pm_max(pm_fma(lr, dw, w), 0.0f), D.w_max);
}
// the same, onto post q
__device__ __forceinline__ float ltd(const PDev& D, float w, int q, int t, float lr) {
    return ltd_lp(D, w, __ldcg(D.last_post + q), t, lr);
}

// the same, from the post's age t - lp kept in 16 bits by the bucketed push
// (SNN_PROP_AGE_NONE: never spiked, or older than the table, where
// exp(-dt/20) is 0 and the weight, which lies in [0, w_max], stays as it is)
constexpr unsigned SNN_PROP_AGE_NONE = 0xFFFFu;
__device__ __forceinline__ float ltd_age(const PDev& D, float w, unsigned age, float lr) {
    if (age > SNN_PROP_EXP_STEPS) return w;  // loaded weights are checked to lie in [0, w_max]
    const float dw = pm_mul(-0.05f, __ldg(D.exp_tab + age));
    return pm_min(pm_max(pm_fma(lr, dw, w), 0.0f), D.w_max);
}

// warp-aggregated append of flagged lanes to list[] (count at *cnt)
__device__ __forceinline__ unsigned warp_append(bool flag, unsigned* cnt, int lane) {
    const unsigned m = __ballot_sync(0xffffffffu, flag);
    unsigned base = 0;
    if (lane == 0 && m) base = atomicAdd(cnt, (unsigned)__popc(m));
    base = __shfl_sync(0xffffffffu, base, 0);
    return base + __popc(m & ((1u << lane) - 1u));
}

// CTA-aggregated append (P_THREADS threads, every one calls it): one
// atomicAdd per CTA instead of one per warp, so that the counter's address
// takes a few thousand additions per step rather than tens of thousands.  The
// order of the entries is irrelevant to their consumers (int32 sums, and
// per-entry updates of distinct neurons).
__device__ __forceinline__ unsigned block_append(bool flag, unsigned* cnt, unsigned* s_cnt) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int NW = P_THREADS / 32;
    const unsigned m = __ballot_sync(0xffffffffu, flag);
    if (lane == 0) s_cnt[warp] = (unsigned)__popc(m);
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned tot = 0;
        for (int w = 0; w < NW; ++w) {
            const unsigned c = s_cnt[w];
            s_cnt[w] = tot;
            tot += c;
        }
        s_cnt[NW] = tot ? atomicAdd(cnt, tot) : 0u;
    }
    __syncthreads();
    const unsigned pos = s_cnt[NW] + s_cnt[warp] + (unsigned)__popc(m & ((1u << lane) - 1u));
    __syncthreads();  // s_cnt is free again
    return pos;
}

// forced spike of neuron j at step tn, appended to the pre-spike list of
// parity tn & 1 with its STP release and the STP state after it; the state
// and the spike time are committed by step tn's push, so that the exported
// state always belongs to the last executed step.  Every thread of the CTA
// calls it.
template <bool STDP, bool STP>
__device__ __forceinline__ void select_spike(const PDev& D, int tn, int j, unsigned* s_cnt) {
    bool ps = false;
    float rel = 1.0f, uu = 0.0f, rr = 0.0f;
    if (j < D.N) {
        ps = snn_prop_spikes(D.key, tn, (uint32_t)j, D.thr);
        if (ps && STP) {
            const int a = D.tA[j];
            uu = D.u[j];
            rr = D.R[j];
            rel = snn_prop_stp(&uu, &rr, a >= 0 ? tn - a : -1);
        }
    }
    const unsigned pos = block_append(ps, &D.ctrl->n_pre[tn & 1], s_cnt);
    if (ps) {
        const size_t x = (size_t)(tn & 1) * D.N + pos;
        D.pre_list[x] = j;
        if (STP) {
            D.rel_list[x] = rel;
            D.un_list[x] = uu;
            D.rn_list[x] = rr;
        }
    }
}

// step t's commit of spiker e (one writer: lane 0 of its first segment)
template <bool STDP, bool STP>
__device__ __forceinline__ void commit_spike(const PDev& D, int i, size_t x, int t) {
    if (STDP) D.tB[i] = D.tA[i];
    if (STDP || STP) D.tA[i] = t;
    if (STP) {
        D.u[i] = D.un_list[x];
        D.R[i] = D.rn_list[x];
    }
}

template <bool STDP, bool STP>
__global__ void __launch_bounds__(P_THREADS) k4_select0(PDev D) {
    __shared__ unsigned s_cnt[P_THREADS / 32 + 1];
    const int j = blockIdx.x * P_THREADS + threadIdx.x;
    select_spike<STDP, STP>(D, D.ctrl->t_base, j, s_cnt);
}

template <bool STDP, bool STP>
__global__ void __launch_bounds__(P_THREADS) k4_push(PDev D, int k) {
    PCtrl* C = D.ctrl;
    const int t = C->t_base + k;
    const int par = t & 1;
    const unsigned n = C->n_pre[par];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        C->n_pre[par ^ 1] = 0;
        C->n_post = 0;
        C->events += (unsigned long long)n * (unsigned)D.F;
        C->pre_spikes += n;
    }
    const int lane = threadIdx.x & 31;
    const long long gw = ((long long)blockIdx.x * P_THREADS + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * P_THREADS) >> 5;
    const int F4 = D.F >> 2;
    const int nseg = (F4 + P_SEG4 - 1) / P_SEG4;
    const long long items = (long long)n * nseg;
    const int32_t* list = D.pre_list + (size_t)par * D.N;
    const float* rl = D.rel_list + (size_t)par * D.N;
    const bool learn = STDP && C->learn;
    const float lr = C->lr;
    for (long long it = gw; it < items; it += nw) {
        const long long e = it / nseg;
        const int c0 = (int)(it - e * nseg) * P_SEG4 + lane;
        const int i = list[e];
        const float rel = STP ? rl[e] : 1.0f;
        if ((STDP || STP) && c0 == 0) commit_spike<STDP, STP>(D, i, (size_t)par * D.N + e, t);
        const int4* p4 = reinterpret_cast<const int4*>(D.post) + (long long)i * F4;
        float4* w4 = reinterpret_cast<float4*>(D.w) + (long long)i * F4;
        int4 pv[P_UNROLL];
        float4 wv[P_UNROLL];
#pragma unroll
        for (int u = 0; u < P_UNROLL; ++u) {
            const int c = c0 + u * 32;
            if (c < F4) {
                pv[u] = __ldcs(p4 + c);
                wv[u] = __ldcs(w4 + c);
            }
        }
        const bool plastic = learn && i < D.n_exc;
#pragma unroll
        for (int u = 0; u < P_UNROLL; ++u) {
            const int c = c0 + u * 32;
            if (c < F4) {
                atomicAdd(D.acc + pv[u].x, snn_prop_quant(wv[u].x, rel, STP));
                atomicAdd(D.acc + pv[u].y, snn_prop_quant(wv[u].y, rel, STP));
                atomicAdd(D.acc + pv[u].z, snn_prop_quant(wv[u].z, rel, STP));
                atomicAdd(D.acc + pv[u].w, snn_prop_quant(wv[u].w, rel, STP));
                if (plastic) {
                    float4 nv;
                    nv.x = ltd(D, wv[u].x, pv[u].x, t, lr);
                    nv.y = ltd(D, wv[u].y, pv[u].y, t, lr);
                    nv.z = ltd(D, wv[u].z, pv[u].z, t, lr);
                    nv.w = ltd(D, wv[u].w, pv[u].w, t, lr);
                    __stcs(w4 + c, nv);
                }
            }
        }
    }
}

// scalar form for fan-outs that are not a multiple of 4
template <bool STDP, bool STP>
__global__ void __launch_bounds__(P_THREADS) k4_push_scalar(PDev D, int k) {
    PCtrl* C = D.ctrl;
    const int t = C->t_base + k;
    const int par = t & 1;
    const unsigned n = C->n_pre[par];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        C->n_pre[par ^ 1] = 0;
        C->n_post = 0;
        C->events += (unsigned long long)n * (unsigned)D.F;
        C->pre_spikes += n;
    }
    const int lane = threadIdx.x & 31;
    const long long gw = ((long long)blockIdx.x * P_THREADS + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * P_THREADS) >> 5;
    const int nseg = (D.F + P_SEG4 - 1) / P_SEG4;
    const long long items = (long long)n * nseg;
    const int32_t* list = D.pre_list + (size_t)par * D.N;
    const float* rl = D.rel_list + (size_t)par * D.N;
    const bool learn = STDP && C->learn;
    const float lr = C->lr;
    for (long long it = gw; it < items; it += nw) {
        const long long e = it / nseg;
        const int c0 = (int)(it - e * nseg) * P_SEG4 + lane;
        const int i = list[e];
        const float rel = STP ? rl[e] : 1.0f;
        if ((STDP || STP) && c0 == 0) commit_spike<STDP, STP>(D, i, (size_t)par * D.N + e, t);
        const bool plastic = learn && i < D.n_exc;
        const long long b = (long long)i * D.F;
        for (int c = c0; c < D.F && c < c0 + P_SEG4; c += 32) {
            const int q = __ldcs(D.post + b + c);
            const float wv = __ldcs(D.w + b + c);
            atomicAdd(D.acc + q, snn_prop_quant(wv, rel, STP));
            if (plastic) __stcs(D.w + b + c, ltd(D, wv, q, t, lr));
        }
    }
}

// Bucketed push: CTA (b, p) owns the posts [b bw, (b + 1) bw)
// and spikers [n p / parts, n (p + 1) / parts).  Each row's synapses are
// stored grouped by post bucket (boff gives the segment of bucket b), so the
// CTA reads only its segments and accumulates them with shared-memory
// atomics; at the end it stores its slots to its own row of part[parts][N]
// (coalesced plain stores: every slot has one writer), which k4_lif sums.  A group of
// B_G lanes streams B_SP spikers' segments at once, B_U loads deep each, so
// that a segment (fan-out / buckets synapses on average, ~48 at 1M x 1,000
// in 21 buckets) is usually read in one round trip; the spiker ids and
// segment bounds of the group's next spikers are fetched while these stream.
// Measured at 1M x 1,000 (10 % forced rate): B_G 8, B_U 8, B_SP 1 streams the
// push in 194 us, against 269 us for 16 x 4 x 1 and 434 us for 8 x 4 x 2.
#ifndef SNN_B_THREADS
#define SNN_B_THREADS 1024
#endif
#ifndef SNN_B_SP
#define SNN_B_SP 1
#endif
#ifndef SNN_B_WMAX
#define SNN_B_WMAX 58112  // widest bucket (int32 slots of shared memory per CTA)
#endif
#ifndef SNN_B_G
#define SNN_B_G 8
#endif
#ifndef SNN_B_U
#define SNN_B_U 8
#endif
constexpr int B_THREADS = SNN_B_THREADS;
constexpr int B_G = SNN_B_G;
constexpr int B_U = SNN_B_U;
constexpr int B_SP = SNN_B_SP;

template <bool STDP, bool STP>
__device__ __forceinline__ void push_b_chunk(const PDev& D, int j0, int o1, long long base, int lo_post,
                                             int* acc_s, const uint16_t* age_s, float rel, bool plastic, int t,
                                             float lr) {
    int q[B_U];
    float wv[B_U];
#pragma unroll
    for (int u = 0; u < B_U; ++u) {
        const int j = j0 + u * B_G;
        if (j < o1) {
            q[u] = D.post[base + j];
            wv[u] = D.w[base + j];
        }
    }
#pragma unroll
    for (int u = 0; u < B_U; ++u) {
        const int j = j0 + u * B_G;
        if (j < o1) {
            atomicAdd(acc_s + (q[u] - lo_post), snn_prop_quant(wv[u], rel, STP));
            if (plastic) D.w[base + j] = ltd_age(D, wv[u], age_s[q[u] - lo_post], lr);
        }
    }
}

template <bool STDP, bool STP>
__global__ void __launch_bounds__(B_THREADS) k4_push_b(PDev D, int k) {
    extern __shared__ int acc_s[];
    PCtrl* C = D.ctrl;
    const int t = C->t_base + k;
    const int par = t & 1;
    const unsigned n = C->n_pre[par];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        C->n_pre[par ^ 1] = 0;
        C->n_post = 0;
        if (!D.sharded) C->events += (unsigned long long)n * (unsigned)D.F;
        C->pre_spikes += n;
    }
    const int b = D.b0 + blockIdx.x % D.nb_loc, p = blockIdx.x / D.nb_loc;
    const int lo_post = b * D.bw;
    const int width = min(D.bw, D.N - lo_post);
    // with STDP the age of each post's last spike (16 bits) follows the
    // slots in shared memory, so that the fused LTD reads it there and a slot
    // costs 6 bytes (wider buckets, longer row segments)
    uint16_t* const age_s = reinterpret_cast<uint16_t*>(acc_s + D.bw);
    const bool learn_s = STDP && C->learn;
    for (int x = threadIdx.x; x < width; x += B_THREADS) {
        acc_s[x] = 0;
        if (learn_s) {
            const int lp = __ldcg(D.last_post + lo_post + x);
            age_s[x] = (lp < 0 || t - lp > SNN_PROP_EXP_STEPS) ? (uint16_t)SNN_PROP_AGE_NONE : (uint16_t)(t - lp);
        }
    }
    __syncthreads();
    const long long e_lo = (long long)n * p / D.parts, e_hi = (long long)n * (p + 1) / D.parts;
    const int gl = threadIdx.x & (B_G - 1);
    const int slot = threadIdx.x / B_G;
    const int nslots = B_THREADS / B_G;
    const bool learn = STDP && C->learn;
    const float lr = C->lr;
    const int32_t* list = D.pre_list + (size_t)par * D.N;
    const float* rl = D.rel_list + (size_t)par * D.N;
    const int nb1 = D.nb + 1;
    int i_n[B_SP], o0_n[B_SP], o1_n[B_SP];
    unsigned n_ev = 0;  // events of this group's segments (sharded runs count them)
    long long e = e_lo + slot;
#pragma unroll
    for (int sp = 0; sp < B_SP; ++sp) {
        const long long es = e + (long long)sp * nslots;
        i_n[sp] = 0;
        o0_n[sp] = o1_n[sp] = 0;
        if (es < e_hi) {
            i_n[sp] = list[es];
            o0_n[sp] = D.boff[(size_t)i_n[sp] * nb1 + b];
            o1_n[sp] = D.boff[(size_t)i_n[sp] * nb1 + b + 1];
        }
    }
    for (; e < e_hi; e += (long long)nslots * B_SP) {
        int i[B_SP], o0[B_SP], o1[B_SP];
#pragma unroll
        for (int sp = 0; sp < B_SP; ++sp) {
            i[sp] = i_n[sp];
            o0[sp] = o0_n[sp];
            o1[sp] = o1_n[sp];
            const long long en = e + (long long)nslots * (B_SP + sp);
            if (en < e_hi) {
                i_n[sp] = list[en];
                o0_n[sp] = D.boff[(size_t)i_n[sp] * nb1 + b];
                o1_n[sp] = D.boff[(size_t)i_n[sp] * nb1 + b + 1];
            }
        }
        float rel[B_SP];
        bool plastic[B_SP];
        long long base[B_SP];
#pragma unroll
        for (int sp = 0; sp < B_SP; ++sp) {
            const long long es = e + (long long)sp * nslots;
            const bool valid = es < e_hi;
            rel[sp] = STP && valid ? rl[es] : 1.0f;
            if ((STDP || STP) && valid && b == D.b0 && gl == 0)
                commit_spike<STDP, STP>(D, i[sp], (size_t)par * D.N + es, t);
            base[sp] = (long long)i[sp] * D.F;
            plastic[sp] = learn && i[sp] < D.n_exc;
            if (!valid) o1[sp] = o0[sp];  // empty segment
            if (gl == 0) n_ev += (unsigned)(o1[sp] - o0[sp]);
        }
        // first B_G * B_U synapses of every segment, all loads in flight together
        int q[B_SP][B_U];
        float wv[B_SP][B_U];
#pragma unroll
        for (int sp = 0; sp < B_SP; ++sp)
#pragma unroll
            for (int u = 0; u < B_U; ++u) {
                const int j = o0[sp] + gl + u * B_G;
                if (j < o1[sp]) {
                    q[sp][u] = D.post[base[sp] + j];
                    wv[sp][u] = D.w[base[sp] + j];
                }
            }
#pragma unroll
        for (int sp = 0; sp < B_SP; ++sp)
#pragma unroll
            for (int u = 0; u < B_U; ++u) {
                const int j = o0[sp] + gl + u * B_G;
                if (j < o1[sp]) {
                    atomicAdd(acc_s + (q[sp][u] - lo_post), snn_prop_quant(wv[sp][u], rel[sp], STP));
                    if (plastic[sp]) D.w[base[sp] + j] = ltd_age(D, wv[sp][u], age_s[q[sp][u] - lo_post], lr);
                }
            }
        // rare long segments
#pragma unroll
        for (int sp = 0; sp < B_SP; ++sp)
            for (int j0 = o0[sp] + B_G * B_U + gl; j0 < o1[sp]; j0 += B_G * B_U)
                push_b_chunk<STDP, STP>(D, j0, o1[sp], base[sp], lo_post, acc_s, age_s, rel[sp], plastic[sp], t,
                                        lr);
    }
    if (D.sharded) {  // events = the rank's segments of the spikers' rows
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) n_ev += __shfl_xor_sync(0xffffffffu, n_ev, o);
        if ((threadIdx.x & 31) == 0 && n_ev) atomicAdd(&C->events, (unsigned long long)n_ev);
    }
    __syncthreads();
    int32_t* out = D.part + (size_t)p * D.N + lo_post;
    for (int x = threadIdx.x; x < width; x += B_THREADS) out[x] = acc_s[x];
}

template <bool STDP, bool STP>
__global__ void __launch_bounds__(P_THREADS) k4_lif(PDev D, int k) {
    PCtrl* C = D.ctrl;
    const int t = C->t_base + k;
    const int j = blockIdx.x * P_THREADS + threadIdx.x;
    const int lane = threadIdx.x & 31;
    bool sp = false;
    if (j >= D.lo && j < D.hi) {  // this rank's posts (one GPU: all)
        // this step's input: the accumulator of the direct push (consumed
        // and cleared), or the per-part sums of the bucketed push (int32
        // addition: the same value in any order)
        int a = 0;
        if (D.lif_parts == 0) {
            a = __ldcg(D.acc + j);
            D.acc[j] = 0;
        } else {
            for (int q = 0; q < D.lif_parts; ++q) a += __ldcg(D.part + (size_t)q * D.N + j);
        }
        const float in = pm_mul(pm_i2f(a), Q_SCALE_INV);
        const int r = D.ref[j];
        float v = D.V[j];
        if (r > 0) {
            D.ref[j] = (int8_t)(r - 1);
            D.V[j] = pm_mul(v, 0.95f);
        } else {
            const float cur = pm_fma(D.I[j], 0.95f, in);
            D.I[j] = cur;
            v = pm_fma(v, 0.95f, cur);
            if (v < 0.0f) v = 0.0f;
            sp = v >= 1.0f;
            if (sp) {
                v = 0.0f;
                D.ref[j] = 2;
                D.last_post[j] = t;
            }
            D.V[j] = v;
        }
    }
    const unsigned m = __ballot_sync(0xffffffffu, sp);
    if (lane == 0 && (j >> 5) < D.words) {
        const long long row = ((long long)t - C->raster_base) % D.raster_cap;
        D.raster[row * D.words + (j >> 5)] = m;
    }
    __shared__ unsigned blk_spikes;
    if (threadIdx.x == 0) blk_spikes = 0;
    __syncthreads();
    if (lane == 0 && m) atomicAdd(&blk_spikes, (unsigned)__popc(m));
    __shared__ unsigned s_cnt[P_THREADS / 32 + 1];
    if (STDP) {
        const unsigned pos = block_append(sp, &C->n_post, s_cnt);
        if (sp) D.post_list[pos] = j;
    }
    select_spike<STDP, STP>(D, t + 1, j, s_cnt);
    __syncthreads();
    if (threadIdx.x == 0 && blk_spikes) atomicAdd(&C->post_spikes, (unsigned long long)blk_spikes);
}

// latest forced spike of p strictly before t (step t's push has committed
// spikes up to t)
__device__ __forceinline__ int pre_before(const PDev& D, int p, int t) {
    const int a = __ldcg(D.tA + p);
    return a < t ? a : __ldcg(D.tB + p);
}

// LTP of the excitatory incoming synapses of every LIF spike: one warp per
// (spiking post, chunk of LTP_CHUNK incoming synapses), so that a few
// thousand spiking posts still give enough warps to cover the latency of
// the scattered weight updates (every synapse is updated once)
constexpr uint32_t LTP_CHUNK = 256;
__global__ void __launch_bounds__(P_THREADS) k4_ltp(PDev D, int k) {
    PCtrl* C = D.ctrl;
    if (!C->learn) return;
    const int t = C->t_base + k;
    const unsigned n = C->n_post;
    const float lr = C->lr;
    const int lane = threadIdx.x & 31;
    const long long gw = ((long long)blockIdx.x * P_THREADS + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * P_THREADS) >> 5;
    const uint32_t F = (uint32_t)D.F;
    const int CH = D.ltp_chunks;
    for (long long v = gw; v < (long long)n * CH; v += nw) {
        const long long e = v / CH;
        const uint32_t c = (uint32_t)(v - e * CH);
        const int j = D.post_list[e];
        const uint32_t rb = D.in_ptr[j], re = D.in_ptr[j + 1];
        const uint32_t b = rb + c * LTP_CHUNK;
        if (b >= re) continue;
        const uint32_t en = min(re, b + LTP_CHUNK);
        if (lane == 0) atomicAdd(&C->ltp_visits, (unsigned long long)(en - b));
        for (uint32_t x0 = b; x0 < en; x0 += 32 * P_UNROLL) {
            uint32_t s[P_UNROLL];
            int tp[P_UNROLL];
#pragma unroll
            for (int u = 0; u < P_UNROLL; ++u) {
                const uint32_t x = x0 + u * 32 + lane;
                s[u] = x < en ? __ldcs(D.rev + x) : 0xffffffffu;
                tp[u] = -1;
                if (s[u] != 0xffffffffu) {
                    const int p = (int)(s[u] / F);
                    if (p < D.n_exc) tp[u] = pre_before(D, p, t);
                }
            }
            // all weight loads before any store: the synapses of one post's
            // list are distinct, so the loads cannot see these stores, and
            // the P_UNROLL random reads overlap instead of queueing behind
            // each store
            float wv[P_UNROLL];
#pragma unroll
            for (int u = 0; u < P_UNROLL; ++u) wv[u] = tp[u] >= 0 ? __ldcg(D.w + s[u]) : 0.0f;
#pragma unroll
            for (int u = 0; u < P_UNROLL; ++u) {
                if (tp[u] >= 0) {
                    const float dw = pm_mul(0.05f, e20(D, t - tp[u]));
                    D.w[s[u]] = pm_min(pm_max(pm_fma(lr, dw, wv[u]), 0.0f), D.w_max);
                }
            }
        }
    }
}

__global__ void k4_advance(PCtrl* C, int n) { C->t_base += n; }

// ---- build kernels ---------------------------------------------------------
__global__ void k4_generate(int32_t* post, float* w, long long S, int N, int F, int n_exc,
                            uint32_t seed, float w_max) {
    for (long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x; s < S;
         s += (long long)gridDim.x * blockDim.x) {
        const uint64_t h = snn_prop_syn_hash(seed, (uint64_t)s);
        post[s] = snn_prop_post(h, (uint32_t)N);
        w[s] = snn_prop_weight(h, w_max, (s / F) < n_exc);
    }
}

// Row i's synapses grouped by post bucket (post / bw), stable in k:
// one warp per row; writes the sorted post / w and the bucket starts.  With
// `unpermute` set it instead scatters a sorted per-synapse array back to the
// generation order (s = i * F + k): out[i F + k] = in[i F + pos(k)].
__global__ void __launch_bounds__(256) k4_sort_rows(int32_t* post, float* w, uint16_t* boff, int N, int F,
                                                    int n_exc, uint32_t seed, float w_max, int nb,
                                                    int bw, const uint32_t* in, uint32_t* out) {
    extern __shared__ int sm[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    int* cnt = sm + wib * 2 * (nb + 1);
    int* basep = cnt + (nb + 1);
    const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long i = gw; i < N; i += nw) {
        const long long row = i * F;
        for (int x = lane; x <= nb; x += 32) cnt[x] = 0;
        __syncwarp();
        for (int kk = lane; kk < F; kk += 32) {
            const int q = snn_prop_post(snn_prop_syn_hash(seed, (uint64_t)(row + kk)), (uint32_t)N);
            atomicAdd(cnt + q / bw, 1);
        }
        __syncwarp();
        if (lane == 0) {
            int run = 0;
            for (int x = 0; x <= nb; ++x) {
                basep[x] = run;
                if (!in) boff[(size_t)i * (nb + 1) + x] = (uint16_t)run;
                run += cnt[x];
            }
        }
        __syncwarp();
        for (int k0 = 0; k0 < F; k0 += 32) {
            const int kk = k0 + lane;
            const bool valid = kk < F;
            int q = 0, bk = -1;
            uint64_t h = 0;
            if (valid) {
                h = snn_prop_syn_hash(seed, (uint64_t)(row + kk));
                q = snn_prop_post(h, (uint32_t)N);
                bk = q / bw;
            }
            const unsigned peers = __match_any_sync(0xffffffffu, bk);
            const int rank = __popc(peers & ((1u << lane) - 1u));
            const int pos = valid ? basep[bk] + rank : 0;
            __syncwarp();
            if (valid && rank == 0) basep[bk] += __popc(peers);
            __syncwarp();
            if (valid) {
                if (in) {
                    out[row + kk] = in[row + pos];
                } else {
                    post[row + pos] = q;
                    w[row + pos] = snn_prop_weight(h, w_max, i < n_exc);
                }
            }
        }
        __syncwarp();
    }
}

__global__ void k4_indegree(const int32_t* post, long long S, uint32_t* deg) {
    for (long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x; s < S;
         s += (long long)gridDim.x * blockDim.x)
        atomicAdd(deg + post[s], 1u);
}

// exclusive scan of deg[0..N) into ptr[0..N] by one block of 1024 threads
__global__ void __launch_bounds__(1024) k4_scan(const uint32_t* deg, uint32_t* ptr, int N) {
    __shared__ unsigned long long part[1024];
    const int tid = threadIdx.x;
    const long long lo = (long long)N * tid / 1024, hi = (long long)N * (tid + 1) / 1024;
    unsigned long long s = 0;
    for (long long j = lo; j < hi; ++j) s += deg[j];
    part[tid] = s;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
        unsigned long long v = tid >= off ? part[tid - off] : 0;
        __syncthreads();
        part[tid] += v;
        __syncthreads();
    }
    unsigned long long run = part[tid] - s;
    for (long long j = lo; j < hi; ++j) {
        ptr[j] = (uint32_t)run;
        run += deg[j];
    }
    if (tid == 1023) ptr[N] = (uint32_t)part[1023];
}

__global__ void k4_fill_rev(const int32_t* post, long long S, uint32_t* cursor, uint32_t* rev) {
    for (long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x; s < S;
         s += (long long)gridDim.x * blockDim.x)
        rev[atomicAdd(cursor + post[s], 1u)] = (uint32_t)s;
}

__global__ void k4_exp_table(float* tab) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k <= SNN_PROP_EXP_STEPS) tab[k] = snn_expf(pm_div(-pm_i2f(k), 20.0f));
}

__global__ void k4_max(const uint32_t* v, int n, uint32_t* out) {
    uint32_t m = 0;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x)
        m = max(m, v[j]);
    for (int o = 16; o; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0 && m) atomicMax(out, m);
}

// ---- host engine -----------------------------------------------------------
struct EngineProp : snnb::Engine {
    snn_config cfg;
    cudaStream_t stream = nullptr;
    PDev D{};
    int mode = 0;
    bool stdp = false, stp = false, built = false, vec = false, sorted = false, bucketed = false;
    size_t push_smem = 0;
    long long S = 0, steps = 0, raster_base_host = 0;
    int raster_cap = 1024;
    int push_grid = 1, lif_grid = 1, ltp_grid = 1;
    uint32_t max_in = 0, spec_seed = 0;
    float dopamine = 1.0f;
    int rank = 0, world = 1;  // post-bucket shards (snn_set_shard)
    snnb::DevBuf<int32_t> post, acc, last_post, tA, tB, pre_list, post_list, part;
    snnb::DevBuf<float> w, V, I, u, R, rel_list, un_list, rn_list, exp_tab;
    snnb::DevBuf<int8_t> ref;
    snnb::DevBuf<uint32_t> in_ptr, rev, raster, tmp;
    snnb::DevBuf<uint16_t> boff;
    snnb::DevBuf<PCtrl> ctrl;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    int graph_steps = 0;
    bool profiling = false;
    std::vector<cudaEvent_t> pev;
    snn_profile prof{};

    explicit EngineProp(const snn_config& c) : cfg(c) {
        mode = c.prop_mode;
        SNN_REQUIRE(mode >= 0 && mode <= 3, SNN_ERR_ARG, "prop_mode must combine SNN_PROP_STDP / SNN_PROP_STP");
        SNN_REQUIRE(c.prop_rate >= 0.0f && c.prop_rate <= 1.0f, SNN_ERR_ARG, "prop_rate must lie in [0, 1]");
        stdp = mode & SNN_PROP_STDP;
        stp = mode & SNN_PROP_STP;
        if (c.raster_steps > 0) raster_cap = c.raster_steps;
        SNN_CUDA(cudaSetDevice(c.device));
        SNN_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    }
    ~EngineProp() override {
        for (auto e : pev) cudaEventDestroy(e);
        drop_graph();
        if (stream) {
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
        }
    }

    void drop_graph() {
        if (graph_exec) cudaGraphExecDestroy(graph_exec);
        if (graph) cudaGraphDestroy(graph);
        graph_exec = nullptr;
        graph = nullptr;
        graph_steps = 0;
    }

    int nkern() const { return stdp ? 3 : 2; }

    // Sharding over `w` GPUs by post bucket: rank r owns the buckets
    // [nb r / w, nb (r + 1) / w) (nb a multiple of w) and their neurons.  The
    // forced pre-spikes are a seeded hash of (step, neuron), so every rank
    // draws all of them and pushes the segments of their rows that fall in
    // its buckets; LIF, LTD (the post's last spike) and LTP (the incoming
    // synapses of a local post spike) only touch local posts, so no data
    // crosses GPUs during the run.  No NCCL communicator is needed.
    void set_shard(int32_t r, int32_t w, const void*) override {
        SNN_REQUIRE(!built, SNN_ERR_STATE, "shard before building the network");
        SNN_REQUIRE(w >= 1 && r >= 0 && r < w, SNN_ERR_ARG, "bad rank / world size");
        rank = r;
        world = w;
    }

    void build(const snn_topology_spec& spec) override {
        SNN_REQUIRE(!built, SNN_ERR_STATE, "network already built");
        SNN_CUDA(cudaSetDevice(cfg.device));
        const int N = spec.l4, F = spec.deg_intra;
        SNN_REQUIRE(N >= 1 && F >= 1, SNN_ERR_ARG, "need l4 >= 1 neurons and deg_intra >= 1 out-edges");
        spec_seed = spec.seed;
        S = (long long)N * F;
        SNN_REQUIRE(S < (1ll << 32) - 1, SNN_ERR_ARG, "N * fan-out must stay below 2^32 - 1");
        D.N = N;
        D.F = F;
        D.n_exc = (int)(((long long)N * 4) / 5);
        D.words = (N + 31) / 32;
        D.raster_cap = raster_cap;
        const double th = (double)cfg.prop_rate * 4294967296.0;
        D.thr = th >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)th;
        D.key = snn_prop_spike_key(spec.seed);
        D.w_max = cfg.prop_w_max > 0.0f ? cfg.prop_w_max
                  : (cfg.prop_rate > 0.0f ? pm_div(0.01f, pm_mul(cfg.prop_rate, (float)F)) : 1.0f);
        SNN_REQUIRE(D.w_max <= 1.0f, SNN_ERR_ARG, "prop_w_max must be <= 1");
        vec = (F % 4) == 0;
        // rows grouped by post bucket of bw posts (bw int32 slots of shared
        // memory per CTA of k4_push_b): among the bucket counts whose buckets
        // fit (bw <= SNN_B_WMAX and the opt-in shared memory), the fewest
        // (widest buckets, longest row segments) whose nb x parts CTAs fill
        // the SMs in whole waves within 1 % of the best fill
        int dev_sms = 0, smem_optin = 0;
        SNN_CUDA(cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, cfg.device));
        SNN_CUDA(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, cfg.device));
        const int slot_bytes = stdp ? 6 : 4;  // int32 sum (+ the post's 16-bit spike age with STDP)
        const int bw_cap = std::max(1024, std::min(SNN_B_WMAX, smem_optin / slot_bytes));
        const int nb_min = (int)(((long long)N + bw_cap - 1) / bw_cap);
        sorted = nb_min <= 256 && F <= 65535;
        SNN_REQUIRE(cfg.prop_push >= 0 && cfg.prop_push <= 2, SNN_ERR_ARG, "prop_push must be 0, 1 or 2");
        SNN_REQUIRE(cfg.prop_push != 2 || sorted, SNN_ERR_ARG,
                    "bucketed push needs at most 256 post buckets and fan-out <= 65535");
        SNN_REQUIRE(world == 1 || (sorted && cfg.prop_push != 1), SNN_ERR_ARG,
                    "a sharded microbench needs the bucketed push (at most 256 post buckets, "
                    "fan-out <= 65535, prop_push 0 or 2)");
        SNN_REQUIRE(world == 1 || (long long)N >= 2ll * world, SNN_ERR_ARG,
                    "a sharded microbench needs at least two neurons per rank");
        D.nb = nb_min;
        D.bw = (int)(((long long)N + nb_min - 1) / nb_min);
        D.parts = 1;
        if (sorted) {
            for (auto kf : {k4_push_b<false, false>, k4_push_b<false, true>, k4_push_b<true, false>,
                            k4_push_b<true, true>})
                SNN_CUDA(cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin));
            struct Cand { int nb, bw, parts; double util; };
            std::vector<Cand> cands;
            double best = 0.0;
            // sharded: nb a multiple of the world size, each rank's nb / world
            // buckets x parts CTAs filling its SMs
            const int nb_hi = std::min(256, std::max(2 * nb_min, nb_min + 8) + (world > 1 ? 2 * world : 0));
            for (int nb = nb_min; nb <= nb_hi; ++nb) {
                if (nb % world != 0) continue;
                const int bw = (int)(((long long)N + nb - 1) / nb);
                if ((int)(((long long)N + bw - 1) / bw) != nb) continue;  // nb buckets of bw cover N
                int occ = 0;
                SNN_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, push_kernel_b(), B_THREADS,
                                                                       (size_t)slot_bytes * bw));
                if (occ < 1) continue;
                const int slots = occ * dev_sms;
                const int nb_loc = nb / world;
                const int parts = std::max(1, slots / nb_loc);
                const long long ctas = (long long)nb_loc * parts;
                const double util = (double)ctas / (double)(((ctas + slots - 1) / slots) * slots);
                cands.push_back({nb, bw, parts, util});
                best = std::max(best, util);
            }
            SNN_REQUIRE(!cands.empty(), SNN_ERR_CUDA, "no bucket width fits the bucketed push");
            for (const Cand& c : cands)
                // (with STDP within 3 %: fewer, wider buckets for longer LTD segments)
                if (c.util >= best - (stdp ? 0.03 : 0.01)) {
                    D.nb = c.nb;
                    D.bw = c.bw;
                    D.parts = c.parts;
                    break;
                }
        }
        push_smem = (size_t)slot_bytes * D.bw;
        // bucketed when a post expects at least one event per step (measured
        // at 1M x 1,000: the bucketed step is faster from 0.1 % forced rate
        // up, 1.4x at 1 %, 2.7x at 10 %; the direct push only wins, by ~1 %,
        // at 0.1 % with STDP)
        bucketed = cfg.prop_push == 2 || world > 1 ||
                   (cfg.prop_push == 0 && sorted && (double)cfg.prop_rate * F >= 1.0);
        D.sharded = world > 1;
        D.nb_loc = D.nb / world;
        D.b0 = rank * D.nb_loc;
        D.lo = D.b0 * D.bw;
        D.hi = (int)std::min<long long>(N, (long long)(D.b0 + D.nb_loc) * D.bw);
        SNN_REQUIRE(D.nb % world == 0 && D.lo < D.hi, SNN_ERR_ARG,
                    "no post-bucket layout gives every rank a share of the neurons");

        post.alloc(S);
        w.alloc(S);
        acc.alloc(N);
        V.alloc(N);
        I.alloc(N);
        ref.alloc(N);
        last_post.alloc(N);
        pre_list.alloc((size_t)2 * N);
        rel_list.alloc(stp ? (size_t)2 * N : 1);
        un_list.alloc(stp ? (size_t)2 * N : 1);
        rn_list.alloc(stp ? (size_t)2 * N : 1);
        raster.alloc((size_t)raster_cap * D.words);
        exp_tab.alloc(SNN_PROP_EXP_STEPS + 1);
        ctrl.alloc(1);
        tmp.alloc((size_t)N + 1);
        const int gen_grid = 148 * 16;
        if (sorted) {
            boff.alloc((size_t)N * (D.nb + 1));
            k4_sort_rows<<<gen_grid, 256, 8 * 2 * (D.nb + 1) * sizeof(int), stream>>>(
                post.p, w.p, boff.p, N, F, D.n_exc, spec.seed, D.w_max, D.nb, D.bw, nullptr, nullptr);
        } else {
            k4_generate<<<gen_grid, 256, 0, stream>>>(post.p, w.p, S, N, F, D.n_exc, spec.seed, D.w_max);
        }
        SNN_CUDA(cudaGetLastError());
        k4_exp_table<<<(SNN_PROP_EXP_STEPS + 256) / 256, 256, 0, stream>>>(exp_tab.p);
        // in-degrees: the int32 accumulator must hold max in-degree * w_max * 2^24
        tmp.zero(stream);
        k4_indegree<<<gen_grid, 256, 0, stream>>>(post.p, S, tmp.p);
        snnb::DevBuf<uint32_t> mx;
        mx.alloc(1);
        mx.zero(stream);
        k4_max<<<148, 256, 0, stream>>>(tmp.p, N, mx.p);
        SNN_CUDA(cudaMemcpyAsync(&max_in, mx.p, 4, cudaMemcpyDeviceToHost, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
        SNN_REQUIRE((double)max_in * D.w_max * 16777216.0 < 2147483647.0, SNN_ERR_ARG,
                    "max in-degree * w_max * 2^24 overflows the int32 accumulator");
        if (stdp) {
            in_ptr.alloc((size_t)N + 1);
            rev.alloc(S);
            k4_scan<<<1, 1024, 0, stream>>>(tmp.p, in_ptr.p, N);
            SNN_CUDA(cudaMemcpyAsync(tmp.p, in_ptr.p, (size_t)N * 4, cudaMemcpyDeviceToDevice, stream));
            k4_fill_rev<<<gen_grid, 256, 0, stream>>>(post.p, S, tmp.p, rev.p);
            post_list.alloc(N);
            tA.alloc(N); tB.alloc(N);
        } else if (stp) {
            tA.alloc(N);
        }
        tmp.release();
        if (stp) {
            u.alloc(N);
            R.alloc(N);
        }
        D.post = post.p; D.w = w.p; D.in_ptr = in_ptr.p; D.rev = rev.p; D.acc = acc.p;
        D.V = V.p; D.I = I.p; D.u = u.p; D.R = R.p; D.ref = ref.p; D.last_post = last_post.p;
        D.tA = tA.p; D.tB = tB.p; D.pre_list = pre_list.p; D.rel_list = rel_list.p;
        D.un_list = un_list.p; D.rn_list = rn_list.p;
        D.post_list = post_list.p; D.raster = raster.p; D.exp_tab = exp_tab.p; D.ctrl = ctrl.p;
        D.boff = boff.p;
        D.ltp_chunks = (int)((max_in + LTP_CHUNK - 1) / LTP_CHUNK);
        if (D.ltp_chunks < 1) D.ltp_chunks = 1;
        if (bucketed) {
            part.alloc((size_t)D.parts * N);
            part.zero(stream);
        }
        D.part = part.p;
        D.lif_parts = bucketed ? D.parts : 0;
        reset_state();
        int occ = 0;
        if (vec) SNN_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, push_kernel(), P_THREADS, 0));
        else SNN_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, push_kernel_scalar(), P_THREADS, 0));
        push_grid = dev_sms * std::max(occ, 1);
        lif_grid = (N + P_THREADS - 1) / P_THREADS;
        ltp_grid = dev_sms * 8;
        built = true;
    }

    void (*push_kernel())(PDev, int) {
        if (stdp) return stp ? k4_push<true, true> : k4_push<true, false>;
        return stp ? k4_push<false, true> : k4_push<false, false>;
    }
    void (*push_kernel_b())(PDev, int) {
        if (stdp) return stp ? k4_push_b<true, true> : k4_push_b<true, false>;
        return stp ? k4_push_b<false, true> : k4_push_b<false, false>;
    }
    void (*push_kernel_scalar())(PDev, int) {
        if (stdp) return stp ? k4_push_scalar<true, true> : k4_push_scalar<true, false>;
        return stp ? k4_push_scalar<false, true> : k4_push_scalar<false, false>;
    }
    void (*lif_kernel())(PDev, int) {
        if (stdp) return stp ? k4_lif<true, true> : k4_lif<true, false>;
        return stp ? k4_lif<false, true> : k4_lif<false, false>;
    }

    void reset_state() {
        const int N = D.N;
        acc.zero(stream);
        V.zero(stream);
        I.zero(stream);
        ref.zero(stream);
        SNN_CUDA(cudaMemsetAsync(last_post.p, 0xff, (size_t)N * 4, stream));  // -1: none
        if (tA.p) SNN_CUDA(cudaMemsetAsync(tA.p, 0xff, (size_t)N * 4, stream));
        if (tB.p) SNN_CUDA(cudaMemsetAsync(tB.p, 0xff, (size_t)N * 4, stream));
        if (stp) {
            std::vector<float> hu((size_t)N, SNN_PROP_STP_U), hr((size_t)N, 1.0f);
            u.upload(hu.data(), N, stream);
            R.upload(hr.data(), N, stream);
            SNN_CUDA(cudaStreamSynchronize(stream));
        }
        raster.zero(stream);
        PCtrl h{};
        h.learn = 1;
        h.lr = pm_mul(dopamine, D.w_max);
        ctrl.upload(&h, 1, stream);
        // forced spikes of step 0
        if (stdp) {
            if (stp) k4_select0<true, true><<<lif_blocks(), P_THREADS, 0, stream>>>(D);
            else k4_select0<true, false><<<lif_blocks(), P_THREADS, 0, stream>>>(D);
        } else {
            if (stp) k4_select0<false, true><<<lif_blocks(), P_THREADS, 0, stream>>>(D);
            else k4_select0<false, false><<<lif_blocks(), P_THREADS, 0, stream>>>(D);
        }
        SNN_CUDA(cudaGetLastError());
        SNN_CUDA(cudaStreamSynchronize(stream));
    }
    int lif_blocks() const { return (D.N + P_THREADS - 1) / P_THREADS; }

    void launch_step(int k, cudaEvent_t* ev, bool capturing) {
        const unsigned fl = capturing ? cudaEventRecordExternal : cudaEventRecordDefault;
        if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[0], stream, fl));
        if (bucketed) push_kernel_b()<<<D.nb_loc * D.parts, B_THREADS, push_smem, stream>>>(D, k);
        else if (vec) push_kernel()<<<push_grid, P_THREADS, 0, stream>>>(D, k);
        else push_kernel_scalar()<<<push_grid, P_THREADS, 0, stream>>>(D, k);
        if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[1], stream, fl));
        lif_kernel()<<<lif_grid, P_THREADS, 0, stream>>>(D, k);
        if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[2], stream, fl));
        if (stdp) {
            k4_ltp<<<ltp_grid, P_THREADS, 0, stream>>>(D, k);
            if (ev) SNN_CUDA(cudaEventRecordWithFlags(ev[3], stream, fl));
        }
    }

    void ensure_events(int n) {
        const size_t need = (size_t)n * (nkern() + 1);
        while (pev.size() < need) {
            cudaEvent_t e;
            SNN_CUDA(cudaEventCreate(&e));
            pev.push_back(e);
        }
    }
    cudaEvent_t* step_events(int q) { return profiling ? &pev[(size_t)q * (nkern() + 1)] : nullptr; }

    void ensure_graph(int n) {
        if (graph_exec && graph_steps == n) return;
        drop_graph();
        if (profiling) ensure_events(n);
        SNN_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
        for (int q = 0; q < n; ++q) launch_step(q, step_events(q), true);
        k4_advance<<<1, 1, 0, stream>>>(ctrl.p, n);
        SNN_CUDA(cudaStreamEndCapture(stream, &graph));
        SNN_CUDA(cudaGraphInstantiate(&graph_exec, graph, 0));
        graph_steps = n;
    }

    void harvest(int n) {
        SNN_CUDA(cudaStreamSynchronize(stream));
        const int nk = nkern();
        for (int q = 0; q < n; ++q)
            for (int kk = 0; kk < nk; ++kk) {
                float ms = 0.0f;
                cudaEvent_t* ev = step_events(q);
                SNN_CUDA(cudaEventElapsedTime(&ms, ev[kk], ev[kk + 1]));
                prof.kernel_ms[kk] += ms;
                prof.launches[kk] += 1;
                prof.step_ms += ms;
            }
        prof.steps += n;
    }

    void set_profiling(int32_t en) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_CUDA(cudaStreamSynchronize(stream));
        profiling = en != 0;
        drop_graph();
        memset(&prof, 0, sizeof(prof));
        prof.n_kernels = nkern();
        strcpy(prof.names[0], bucketed ? "k4_push_b" : vec ? "k4_push" : "k4_push_scalar");
        strcpy(prof.names[1], "k4_lif");
        if (stdp) strcpy(prof.names[2], "k4_ltp");
    }
    void get_profile(snn_profile* o) override { *o = prof; }

    void set_corpus(const uint8_t*, int64_t) override {}  // the input is the forced spikes

    void run(int32_t n_steps, int32_t byte_override, int32_t learn, uint32_t* raster_out,
             int32_t* counts_out) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_REQUIRE(n_steps >= 0, SNN_ERR_ARG, "negative step count");
        (void)byte_override;
        if (n_steps == 0) return;
        const int lr = learn ? 1 : 0;
        SNN_CUDA(cudaMemcpyAsync((char*)ctrl.p + offsetof(PCtrl, learn), &lr, 4, cudaMemcpyHostToDevice, stream));
        const long long rb = steps;
        raster_base_host = rb;
        SNN_CUDA(cudaMemcpyAsync((char*)ctrl.p + offsetof(PCtrl, raster_base), &rb, 8, cudaMemcpyHostToDevice, stream));
        const int chunk = 50;
        int done = 0;
        while (done < n_steps) {
            const int span = std::min(n_steps - done, raster_cap - (done % raster_cap));
            int q = 0;
            while (q < span) {
                const int m = span - q >= chunk ? chunk : 1;
                if (m == chunk) {
                    ensure_graph(chunk);
                    SNN_CUDA(cudaGraphLaunch(graph_exec, stream));
                } else {
                    if (profiling) ensure_events(1);
                    launch_step(0, step_events(0), false);
                    k4_advance<<<1, 1, 0, stream>>>(ctrl.p, 1);
                    SNN_CUDA(cudaGetLastError());
                }
                if (profiling) harvest(m);
                q += m;
            }
            if (raster_out || counts_out) {
                const long long row0 = done % raster_cap;
                std::vector<uint32_t> tmpr;
                uint32_t* dst = raster_out ? raster_out + (size_t)done * D.words : nullptr;
                if (!dst) {
                    tmpr.resize((size_t)span * D.words);
                    dst = tmpr.data();
                }
                SNN_CUDA(cudaMemcpyAsync(dst, raster.p + row0 * D.words, (size_t)span * D.words * 4,
                                         cudaMemcpyDeviceToHost, stream));
                SNN_CUDA(cudaStreamSynchronize(stream));
                if (counts_out)
                    for (int r = 0; r < span; ++r) {
                        int cnt = 0;
                        for (int x = 0; x < D.words; ++x) cnt += __builtin_popcount(dst[(size_t)r * D.words + x]);
                        counts_out[done + r] = cnt;
                    }
            }
            done += span;
        }
        steps += n_steps;
        SNN_CUDA(cudaGetLastError());
    }

    void sync() override { SNN_CUDA(cudaStreamSynchronize(stream)); }
    int64_t steps_done() const override { return steps; }

    void counters(snn_counters* o) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        PCtrl h;
        SNN_CUDA(cudaMemcpyAsync(&h, ctrl.p, sizeof(PCtrl), cudaMemcpyDeviceToHost, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
        memset(o, 0, sizeof(*o));
        o->step = steps;
        o->total_spikes = (int64_t)h.post_spikes;
        o->arrivals = (int64_t)h.events;
        o->dispatched = (int64_t)h.pre_spikes;
        o->ltp_visits = (int64_t)h.ltp_visits;
        o->n_neurons = D.N;
        o->n_synapses = S;
        o->local_lo = D.lo;
        o->local_hi = D.hi;
        o->last_byte = -1;
        if (steps > 0) {
            std::vector<uint32_t> row(D.words);
            get_spikes(row.data(), D.words);
            int c = 0;
            for (uint32_t x : row) c += __builtin_popcount(x);
            o->last_spikes = c;
        }
        o->modeled_bytes = (double)h.events * 8.0 + (double)h.pre_spikes * 4.0 +
                           (double)steps * D.N * 22.0;
    }

    void get_spikes(uint32_t* words, int64_t n_words) override {
        SNN_REQUIRE(built && steps > 0, SNN_ERR_STATE, "no step executed yet");
        SNN_REQUIRE(n_words >= D.words, SNN_ERR_ARG, "bitmask buffer too small");
        const long long row = (steps - 1 - raster_base_host) % raster_cap;
        SNN_CUDA(cudaMemcpyAsync(words, raster.p + row * D.words, (size_t)D.words * 4,
                                 cudaMemcpyDeviceToHost, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
    }

    void get_state(int32_t which, void* buf, int64_t nbytes) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        const int64_t N = D.N;
        auto need = [&](int64_t b) { SNN_REQUIRE(nbytes >= b, SNN_ERR_ARG, "state buffer too small"); };
        auto dl = [&](const void* src, size_t b) {
            need((int64_t)b);
            SNN_CUDA(cudaMemcpyAsync(buf, src, b, cudaMemcpyDeviceToHost, stream));
            SNN_CUDA(cudaStreamSynchronize(stream));
        };
        switch (which) {
            case SNN_STATE_V: dl(V.p, N * 4); break;
            case SNN_STATE_SYN_CURRENT: dl(I.p, N * 4); break;
            case SNN_STATE_LAST_SPIKE: dl(last_post.p, N * 4); break;
            case SNN_STATE_REFRACTORY: {
                need(N * 4);
                std::vector<int8_t> h((size_t)N);
                SNN_CUDA(cudaMemcpyAsync(h.data(), ref.p, (size_t)N, cudaMemcpyDeviceToHost, stream));
                SNN_CUDA(cudaStreamSynchronize(stream));
                for (int64_t j = 0; j < N; ++j) ((int32_t*)buf)[j] = h[j];
                break;
            }
            case SNN_STATE_WEIGHT: dl_syn(w.p, buf, nbytes); break;
            case SNN_STATE_POST: dl_syn(post.p, buf, nbytes); break;
            case SNN_STATE_RESOURCE:
                SNN_REQUIRE(stp, SNN_ERR_UNSUPPORTED, "STP state exists only with SNN_PROP_STP");
                dl(R.p, N * 4);
                break;
            case SNN_STATE_UTIL:
                SNN_REQUIRE(stp, SNN_ERR_UNSUPPORTED, "STP state exists only with SNN_PROP_STP");
                dl(u.p, N * 4);
                break;
            case SNN_STATE_ROW_PTR:
                SNN_REQUIRE(stdp, SNN_ERR_UNSUPPORTED, "the reverse CSR exists only with SNN_PROP_STDP");
                dl(in_ptr.p, (N + 1) * 4);
                break;
            default: throw snnb::Error(SNN_ERR_UNSUPPORTED, "state field not available in this model");
        }
    }

    // a per-synapse array in generation order (rows are stored bucket-sorted)
    void dl_syn(const void* src, void* buf, int64_t nbytes) {
        SNN_REQUIRE(nbytes >= S * 4, SNN_ERR_ARG, "state buffer too small");
        const void* from = src;
        snnb::DevBuf<uint32_t> tmpo;
        if (sorted) {
            tmpo.alloc(S);
            k4_sort_rows<<<148 * 16, 256, 8 * 2 * (D.nb + 1) * sizeof(int), stream>>>(
                nullptr, nullptr, nullptr, D.N, D.F, D.n_exc, spec_seed, D.w_max, D.nb, D.bw,
                (const uint32_t*)src, tmpo.p);
            SNN_CUDA(cudaGetLastError());
            from = tmpo.p;
        }
        SNN_CUDA(cudaMemcpyAsync(buf, from, (size_t)S * 4, cudaMemcpyDeviceToHost, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
    }

    void set_dopamine(float da) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        dopamine = da;
        const float lr = pm_mul(da, D.w_max);
        SNN_CUDA(cudaMemcpyAsync((char*)ctrl.p + offsetof(PCtrl, lr), &lr, 4, cudaMemcpyHostToDevice, stream));
        SNN_CUDA(cudaStreamSynchronize(stream));
    }

    // native full state (SNN_FMT_NATIVE) for bit-exact resume
    struct NativeBlob {
        int64_t steps, raster_base, N, S;
        float dopamine, w_max;
        int32_t mode, raster_cap;
        uint32_t thr, bw;  // bw: bucket width of the stored row order (0: generation order)
    };
    NativeBlob blob() const {
        NativeBlob b{};
        b.steps = steps; b.raster_base = raster_base_host; b.N = D.N; b.S = S;
        b.dopamine = dopamine; b.w_max = D.w_max; b.mode = mode; b.raster_cap = raster_cap; b.thr = D.thr;
        b.bw = sorted ? (uint32_t)D.bw : 0u;
        return b;
    }
    std::vector<snnb::DevSection> native_sections() {
        std::vector<snnb::DevSection> v;
        auto add = [&](const char* n, auto& b) {
            if (b.p) v.push_back({n, (void*)b.p, b.bytes()});
        };
        add("acc", acc); add("V", V); add("I", I); add("ref", ref); add("last_post", last_post);
        add("w", w); add("tA", tA); add("tB", tB); add("u", u); add("R", R); add("pre_list", pre_list);
        add("rel_list", rel_list); add("un_list", un_list); add("rn_list", rn_list);
        add("post_list", post_list); add("raster", raster); add("ctrl", ctrl);
        return v;
    }
    void save(const char* path, int32_t fmt) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_REQUIRE(fmt == SNN_FMT_NATIVE, SNN_ERR_UNSUPPORTED, "the microbench writes the native format only");
        SNN_REQUIRE(world == 1, SNN_ERR_UNSUPPORTED, "a sharded microbench has no checkpoint format");
        const NativeBlob b = blob();
        snnb::save_native(path, SNN_MODEL_PROP, &b, sizeof(b), native_sections(), stream);
    }
    void load(const char* path, int32_t fmt) override {
        SNN_REQUIRE(built, SNN_ERR_STATE, "build the network first");
        SNN_REQUIRE(fmt == SNN_FMT_NATIVE, SNN_ERR_UNSUPPORTED, "the microbench reads the native format only");
        SNN_REQUIRE(world == 1, SNN_ERR_UNSUPPORTED, "a sharded microbench has no checkpoint format");
        const NativeBlob want = blob();
        NativeBlob got{};
        // the weights must keep their sign ranges (excitatory rows [0, w_max],
        // inhibitory rows [-w_max, 0]): the push's int32 sums and the
        // plasticity clamps rely on them
        auto secs = native_sections();
        const size_t n_exc_w = (size_t)D.n_exc * (size_t)D.F;
        const float wm = D.w_max;
        for (auto& sec : secs)
            if (!strcmp(sec.name, "w"))
                sec.validate = [n_exc_w, wm](const char* data, size_t n, size_t off) {
                    const size_t i0 = off / sizeof(float), cnt = n / sizeof(float);
                    const float* x = reinterpret_cast<const float*>(data);
                    for (size_t q = 0; q < cnt; ++q) {
                        const float v = x[q];
                        const bool ok = (i0 + q < n_exc_w) ? (v >= 0.0f && v <= wm) : (v <= 0.0f && v >= -wm);
                        SNN_REQUIRE(ok, SNN_ERR_IO, "checkpoint weight outside its range [0, w_max] / [-w_max, 0]");
                    }
                };
        snnb::load_native(path, SNN_MODEL_PROP, &got, sizeof(got), secs, stream,
                          [&](const void* p) {
                              NativeBlob f;
                              memcpy(&f, p, sizeof(f));
                              SNN_REQUIRE(f.N == want.N && f.S == want.S && f.mode == want.mode &&
                                              f.thr == want.thr && f.raster_cap == want.raster_cap &&
                                              f.w_max == want.w_max && f.bw == want.bw,
                                          SNN_ERR_IO, "checkpoint of another microbench network");
                          });
        steps = got.steps;
        raster_base_host = got.raster_base;
        dopamine = got.dopamine;
    }
};

// ---- snn_propagate ----------------------------------------------------------
__global__ void __launch_bounds__(P_THREADS) k_compact(const uint8_t* spikes, long long n,
                                                        int32_t* list, unsigned* count) {
    const int lane = threadIdx.x & 31;
    for (long long i0 = (long long)blockIdx.x * P_THREADS; i0 < n; i0 += (long long)gridDim.x * P_THREADS) {
        const long long i = i0 + threadIdx.x;
        const bool f = i < n && spikes[i] != 0;
        const unsigned pos = warp_append(f, count, lane);
        if (f && pos < (unsigned long long)n) list[pos] = (int32_t)i;
    }
}

// post indices outside [0, n_post) are skipped (the caller's arrays are not
// trusted to be in range)
__device__ __forceinline__ void add_checked(int32_t* acc, int n_post, int q, float w, float scale) {
    if ((unsigned)q < (unsigned)n_post) atomicAdd(acc + q, (int32_t)pm_rint(pm_mul(w, scale)));
}

template <bool VEC>
__global__ void __launch_bounds__(P_THREADS) k_push_fixed(const int32_t* post, const float* w, int F,
                                                          const int32_t* list, const unsigned* count,
                                                          int32_t* acc, int n_post, float scale) {
    const unsigned n = *count;
    const int lane = threadIdx.x & 31;
    const long long gw = ((long long)blockIdx.x * P_THREADS + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * P_THREADS) >> 5;
    const int F4 = VEC ? F >> 2 : F;
    const int nseg = (F4 + P_SEG4 - 1) / P_SEG4;
    const long long items = (long long)n * nseg;
    for (long long it = gw; it < items; it += nw) {
        const long long e = it / nseg;
        const int c0 = (int)(it - e * nseg) * P_SEG4 + lane;
        const long long i = list[e];
        if (VEC) {
            const int4* p4 = reinterpret_cast<const int4*>(post) + i * F4;
            const float4* w4 = reinterpret_cast<const float4*>(w) + i * F4;
            int4 pv[P_UNROLL];
            float4 wv[P_UNROLL];
#pragma unroll
            for (int u = 0; u < P_UNROLL; ++u) {
                const int c = c0 + u * 32;
                if (c < F4) {
                    pv[u] = __ldcs(p4 + c);
                    wv[u] = __ldcs(w4 + c);
                }
            }
#pragma unroll
            for (int u = 0; u < P_UNROLL; ++u) {
                const int c = c0 + u * 32;
                if (c < F4) {
                    add_checked(acc, n_post, pv[u].x, wv[u].x, scale);
                    add_checked(acc, n_post, pv[u].y, wv[u].y, scale);
                    add_checked(acc, n_post, pv[u].z, wv[u].z, scale);
                    add_checked(acc, n_post, pv[u].w, wv[u].w, scale);
                }
            }
        } else {
            const long long b = i * F;
            for (int c = c0; c < F && c < c0 + P_SEG4; c += 32)
                add_checked(acc, n_post, __ldcs(post + b + c), __ldcs(w + b + c), scale);
        }
    }
}

// per-device scratch of snn_propagate: compacted spike list + its count.
// Calls are chained on the device through `done` (each call's stream waits
// for the previous call), so two calls never use the scratch at once even
// when they are issued on different streams.
struct PropScratch {
    std::mutex mu;
    int32_t* list = nullptr;
    unsigned* count = nullptr;
    long long cap = 0;
    int sms = 0;
    cudaEvent_t done = nullptr;
    bool recorded = false;
    ~PropScratch() {
        if (list) cudaFree(list);
        if (count) cudaFree(count);
        if (done) cudaEventDestroy(done);
    }
};
PropScratch g_scratch[64];

// Scratch of snn_propagate_static: file-scope device arrays, so that entry
// point allocates nothing.  The list holds at most STATIC_MAX_PRE spiking
// neurons; the count is zeroed by every call before the compaction.
constexpr long long STATIC_MAX_PRE = 1ll << 20;
static __device__ __align__(256) int32_t g_static_list[STATIC_MAX_PRE];
static __device__ __align__(256) unsigned g_static_count;

// device addresses of the static scratch, looked up once per device
struct StaticScratch {
    std::mutex mu;
    int32_t* list = nullptr;
    unsigned* count = nullptr;
    int sms = 0;
};
StaticScratch g_static[64];

}  // namespace

namespace snnb {
Engine* make_engine_prop(const snn_config& cfg) { return new EngineProp(cfg); }

void propagate(const int32_t* post, const float* w, int64_t n_pre, int32_t fanout, const uint8_t* spikes,
               int32_t* acc, int64_t n_post, int32_t frac_bits, cudaStream_t st) {
    SNN_REQUIRE(post && w && spikes && acc, SNN_ERR_ARG, "null device pointer");
    SNN_REQUIRE(n_pre >= 0 && n_pre < (1ll << 31), SNN_ERR_ARG, "n_pre must lie in [0, 2^31)");
    SNN_REQUIRE(fanout >= 1, SNN_ERR_ARG, "fanout must be >= 1");
    SNN_REQUIRE(n_post >= 1 && n_post < (1ll << 31), SNN_ERR_ARG, "n_post must lie in [1, 2^31)");
    SNN_REQUIRE(frac_bits >= 0 && frac_bits <= 30, SNN_ERR_ARG, "frac_bits must lie in [0, 30]");
    if (n_pre == 0) return;
    int dev = 0;
    SNN_CUDA(cudaGetDevice(&dev));
    SNN_REQUIRE(dev >= 0 && dev < 64, SNN_ERR_ARG, "device ordinal above 63");
    PropScratch& sc = g_scratch[dev];
    std::lock_guard<std::mutex> lk(sc.mu);
    if (!sc.done) SNN_CUDA(cudaEventCreateWithFlags(&sc.done, cudaEventDisableTiming));
    if (sc.cap < n_pre) {
        if (sc.recorded) SNN_CUDA(cudaEventSynchronize(sc.done));  // the old list may still be read
        if (sc.list) cudaFree(sc.list);
        sc.list = nullptr;
        sc.cap = 0;
        SNN_CUDA(cudaMalloc((void**)&sc.list, (size_t)n_pre * 4));
        sc.cap = n_pre;
    }
    if (!sc.count) SNN_CUDA(cudaMalloc((void**)&sc.count, 4));
    if (!sc.sms) SNN_CUDA(cudaDeviceGetAttribute(&sc.sms, cudaDevAttrMultiProcessorCount, dev));
    if (sc.recorded) SNN_CUDA(cudaStreamWaitEvent(st, sc.done, 0));
    SNN_CUDA(cudaMemsetAsync(sc.count, 0, 4, st));
    const long long cb = std::min<long long>((n_pre + P_THREADS - 1) / P_THREADS, (long long)sc.sms * 8);
    k_compact<<<(unsigned)cb, P_THREADS, 0, st>>>(spikes, n_pre, sc.list, sc.count);
    const float scale = pm_bits2f((uint32_t)(127 + frac_bits) << 23);
    const bool vec = (fanout % 4) == 0 && ((uintptr_t)post % 16) == 0 && ((uintptr_t)w % 16) == 0;
    if (vec) k_push_fixed<true><<<sc.sms * 8, P_THREADS, 0, st>>>(post, w, fanout, sc.list, sc.count, acc, (int)n_post, scale);
    else k_push_fixed<false><<<sc.sms * 8, P_THREADS, 0, st>>>(post, w, fanout, sc.list, sc.count, acc, (int)n_post, scale);
    SNN_CUDA(cudaGetLastError());
    SNN_CUDA(cudaEventRecord(sc.done, st));
    sc.recorded = true;
}

void propagate_static(const int32_t* post, const float* w, int64_t n_pre, int32_t fanout,
                      const uint8_t* spikes, int32_t* acc, int64_t n_post, int32_t frac_bits,
                      cudaStream_t st) {
    SNN_REQUIRE(post && w && spikes && acc, SNN_ERR_ARG, "null device pointer");
    SNN_REQUIRE(n_pre >= 0 && n_pre <= STATIC_MAX_PRE, SNN_ERR_ARG,
                "n_pre above the 1,048,576 neurons of the static scratch (use snn_propagate)");
    SNN_REQUIRE(fanout >= 1, SNN_ERR_ARG, "fanout must be >= 1");
    SNN_REQUIRE(n_post >= 1 && n_post < (1ll << 31), SNN_ERR_ARG, "n_post must lie in [1, 2^31)");
    SNN_REQUIRE(frac_bits >= 0 && frac_bits <= 30, SNN_ERR_ARG, "frac_bits must lie in [0, 30]");
    if (n_pre == 0) return;
    int dev = 0;
    SNN_CUDA(cudaGetDevice(&dev));
    SNN_REQUIRE(dev >= 0 && dev < 64, SNN_ERR_ARG, "device ordinal above 63");
    StaticScratch& sa = g_static[dev];
    {
        std::lock_guard<std::mutex> lk(sa.mu);
        if (!sa.list) {  // first call on this device (the current one)
            int32_t* l = nullptr;
            unsigned* c = nullptr;
            SNN_CUDA(cudaGetSymbolAddress((void**)&l, g_static_list));
            SNN_CUDA(cudaGetSymbolAddress((void**)&c, g_static_count));
            SNN_CUDA(cudaDeviceGetAttribute(&sa.sms, cudaDevAttrMultiProcessorCount, dev));
            sa.count = c;
            sa.list = l;
        }
    }
    SNN_CUDA(cudaMemsetAsync(sa.count, 0, 4, st));
    const long long cb = std::min<long long>((n_pre + P_THREADS - 1) / P_THREADS, (long long)sa.sms * 8);
    k_compact<<<(unsigned)cb, P_THREADS, 0, st>>>(spikes, n_pre, sa.list, sa.count);
    const float scale = pm_bits2f((uint32_t)(127 + frac_bits) << 23);
    const bool vec = (fanout % 4) == 0 && ((uintptr_t)post % 16) == 0 && ((uintptr_t)w % 16) == 0;
    if (vec) k_push_fixed<true><<<sa.sms * 8, P_THREADS, 0, st>>>(post, w, fanout, sa.list, sa.count, acc, (int)n_post, scale);
    else k_push_fixed<false><<<sa.sms * 8, P_THREADS, 0, st>>>(post, w, fanout, sa.list, sa.count, acc, (int)n_post, scale);
    SNN_CUDA(cudaGetLastError());
}
}  // namespace snnb
