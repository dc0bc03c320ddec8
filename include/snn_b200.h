/*
 * snn_b200.h - C ABI of the B200-native spiking-network core.
 *
 * A thin, exception-free C boundary over the host C++ engines and their
 * sm_100a CUDA kernels.  All device memory is owned by the context handle;
 * host buffers are owned by the caller.  A context is used by one host
 * thread at a time.  Every entry point returns SNN_OK (0) or an SNN_ERR_*
 * code; snn_last_error() gives the message.  Nothing here calls exit().
 *
 * Each entry point replaces a piece of the reference's host C++ API
 * (TSOFTP-afk/pure-snn-language; paths relative to that project):
 *
 *   snn_create / snn_destroy
 *       stage2e::MemoryAllocator::allocate_all / free_all
 *           (src/stage2e/memory_allocator.cuh:306-339),
 *       SNNNetwork::SNNNetwork / ~SNNNetwork / cleanup
 *           (src/include/network.h:11-95, src/host/network.cpp:15-26)
 *   snn_build_columns
 *       stage2e::init_network (src/stage2e/network_init.cuh:42,
 *           src/stage2e/network_init.cu:573-594),
 *       SNNNetwork::initialize / allocate_only + init_columnar_synapses
 *           (src/host/network.cpp:78-135, src/stage2/columnar_topology.cu:47-143)
 *   snn_set_corpus
 *       stage2e::load_text_corpus (src/stage2e/input_encoding.cuh:35-50,
 *           src/stage2e/input_encoding.cu:40-96)
 *   snn_step
 *       stage2e::BioMechanismScheduler::step(int) (src/stage2e/scheduler.cuh:75,
 *           src/stage2e/scheduler.cu:485-676),
 *       SNNNetwork::step(const float*, int) (src/include/network.h:29,
 *           src/host/network.cpp:143-191)
 *   snn_run
 *       the per-step host loops of src/stage2e/main.cpp:679-743 and
 *       src/stage2/unsupervised_trainer.cu:96-171, as one call
 *   snn_set_dopamine    SNNNetwork::set_dopamine (src/include/network.h:44)
 *   snn_set_e0          stage2e::set_e0_ablation (src/stage2e/synapse_kernels.cuh:82)
 *                       + BioMechanismScheduler::e0_ablation (scheduler.cuh:72)
 *   snn_get_spikes      d_spike_flags reads (src/stage2e/scheduler.cu:627-634)
 *   snn_get_state       the raw device-pointer getters (src/include/network.h:58-67)
 *                       and PersistentBuffers (src/stage2e/memory_allocator.cuh:226-301)
 *   snn_get_counters    BioMechanismScheduler stats getters (scheduler.cuh:78-123),
 *                       SNNNetwork::get_stats (src/include/network.h:40)
 *   snn_save / snn_load SNNNetwork::save_weights / load_weights
 *                       (src/host/network.cpp:224-290), save_checkpoint /
 *                       load_checkpoint (src/stage2/unsupervised_trainer.cu:176-348),
 *                       BioMechanismScheduler::save_checkpoint (scheduler.cu:402-483)
 */
#ifndef SNN_B200_H
#define SNN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define SNN_OK 0
#define SNN_ERR_ARG 1          /* bad argument / size mismatch            */
#define SNN_ERR_CUDA 2         /* CUDA runtime error (message has detail) */
#define SNN_ERR_OOM 3          /* device or host allocation failed        */
#define SNN_ERR_STATE 4        /* call out of order (e.g. step before build) */
#define SNN_ERR_IO 5           /* file missing / truncated / bad magic    */
#define SNN_ERR_UNSUPPORTED 6  /* option not available for this model    */
#define SNN_ERR_NO_DEVICE 7    /* no CUDA device visible                  */

/* ---- models and presets ---------------------------------------------- */
#define SNN_MODEL_STAGE2E 0  /* AdEx + NMDA/Ca + STP + PSW STDP + delays   */
#define SNN_MODEL_STAGE0 1   /* LIF + pair STDP + eligibility + dopamine   */
#define SNN_MODEL_PROP 2     /* propagation microbench: forced Poisson pre-spikes,
                                fixed fan-out, push propagation into LIF neurons */

/* Propagation microbench modes (bit flags, SNN_MODEL_PROP only).  The model
 * has no counterpart in the reference; its step t is:
 *   1. pre-spikes: neuron i spikes iff hash(seed, t, i) < prop_rate * 2^32;
 *      with SNN_PROP_STP its release is u*R of a per-neuron Tsodyks-Markram
 *      state (U 0.5, tau_d 200, tau_f 50 steps), else 1;
 *   2. push: acc[post] += round(w * release * 2^24) over the out-edges of
 *      every spiking neuron (exact int32 sums); with SNN_PROP_STDP each
 *      excitatory out-synapse then gets LTD -0.05*exp(-dt/20) scaled by
 *      dopamine * w_max (dt = t - last LIF spike of its post);
 *   3. LIF (Stage 0 form, threshold 1, refractory 2) on input acc * 2^-24;
 *   4. with SNN_PROP_STDP: LTP +0.05*exp(-dt/20) * dopamine * w_max on the
 *      excitatory incoming synapses of every LIF spike (dt = t - last
 *      pre-spike before t), through a reverse CSR; weights clamp to
 *      [0, w_max].  The first 80 % of neurons are excitatory. */
#define SNN_PROP_PLAIN 0
#define SNN_PROP_STDP 1
#define SNN_PROP_STP 2

#define SNN_PRESET_REF 0      /* constants exactly as the reference kernels
                                 (Stage 0 model: the reference's Stage 0 build
                                 for the block network, its Stage 2 build for
                                 columns) */
#define SNN_PRESET_BASELINE 1 /* constants as stated in the benchmark spec  */

typedef struct snn_ctx snn_ctx;

typedef struct snn_config {
    int32_t model;         /* SNN_MODEL_*                                     */
    int32_t preset;        /* SNN_PRESET_*                                    */
    int32_t device;        /* CUDA device ordinal                             */
    int32_t e0;            /* Stage 2e E0 ablation (pure STDP)                 */
    int32_t phase_offset;  /* Stage 2e: added to the step for the phase table */
    int32_t raster_steps;  /* device spike-raster capacity in steps (0 = 1024) */
    int32_t prop_mode;     /* SNN_MODEL_PROP: SNN_PROP_* flags                 */
    float prop_rate;       /* SNN_MODEL_PROP: forced spike probability per step */
    float prop_w_max;      /* SNN_MODEL_PROP: weight bound (0 = 0.01 / (rate * fan-out)) */
    int32_t prop_push;     /* SNN_MODEL_PROP push kernel: 0 auto, 1 one L2 atomic per
                              synapse, 2 bucketed shared-memory accumulation (same sums) */
    int32_t reserved[6];
} snn_config;

/* Network construction by columns and layers.
 * Stage 2e: n_columns cortical columns of l4/l23/l5/l6 neurons plus
 *   pf_groups prefrontal groups of pf_group_size neurons, generated with the
 *   reference rules (src/stage2e/network_init.cu:158-473) when rule == 0.
 * Stage 0: n_columns == 0 gives the single-block 2000/6000/2000 network; with
 *   n_columns > 0 each column is l4 (sensory) / l23 (association) / l5
 *   (motor) neurons.
 * Propagation microbench: l4 neurons, deg_intra out-edges each (uniform
 *   random targets, generated on the device from `seed`). */
typedef struct snn_topology_spec {
    int32_t n_columns;
    int32_t l4, l23, l5, l6;
    int32_t pf_groups, pf_group_size;
    int32_t deg_intra, deg_inter, deg_l5_pf, deg_pf_self, deg_pf_assoc;
    int64_t total_synapses;
    uint32_t seed;
    int32_t rule;          /* 0 = reference generator; 1 = uniform out-degree */
    int32_t reserved[8];
} snn_topology_spec;

typedef struct snn_counters {
    int64_t step;            /* steps executed                              */
    int64_t total_spikes;
    int64_t arrivals;        /* delivered (pre-spike, synapse) events       */
    int64_t dispatched;      /* out-edges of spiking neurons                */
    int64_t dropped_ref;     /* events the reference's 750K slots would drop */
    int64_t ltp_visits;      /* incoming synapses of spiking neurons        */
    int64_t burst_spikes;    /* spikes within 5 steps of the previous one   */
    int64_t n_neurons;
    int64_t n_synapses;
    int64_t n_groups;        /* Stage 2e (pre, delay, class) synapse groups */
    int32_t last_spikes;     /* spikes of the last executed step            */
    int32_t last_byte;       /* byte injected at the last step, -1 = none   */
    double modeled_bytes;    /* algorithmic HBM bytes of the executed steps */
    int64_t local_lo;        /* [local_lo, local_hi): the neurons this context
                                advances (a sharded microbench's post buckets; */
    int64_t local_hi;        /*  otherwise 0 / n_neurons)                     */
    int64_t reserved[4];
} snn_counters;

/* fields for snn_get_state (host_buf gets n elements of the listed type;
 * synapse fields are returned in the reference's pre-major synapse order) */
enum {
    SNN_STATE_V = 0,           /* f32[N] membrane potential                 */
    SNN_STATE_W_ADAPT = 1,     /* f32[N] AdEx adaptation w                  */
    SNN_STATE_SYN_CURRENT = 2, /* f32[N] leaky synaptic current s           */
    SNN_STATE_FIRE_RATE = 3,   /* f32[N]                                    */
    SNN_STATE_CA_NEURON = 4,   /* f32[N]                                    */
    SNN_STATE_INPUT = 5,       /* f32[N] input current for the next step    */
    SNN_STATE_NMDA_CUR = 6,    /* f32[N] NMDA current for the next step     */
    SNN_STATE_LAST_SPIKE = 7,  /* i32[N]                                    */
    SNN_STATE_REFRACTORY = 8,  /* i32[N]                                    */
    SNN_STATE_X_POST = 9,      /* f32[N] post trace                         */
    SNN_STATE_THRESH_OFF = 10, /* i32[N] threshold offset (fixed point)     */
    SNN_STATE_ALPHA = 20,      /* f32[S] PSW alpha                          */
    SNN_STATE_BETA = 21,       /* f32[S] PSW beta                           */
    SNN_STATE_WEIGHT = 22,     /* f32[S] weight (derived for Stage 2e)      */
    SNN_STATE_X_PRE = 23,      /* f32[S]                                    */
    SNN_STATE_NMDA_G = 24,     /* f32[S]                                    */
    SNN_STATE_CA = 25,         /* f32[S]                                    */
    SNN_STATE_RESOURCE = 26,   /* f32[S] STP R                              */
    SNN_STATE_UTIL = 27,       /* f32[S] STP u                              */
    SNN_STATE_ELIG = 28,       /* f32[S]                                    */
    SNN_STATE_CAMKII_ACT = 29, /* f32[S]                                    */
    SNN_STATE_CAMKII_AUTO = 30,/* f32[S]                                    */
    SNN_STATE_E1 = 31,         /* f32[S]                                    */
    SNN_STATE_E2 = 32,         /* f32[S]                                    */
    SNN_STATE_AMPA = 33,       /* f32[S] AMPA conductance (Stage 2e)        */
    SNN_STATE_LAST_PRE = 34,   /* f32[S] step of the last arrival (Stage 2e) */
    SNN_STATE_POST = 40,       /* i32[S] post neuron of each synapse        */
    SNN_STATE_DELAY = 41,      /* u8[S]                                     */
    SNN_STATE_ROW_PTR = 42,    /* i32[N+1] pre-major CSR row pointer        */
    SNN_STATE_FLAGS = 43,      /* u8[S] receptor flags                      */
    SNN_STATE_GATES = 50,      /* f32[4*n_columns] gate, act_ema, nov_ema, l6_ema */
    SNN_STATE_MODULATORS = 51, /* f32[4] DA, ACh, NE, 5HT                   */
    SNN_STATE_BYTE_HIST = 52,  /* i32[256] spikes per injected byte         */
    SNN_STATE_NEURON_BYTE_COUNTS = 53 /* i32[N*256]                         */
};

/* on-disk formats for snn_save / snn_load */
enum {
    SNN_FMT_NATIVE = 0,   /* full state, bit-exact resume                  */
    SNN_FMT_SNN2_V1 = 1,  /* src/stage2/unsupervised_trainer.cu:176-262     */
    SNN_FMT_SCKP_V2 = 2,  /* src/stage2e/scheduler.cu:411-483 (save only in the reference) */
    SNN_FMT_RAW_F32 = 3   /* src/host/network.cpp:224-290                   */
};

int snn_config_init(snn_config* cfg, int32_t model, int32_t preset);
int snn_topology_init(snn_topology_spec* spec, int32_t model, int32_t n_columns);
int snn_create(const snn_config* cfg, snn_ctx** out);
void snn_destroy(snn_ctx* ctx);
const char* snn_last_error(const snn_ctx* ctx);
const char* snn_version(void);

int snn_build_columns(snn_ctx* ctx, const snn_topology_spec* spec);

/* Text stream with the reference semantics: one byte per inject step,
 * wrapping at the end (src/stage2e/input_encoding.cu:192-203).  The bytes
 * are copied to device memory. */
int snn_set_corpus(snn_ctx* ctx, const uint8_t* bytes, int64_t n);

/* snn_set_corpus with options.  flags = SNN_CORPUS_TEXT_FILTER applies the
 * reference's text-corpus filter first: NUL bytes dropped, CR / LF / TAB
 * mapped to a space, every other byte (UTF-8 included) kept
 * (src/stage2e/input_encoding.cu:49-64, src/stage2/text_stream.cu:38-52);
 * flags = 0 is snn_set_corpus.  n_kept (nullable) receives the length of the
 * corpus the network reads. */
#define SNN_CORPUS_TEXT_FILTER 1
int snn_set_corpus_ex(snn_ctx* ctx, const uint8_t* bytes, int64_t n, int32_t flags,
                      int64_t* n_kept);

/* stage2e::load_text_corpus(const char* path) (src/stage2e/input_encoding.cu:
 * 40-96) and TextStream::load_from_file (src/stage2/text_stream.cu:30-63):
 * reads the whole file, applies the text-corpus filter and makes the result
 * the corpus (read position 0).  SNN_ERR_IO if the file cannot be read or
 * nothing is left after filtering (the reference returns 0 / false there).
 * n_kept (nullable) receives the filtered length. */
int snn_load_text_corpus(snn_ctx* ctx, const char* path, int64_t* n_kept);

/* Byte classes of a buffer, as the reference's loader reports them
 * (src/stage2e/input_encoding.cu:68-74): out[0] ASCII (< 0x80), out[1] UTF-8
 * lead bytes (0xC0..0xF7), out[2] continuation bytes (0x80..0xBF); n_out >= 3.
 * Host only. */
int snn_byte_classes(const uint8_t* bytes, int64_t n, int64_t* out, int32_t n_out);

/* One step.  `step` must equal the number of steps executed so far.
 * Stage 2e: on steps with step % 3 == 0 the byte is inject_byte if >= 0,
 *   else the next corpus byte (or (step/3)%256 without a corpus).
 * Stage 0: inject_byte >= 0 drives its one-hot input, -1 = no input.
 * learn = 0 freezes plasticity (gain forced to 0). */
int snn_step(snn_ctx* ctx, int32_t step, int32_t inject_byte, int32_t learn);

/* n_steps steps as one call, with no host synchronisation between steps.
 * bytes (nullable) replaces the corpus for this and later calls.  If
 * raster_out is non-null it receives n_steps spike bitmasks of
 * ceil(N/32) words each; counts_out (nullable) receives n_steps spike counts.
 * Stage 2e runs the steps as CUDA graphs on the context's own stream: graphs
 * of 50 steps and one of the remainder, captured the first time a length is
 * needed (a few milliseconds) and kept for the four most recently used
 * lengths, so repeated calls of one size replay graphs.  snn_step is a call of
 * one step.  Do not call these while the calling thread is capturing a
 * stream of its own. */
int snn_run(snn_ctx* ctx, int32_t n_steps, const uint8_t* bytes, int64_t n_bytes,
            int32_t learn, uint32_t* raster_out, int32_t* counts_out);

int snn_synchronize(snn_ctx* ctx);
int snn_get_spikes(snn_ctx* ctx, uint32_t* bitmask, int64_t n_words);
int snn_get_state(snn_ctx* ctx, int32_t which, void* host_buf, int64_t n_bytes);
int snn_get_counters(snn_ctx* ctx, snn_counters* out);

/* Semantic evaluation of a Stage 2e network, replacing
 * BioMechanismScheduler::run_semantic_eval / launch_semantic_eval
 * (src/stage2e/scheduler.cuh:126, scheduler.cu:785-1036), which the
 * reference runs every 10,000 steps: the columns' byte responses (the neuron
 * x byte spike counts summed per column on the device), their pairwise
 * Jensen-Shannon divergences (natural log; an empty column counts as
 * uniform), k-means (k 5, JS distance, round-robin start, at most 20
 * rounds), the silhouette, the column ratio (largest / smallest non-zero
 * column total), each layer's mean spike delay after the last injection
 * step before `step`, and each layer's chi-squared byte selectivity (rows
 * with >= 10 spikes, uniform expectation, df 255, critical 293.2).  Host
 * arithmetic in double as the reference's; per-neuron chi-squared in float
 * on the device, each layer's float sum taken in ascending neuron order (the
 * reference adds them with float atomics, in no fixed order).  Layers are
 * L4, L2/3, L5, L6, prefrontal.  assign (nullable, n_assign >= columns)
 * receives each column's cluster.  Not available on sharded contexts. */
typedef struct snn_semantic {
    double silhouette, js_mean, js_max, column_ratio, grand_total;
    int32_t n_columns, nonzero_columns;
    double layer_delay[5];       /* -1: no neuron of the layer spiked since */
    int32_t layer_delay_n[5];    /* neurons counted in layer_delay          */
    int32_t layer_sig[5];        /* rows above the chi-squared critical value */
    int32_t layer_act[5];        /* rows with >= 10 spikes                  */
    double layer_chi2_mean[5];   /* float sum / layer_act                   */
    int32_t reserved[8];
} snn_semantic;
int snn_semantic_eval(snn_ctx* ctx, int64_t step, snn_semantic* out, int32_t* assign,
                      int64_t n_assign);

int snn_set_dopamine(snn_ctx* ctx, float level);
int snn_set_e0(snn_ctx* ctx, int32_t enable);
/* Device timing of the engine's kernels: with level 1, CUDA events recorded
 * on the engine stream around every kernel of every step (captured into the
 * step graph), cumulative since snn_set_profiling(ctx, 1).  With level 2
 * (Stage 2e engine) only one event pair around each snn_run / snn_step call:
 * step_ms and steps without per-kernel slots and without events inside the
 * steps; other engines treat 2 as 1. */
typedef struct snn_profile {
    int64_t steps;           /* steps timed                                  */
    int32_t n_kernels;       /* kernels per step                              */
    int32_t reserved0;
    double kernel_ms[8];     /* summed device time per kernel slot            */
    int64_t launches[8];     /* launches per kernel slot                      */
    double step_ms;          /* summed device time of whole steps             */
    char names[8][32];       /* kernel names                                  */
} snn_profile;
int snn_set_profiling(snn_ctx* ctx, int32_t enable);
int snn_get_profile(snn_ctx* ctx, snn_profile* out);

int snn_save(snn_ctx* ctx, const char* path, int32_t fmt);
int snn_load(snn_ctx* ctx, const char* path, int32_t fmt);

/* Column sharding of the Stage 2e network over `world` GPUs, one process (and
 * one snn_ctx) per GPU; call before snn_build_columns.  Rank r owns the
 * columns [ncol r / world, ncol (r+1) / world) and the prefrontal groups
 * split the same way, keeps only the synapses onto its neurons, and mirrors
 * the groups of remote pres; every step all-gathers the ranks' spike
 * bitmasks, spike counts and TD sub-population counts over NCCL, so the
 * dynamics stay bit-identical to one GPU.  Rasters, neuron state and
 * per-synapse state are the rank's own; total_spikes / last_spikes in
 * snn_get_counters are global, the event counters local.  uid is the
 * 128-byte ncclUniqueId from snn_nccl_unique_id on one rank, shared with
 * the others by the caller (no counterpart in the reference, which runs on
 * one GPU; replaces its single-device MemoryAllocator,
 * src/stage2e/memory_allocator.cuh:306-339).
 * The propagation microbench shards by post bucket instead (uid may be
 * null; nothing is exchanged): rank r advances the neurons
 * [local_lo, local_hi) of snn_get_counters (the post buckets
 * [nb r / world, nb (r+1) / world), nb a multiple of world), draws every
 * forced pre-spike itself and pushes the segments of their rows that land
 * on its neurons; rasters, neuron state and the weights onto its neurons are
 * its own (entries of other ranks' neurons stay as built), total_spikes,
 * arrivals and ltp_visits are local, dispatched is global; sharded
 * microbench contexts have no checkpoint format. */
int snn_nccl_unique_id(uint8_t* out, int64_t n);
int snn_set_shard(snn_ctx* ctx, int32_t rank, int32_t world, const uint8_t* uid, int64_t n);
/* Host-only partition plan (no GPU): out[0..9] = local neurons, a0, a1, pf0,
 * pf1 (the two global neuron ranges), local synapses, groups of local pres,
 * mirror groups, mirror pres, and the number of local synapses whose remote
 * pre has an effective delay below 5 steps. */
int snn_shard_plan(const snn_topology_spec* spec, int32_t rank, int32_t world, int64_t* out,
                   int32_t n_out);

/* Push propagation of one step's spikes through a fixed-fan-out CSR held in
 * device memory (replaces synaptic_transmission_kernel,
 * src/cuda/synapse_kernel.cu:28-47, whose float atomicAdd order is not
 * deterministic).  All pointers are device pointers; the call is
 * asynchronous on `stream` (a cudaStream_t, NULL = legacy default stream):
 *   for every neuron i < n_pre with spikes[i] != 0 and every k < fanout:
 *     acc[post[i*fanout + k]] += rint(w[i*fanout + k] * 2^frac_bits)   (int32)
 * The sum is exact integer arithmetic (wrapping on overflow), so the result
 * does not depend on the order of the additions.  post[] entries must lie in
 * [0, n_post) (others are skipped); |w| * 2^frac_bits < 2^31; 0 <= frac_bits
 * <= 30.  The compacted list of spiking neurons lives in scratch device
 * memory that the first call on a device allocates and later calls reuse
 * (grown when n_pre grows; freed at process exit).  Calls on one device are
 * chained on the device (each call's stream waits for the previous call), so
 * calls from several streams or threads are safe but do not overlap; the call
 * may allocate and must not be captured into a CUDA graph.  This is the push
 * kernel of SNN_MODEL_PROP. */
int snn_propagate(const int32_t* post, const float* w, int64_t n_pre, int32_t fanout,
                  const uint8_t* spikes, int32_t* acc, int64_t n_post, int32_t frac_bits,
                  void* stream);

/* snn_propagate without any allocation (no counterpart in the reference).
 * For callers that must not allocate device memory once they run: cudaMalloc
 * and cudaFree synchronise the whole device, which stalls a pipelined
 * multi-stream simulation loop, and a process that reserves its device
 * memory up front (a fixed budget, or a pool that owns the rest of the GPU)
 * has nothing left to grant.  Same arguments, semantics and error codes as
 * snn_propagate; the spike list lives in a file-scope device array of
 * 1,048,576 entries (4 MiB), so n_pre above 1,048,576 is rejected with
 * SNN_ERR_ARG.  The first call on a device looks up that array's address
 * (with the device current), so make it before any stream capture; the
 * address is kept for the life of the process, so a device reset
 * (cudaDeviceReset) or a new primary context invalidates it (as it does the
 * scratch of snn_propagate): do not call either after one.  Each
 * call zeroes the list count on `stream` before use.  All calls on one device
 * share the array: calls that overlap in time on different streams race and
 * give wrong sums; order them on one stream (or with events). */
int snn_propagate_static(const int32_t* post, const float* w, int64_t n_pre, int32_t fanout,
                         const uint8_t* spikes, int32_t* acc, int64_t n_post, int32_t frac_bits,
                         void* stream);

/* Seeded synthetic UTF-8 byte stream: a fraction p_cjk of characters are
 * CJK code points U+4E00..U+9FFF drawn Zipf(zipf_s) by rank (rank -> code
 * point through a seeded permutation), 3 bytes each; the rest are ASCII
 * space (90 %) or one of ",.!?;:".  Writes exactly n bytes. */
int snn_stream_generate(uint8_t* out, int64_t n, uint64_t seed, double p_cjk, double zipf_s);

#ifdef __cplusplus
}
#endif
#endif /* SNN_B200_H */
