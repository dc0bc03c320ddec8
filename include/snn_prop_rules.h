/* snn_prop_rules.h - the seeded rules of the propagation microbench
 * (SNN_MODEL_PROP), shared by the CUDA engine and the CPU oracle so that both
 * generate the same synapses and the same forced spikes.
 *
 * The reference has no propagation microbench; the model is defined here:
 *   - N neurons, F out-edges each; synapse s = i*F + k of pre i targets
 *     post(s) = hi32(h) * N >> 32 with h = mix64(seed * GOLDEN + s), a
 *     uniform draw in [0, N) (self-edges and repeated targets allowed);
 *   - the first floor(0.8 N) neurons are excitatory with w = u * w_max,
 *     the rest inhibitory with w = -u * w_max, u = (h & 0xFFFFFF) * 2^-24;
 *   - pre i spikes at step t iff hi32(mix64(((t << 32) | i) ^ spike_key)) <
 *     thr, thr = floor(rate * 2^32), spike_key = mix64(seed + 1).
 * mix64 is the SplitMix64 output function (Steele, Lea, Flood 2014).
 */
#ifndef SNN_PROP_RULES_H
#define SNN_PROP_RULES_H
#include "snn_pmath.h"

#define SNN_PROP_GOLDEN 0x9E3779B97F4A7C15ull
#define SNN_PROP_FRAC_BITS 24        /* fixed-point scale of the accumulator */
#define SNN_PROP_STP_U 0.5f
#define SNN_PROP_STP_TAU_D 200.0f
#define SNN_PROP_STP_TAU_F 50.0f
#define SNN_PROP_EXP_STEPS 2200      /* exp(-dt/20) table length - 1 */

SNN_HD uint64_t snn_mix64(uint64_t z) {
    z += SNN_PROP_GOLDEN;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

SNN_HD uint64_t snn_prop_syn_hash(uint32_t seed, uint64_t s) {
    return snn_mix64((uint64_t)seed * SNN_PROP_GOLDEN + s);
}

SNN_HD int32_t snn_prop_post(uint64_t h, uint32_t n) {
    return (int32_t)(((h >> 32) * (uint64_t)n) >> 32);
}

/* u * w_max, u in [0, 1) with 24 random bits; negative for inhibitory pres */
SNN_HD float snn_prop_weight(uint64_t h, float w_max, int exc) {
    float u = pm_mul(pm_u2f((uint32_t)(h & 0xFFFFFFu)), 5.9604644775390625e-8f);
    float w = pm_mul(u, w_max);
    return exc ? w : -w;
}

SNN_HD uint64_t snn_prop_spike_key(uint32_t seed) { return snn_mix64((uint64_t)seed + 1ull); }

SNN_HD int snn_prop_spikes(uint64_t key, int32_t t, uint32_t i, uint32_t thr) {
    uint64_t h = snn_mix64((((uint64_t)(uint32_t)t) << 32 | i) ^ key);
    return (uint32_t)(h >> 32) < thr;
}

/* Tsodyks-Markram update of one pre neuron at a spike; dt = steps since its
 * previous spike (< 0: none).  Returns the release u*R. */
SNN_HD float snn_prop_stp(float* u, float* R, int32_t dt) {
    const float U = SNN_PROP_STP_U;
    float uu = *u, rr = *R;
    if (dt >= 0) {
        float x = pm_i2f(-dt);
        float ed = snn_expf(pm_div(x, SNN_PROP_STP_TAU_D));
        float ef = snn_expf(pm_div(x, SNN_PROP_STP_TAU_F));
        rr = pm_sub(1.0f, pm_mul(pm_sub(1.0f, rr), ed));
        uu = pm_fma(pm_sub(uu, U), ef, U);
    }
    uu = pm_fma(U, pm_sub(1.0f, uu), uu);
    float rel = pm_mul(uu, rr);
    *u = uu;
    *R = pm_sub(rr, rel);
    return rel;
}

/* fixed-point contribution of one synapse: rint(w * release * 2^24) */
SNN_HD int32_t snn_prop_quant(float w, float rel, int stp) {
    float x = stp ? pm_mul(w, rel) : w;
    return (int32_t)pm_rint(pm_mul(x, 16777216.0f));
}

#endif /* SNN_PROP_RULES_H */
