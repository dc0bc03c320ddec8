/*
 * snn_pmath.h - portable, bit-reproducible float32 arithmetic shared by the
 * CUDA kernels (sm_100a) and the CPU oracle.
 *
 * Every rounding step on the simulation path goes through these helpers so
 * that the GPU and the CPU produce identical IEEE-754 binary32 results:
 *   - add/mul/div/fma are single correctly-rounded operations
 *     (__fadd_rn/__fmul_rn/__fdiv_rn/__fmaf_rn on the device, which the
 *     compiler never contracts; plain operators with -ffp-contract=off and
 *     std::fmaf on the host);
 *   - denormals are kept on both sides (no FTZ/DAZ);
 *   - snn_expf() is this project's own exponential, not the CUDA or libm one.
 *
 * snn_expf method: Cody & Waite additive range reduction (W. J. Cody and
 * W. Waite, "Software Manual for the Elementary Functions", 1980):
 *     k = rint(x * log2(e)),  r = (x - k*ln2_hi) - k*ln2_lo   (two fmas)
 * so that |r| <= ln2/2, followed by the degree-7 Taylor polynomial of e^r in
 * Horner form (truncation error < 5e-9 relative on |r| <= 0.3466, below half
 * an ulp of binary32), and an exact scaling by 2^k built from the exponent
 * bits (split in two factors when the result is subnormal).  The result is
 * within a couple of ulp of the true exponential; tests measure the error
 * against libm expf.
 */
#ifndef SNN_PMATH_H
#define SNN_PMATH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define SNN_HD __host__ __device__ __forceinline__
#else
#define SNN_HD static inline
#include <math.h>
#include <string.h>
#endif

#if defined(__CUDA_ARCH__)
SNN_HD float pm_add(float a, float b) { return __fadd_rn(a, b); }
SNN_HD float pm_sub(float a, float b) { return __fsub_rn(a, b); }
SNN_HD float pm_mul(float a, float b) { return __fmul_rn(a, b); }
SNN_HD float pm_div(float a, float b) { return __fdiv_rn(a, b); }
SNN_HD float pm_fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
SNN_HD float pm_rint(float x) { return rintf(x); }
SNN_HD float pm_i2f(int x) { return __int2float_rn(x); }
SNN_HD float pm_u2f(unsigned x) { return __uint2float_rn(x); }
SNN_HD float pm_ll2f(long long x) { return __ll2float_rn(x); }
SNN_HD float pm_bits2f(uint32_t b) { return __uint_as_float(b); }
SNN_HD uint32_t pm_f2bits(float f) { return __float_as_uint(f); }
#else
/* Host side: compiled with -ffp-contract=off, no fast-math. volatile-free:
 * each operator below is one IEEE operation in round-to-nearest-even. */
SNN_HD float pm_add(float a, float b) { return a + b; }
SNN_HD float pm_sub(float a, float b) { return a - b; }
SNN_HD float pm_mul(float a, float b) { return a * b; }
SNN_HD float pm_div(float a, float b) { return a / b; }
SNN_HD float pm_fma(float a, float b, float c) { return fmaf(a, b, c); }
SNN_HD float pm_rint(float x) { return rintf(x); }
SNN_HD float pm_i2f(int x) { return (float)x; }
SNN_HD float pm_u2f(unsigned x) { return (float)x; }
SNN_HD float pm_ll2f(long long x) { return (float)x; }
SNN_HD float pm_bits2f(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
SNN_HD uint32_t pm_f2bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
#endif

SNN_HD float pm_min(float a, float b) { return (b < a) ? b : a; }
SNN_HD float pm_max(float a, float b) { return (b > a) ? b : a; }

/* e^x in binary32, bit-identical on host and device (see header comment). */
SNN_HD float snn_expf(float x) {
    if (x != x) return x;                          /* NaN */
    if (x > 88.75f) return pm_bits2f(0x7f800000u); /* +inf */
    if (x < -104.0f) return 0.0f;
    const float LOG2E = 1.44269502162933349609375f;   /* 0x3fb8aa3b */
    const float LN2_HI = 0.693145751953125f;          /* 0x3f317200, 16 bits */
    const float LN2_LO = 1.428606765330187045e-06f;   /* ln2 - LN2_HI */
    float kf = pm_rint(pm_mul(x, LOG2E));
    float r = pm_fma(-kf, LN2_HI, x);
    r = pm_fma(-kf, LN2_LO, r);
    /* Taylor coefficients 1/n!, n = 7..0 */
    float p = 1.98412701138295233249664306640625e-4f;   /* 1/5040 */
    p = pm_fma(p, r, 1.388888922519981861114501953125e-3f); /* 1/720 */
    p = pm_fma(p, r, 8.333333767950534820556640625e-3f);    /* 1/120 */
    p = pm_fma(p, r, 4.1666667163372039794921875e-2f);      /* 1/24 */
    p = pm_fma(p, r, 1.6666667163372039794921875e-1f);      /* 1/6 */
    p = pm_fma(p, r, 0.5f);
    p = pm_fma(p, r, 1.0f);
    p = pm_fma(p, r, 1.0f);
    int k = (int)kf;
    if (k > 127) /* k == 128: p < 1 can still be finite */
        return pm_mul(pm_mul(p, pm_bits2f(0x7f000000u)), 2.0f);
    if (k >= -126) return pm_mul(p, pm_bits2f((uint32_t)(k + 127) << 23));
    /* subnormal result: 2^k = 2^-126 * 2^(k+126), second factor >= 2^-24 */
    float t = pm_mul(p, pm_bits2f(1u << 23)); /* * 2^-126 */
    return pm_mul(t, pm_bits2f((uint32_t)(k + 126 + 127) << 23));
}

#endif /* SNN_PMATH_H */
