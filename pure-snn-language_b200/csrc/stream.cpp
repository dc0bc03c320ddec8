// stream.cpp - seeded synthetic Chinese-like UTF-8 byte stream.
//
// Stands in for the LCCC text corpus the reference trains on (its
// data/lccc_sample_1mb.txt is read by src/stage2e/main.cpp:637-643).  A
// character is CJK with probability p_cjk: rank r in [0, 20992) drawn from a
// Zipf(s) law, mapped to a code point U+4E00 + perm[r] through a seeded
// Fisher-Yates permutation, encoded as 3 UTF-8 bytes; otherwise ASCII: space
// with probability 0.9, else one of ",.!?;:".  The output is cut at exactly
// n bytes.  Random source: splitmix64.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>
#include "snn_b200.h"

namespace {
struct SplitMix64 {
    uint64_t s;
    uint64_t next() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double uniform() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
};
}  // namespace

extern "C" int snn_stream_generate(uint8_t* out, int64_t n, uint64_t seed, double p_cjk,
                                   double zipf_s) {
    if (!out || n < 0 || p_cjk < 0.0 || p_cjk > 1.0 || zipf_s <= 0.0) return SNN_ERR_ARG;
    const int NC = 0x9FFF - 0x4E00 + 1;  // 20992 code points
    SplitMix64 rng{seed};
    std::vector<int> perm(NC);
    for (int i = 0; i < NC; ++i) perm[i] = i;
    for (int i = NC - 1; i > 0; --i) {
        int j = (int)(rng.next() % (uint64_t)(i + 1));
        std::swap(perm[i], perm[j]);
    }
    std::vector<double> cdf(NC);
    double acc = 0.0;
    for (int r = 0; r < NC; ++r) {
        acc += 1.0 / std::pow((double)(r + 1), zipf_s);
        cdf[r] = acc;
    }
    for (int r = 0; r < NC; ++r) cdf[r] /= acc;
    static const char punct[6] = {',', '.', '!', '?', ';', ':'};
    int64_t k = 0;
    while (k < n) {
        if (rng.uniform() < p_cjk) {
            double u = rng.uniform();
            int r = (int)(std::lower_bound(cdf.begin(), cdf.end(), u) - cdf.begin());
            if (r >= NC) r = NC - 1;
            uint32_t cp = 0x4E00u + (uint32_t)perm[r];
            uint8_t b[3] = {(uint8_t)(0xE0 | (cp >> 12)), (uint8_t)(0x80 | ((cp >> 6) & 0x3F)),
                            (uint8_t)(0x80 | (cp & 0x3F))};
            for (int q = 0; q < 3 && k < n; ++q) out[k++] = b[q];
        } else {
            out[k++] = rng.uniform() < 0.9 ? (uint8_t)' ' : (uint8_t)punct[rng.next() % 6];
        }
    }
    return SNN_OK;
}
