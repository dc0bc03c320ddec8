// oracle_stream.cpp - TEST INFRASTRUCTURE ONLY (CPU oracle library).
//
// The synthetic input of the benchmark, restated here so that the CPU legs
// of bench.py (the reference arm, the CPU baseline) drive the oracle without
// loading the product library:
//   o_stream_generate   the seeded Chinese-like UTF-8 stream (splitmix64;
//                       a character is CJK with probability p_cjk, its
//                       Zipf(s) rank over U+4E00..U+9FFF mapped through a
//                       seeded Fisher-Yates permutation, 3 UTF-8 bytes; else
//                       space (90 %) or one of ",.!?;:"), cut at n bytes.
//                       tests/test_oracle.py checks it byte for byte against
//                       the product's snn_stream_generate.
//   o_text_filter       the reference corpus filter: NUL dropped, \r \n \t
//                       mapped to a space, every other byte kept
//                       (src/stage2e/input_encoding.cu:49-64,
//                       src/stage2/text_stream.cu:38-52).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

namespace {
struct Mix64 {
    uint64_t s;
    uint64_t next() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double unit() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
};
}  // namespace

extern "C" int o_stream_generate(uint8_t* out, int64_t n, uint64_t seed, double p_cjk,
                                 double zipf_s) {
    if (!out || n < 0 || p_cjk < 0.0 || p_cjk > 1.0 || zipf_s <= 0.0) return 1;
    constexpr int kCodes = 0x9FFF - 0x4E00 + 1;
    Mix64 rng{seed};
    std::vector<int> perm(kCodes);
    for (int i = 0; i < kCodes; ++i) perm[i] = i;
    for (int i = kCodes - 1; i > 0; --i) {
        const int j = (int)(rng.next() % (uint64_t)(i + 1));
        std::swap(perm[i], perm[j]);
    }
    std::vector<double> cdf(kCodes);
    double total = 0.0;
    for (int r = 0; r < kCodes; ++r) {
        total += 1.0 / std::pow((double)(r + 1), zipf_s);
        cdf[r] = total;
    }
    for (int r = 0; r < kCodes; ++r) cdf[r] /= total;
    static const uint8_t kPunct[6] = {',', '.', '!', '?', ';', ':'};
    int64_t k = 0;
    while (k < n) {
        if (rng.unit() < p_cjk) {
            const double u = rng.unit();
            int r = (int)(std::lower_bound(cdf.begin(), cdf.end(), u) - cdf.begin());
            if (r >= kCodes) r = kCodes - 1;
            const uint32_t cp = 0x4E00u + (uint32_t)perm[r];
            const uint8_t enc[3] = {(uint8_t)(0xE0 | (cp >> 12)), (uint8_t)(0x80 | ((cp >> 6) & 0x3F)),
                                    (uint8_t)(0x80 | (cp & 0x3F))};
            for (int q = 0; q < 3 && k < n; ++q) out[k++] = enc[q];
        } else {
            out[k++] = rng.unit() < 0.9 ? (uint8_t)' ' : kPunct[rng.next() % 6];
        }
    }
    return 0;
}

// filtered copy of in[0..n) into out (capacity n); returns the kept length
extern "C" int64_t o_text_filter(const uint8_t* in, int64_t n, uint8_t* out) {
    int64_t k = 0;
    for (int64_t i = 0; i < n; ++i) {
        const uint8_t c = in[i];
        if (c == 0x00) continue;
        out[k++] = (c == '\r' || c == '\n' || c == '\t') ? (uint8_t)' ' : c;
    }
    return k;
}
