// topo_pin.cpp - runs the reference's own host-side Stage 2e topology
// generator (stage2e::init_synapses_host, src/stage2e/network_init.cu:158-473,
// compiled unmodified from the reference tree) and prints FNV-1a 64 hashes of
// every array it produces.  No GPU is touched.  Used to pin the oracle's
// generator: tests compare these hashes with the oracle's arrays.
#include <cstdio>
#include <cstdint>
#include <vector>
#include "types.h"   // reference BioSynapse layout (src/stage2e/types.h)

namespace stage2e {
void init_synapses_host(std::vector<BioSynapse>& h_synapses, std::vector<int>& h_row_ptr,
                        std::vector<int>& h_col_idx, std::vector<float>& h_weights_cache,
                        std::vector<uint8_t>& h_delay, std::vector<float>& h_alpha,
                        std::vector<float>& h_beta);
}

static uint64_t fnv(const void* p, size_t n, uint64_t h = 1469598103934665603ull) {
    const unsigned char* b = (const unsigned char*)p;
    for (size_t i = 0; i < n; ++i) { h ^= b[i]; h *= 1099511628211ull; }
    return h;
}

int main() {
    std::vector<BioSynapse> syn; std::vector<int> row, col; std::vector<float> w, a, b;
    std::vector<uint8_t> d;
    stage2e::init_synapses_host(syn, row, col, w, d, a, b);
    std::vector<uint8_t> flags(syn.size()); std::vector<float> u(syn.size());
    std::vector<int> post(syn.size());
    for (size_t i = 0; i < syn.size(); ++i) { flags[i] = syn[i].receptor_flags; u[i] = syn[i].utilization; post[i] = syn[i].post_idx; }
    printf("n_synapses %zu\n", syn.size());
    printf("row_ptr %016llx\n", (unsigned long long)fnv(row.data(), row.size() * 4));
    printf("col_idx %016llx\n", (unsigned long long)fnv(col.data(), col.size() * 4));
    printf("post %016llx\n", (unsigned long long)fnv(post.data(), post.size() * 4));
    printf("weights %016llx\n", (unsigned long long)fnv(w.data(), w.size() * 4));
    printf("delay %016llx\n", (unsigned long long)fnv(d.data(), d.size()));
    printf("alpha %016llx\n", (unsigned long long)fnv(a.data(), a.size() * 4));
    printf("beta %016llx\n", (unsigned long long)fnv(b.data(), b.size() * 4));
    printf("flags %016llx\n", (unsigned long long)fnv(flags.data(), flags.size()));
    printf("utilization %016llx\n", (unsigned long long)fnv(u.data(), u.size() * 4));
    printf("sample");
    for (size_t i = 0; i < syn.size(); i += syn.size() / 7) printf(" %zu:%d:%d:%.9g:%d", i, syn[i].pre_idx, syn[i].post_idx, syn[i].weight, (int)d[i]);
    printf("\n");
    return 0;
}
