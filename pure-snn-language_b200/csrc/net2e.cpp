// net2e.cpp - Stage 2e network generator (reference rules) and the
// group / post-major layout used by the CUDA kernels.  Host C++ only.
#include "net2e.h"
#include <algorithm>
#include <cmath>
#include "snn_pmath.h"

namespace snn2e {

namespace {
struct XorShift32 {  // src/stage2e/network_init.cu:167-179
    uint32_t s;
    uint32_t next() {
        s ^= s << 13;
        s ^= s >> 17;
        s ^= s << 5;
        return s;
    }
    float uniform(float lo, float hi) {  // lo + (hi-lo) * (r / 2^32), in float
        float r = pm_div(pm_u2f(next()), 4294967296.0f);
        return pm_add(lo, pm_mul(pm_sub(hi, lo), r));
    }
    int range(int lo, int hi) { return lo + (int)(next() % (uint32_t)(hi - lo)); }
};
}  // namespace

Shard make_shard(const snn_topology_spec& sp, int rank, int world) {
    SNN_REQUIRE(world >= 1 && rank >= 0 && rank < world, SNN_ERR_ARG, "bad shard rank / world");
    SNN_REQUIRE(sp.n_columns >= world && sp.pf_groups >= world, SNN_ERR_ARG,
                "fewer columns or prefrontal groups than shards");
    const int NPC = sp.l4 + sp.l23 + sp.l5 + sp.l6;
    const int NA = sp.n_columns * NPC;
    Shard h;
    h.rank = rank;
    h.world = world;
    h.c0 = (int)((int64_t)sp.n_columns * rank / world);
    h.c1 = (int)((int64_t)sp.n_columns * (rank + 1) / world);
    h.p0 = (int)((int64_t)sp.pf_groups * rank / world);
    h.p1 = (int)((int64_t)sp.pf_groups * (rank + 1) / world);
    h.a0 = h.c0 * NPC;
    h.a1 = h.c1 * NPC;
    h.pf0 = NA + h.p0 * sp.pf_group_size;
    h.pf1 = NA + h.p1 * sp.pf_group_size;
    return h;
}

void generate_reference(const snn_topology_spec& sp, HostNet& n, const Shard* shard) {
    SNN_REQUIRE(sp.n_columns >= 2 && sp.l4 > 0 && sp.l23 > 0 && sp.l5 > 0 && sp.l6 > 0 &&
                    sp.pf_groups > 0 && sp.pf_group_size > 0,
                SNN_ERR_ARG, "stage2e topology: need >= 2 columns and non-empty layers");
    n.ncol = sp.n_columns;
    n.l4 = sp.l4; n.l23 = sp.l23; n.l5 = sp.l5; n.l6 = sp.l6;
    n.NPC = sp.l4 + sp.l23 + sp.l5 + sp.l6;
    n.N_assoc = n.ncol * n.NPC;
    n.pf_groups = sp.pf_groups;
    n.pf_size = sp.pf_group_size;
    const int N_pf = sp.pf_groups * sp.pf_group_size;
    n.N = n.N_assoc + N_pf;
    const int N = n.N, NPC = n.NPC, NA = n.N_assoc;
    const int lbase[4] = {0, sp.l4, sp.l4 + sp.l23, sp.l4 + sp.l23 + sp.l5};
    const int lsize[4] = {sp.l4, sp.l23, sp.l5, sp.l6};
    auto layer_of = [&](int off) -> int {
        return off < lbase[1] ? L4 : off < lbase[2] ? L23 : off < lbase[3] ? L5 : L6;
    };

    // neurons (src/stage2e/network_init.cu:38-127)
    n.type.assign(N, 0); n.region.assign(N, 0); n.subtype.assign(N, 0); n.column.assign(N, -1);
    for (int i = 0; i < N; ++i) {
        if (i < NA) {
            int off = i % NPC, L = layer_of(off);
            int lo = off - lbase[L], ls = lsize[L];
            n.column[i] = i / NPC;
            n.region[i] = (uint8_t)L;
            int exc = (int)pm_mul(pm_i2f(ls), 0.8f);
            if (lo >= exc) {
                n.type[i] = 1;
                float frac = pm_div(pm_i2f(lo - exc), pm_i2f(ls - exc));
                n.subtype[i] = frac < 0.5f ? 1 : (frac < pm_add(0.5f, 0.3f) ? 2 : 3);
            }
        } else {
            n.region[i] = PF;
            int og = (i - NA) % sp.pf_group_size;
            if (og >= (int)pm_mul(pm_i2f(sp.pf_group_size), 0.8f)) { n.type[i] = 1; n.subtype[i] = 1; }
        }
    }

    // out-degrees and top-up (src/stage2e/network_init.cu:194-239)
    XorShift32 rng{sp.seed};
    std::vector<int32_t> deg(N);
    int64_t total = 0;
    for (int i = 0; i < N; ++i) {
        int d;
        if (i < NA) {
            int L = layer_of(i % NPC);
            d = sp.deg_intra + (L == L23 ? sp.deg_inter : 0) + (L == L5 ? sp.deg_l5_pf : 0);
        } else {
            d = sp.deg_pf_self + sp.deg_pf_assoc;
        }
        deg[i] = d;
        total += d;
    }
    while (total < sp.total_synapses) { deg[rng.range(0, NA)]++; total++; }
    while (total > sp.total_synapses) {
        int i = rng.range(0, NA);
        if (deg[i] > 50) { deg[i]--; total--; }
    }
    SNN_REQUIRE(total < (int64_t)INT32_MAX, SNN_ERR_ARG, "synapse count exceeds int32 indexing");
    // generated rows: the reference's row pointer over all synapses
    std::vector<int64_t> gen_ptr(N + 1, 0);
    for (int i = 0; i < N; ++i) gen_ptr[i + 1] = gen_ptr[i] + deg[i];
    const bool filter = shard && shard->world > 1;
    const size_t cap = filter ? (size_t)(total / shard->world + total / (4 * shard->world) + 4096)
                              : (size_t)total;
    n.row_ptr.assign(N + 1, 0);
    n.post.clear(); n.delay.clear(); n.flags.clear();
    n.w0.clear(); n.alpha.clear(); n.beta.clear(); n.u0.clear();
    n.post.reserve(cap);
    n.delay.reserve(cap); n.flags.reserve(cap);
    n.w0.reserve(cap); n.alpha.reserve(cap); n.beta.reserve(cap); n.u0.reserve(cap);

    const float w_scale = pm_div(2.0f, sqrtf(200.0f));
    auto put = [&](int64_t, int post, float w, int d, bool exc, bool ff) {
        if (filter && !shard->owns(post)) return;
        n.post.push_back(post);
        n.delay.push_back((uint8_t)d);
        n.w0.push_back(w);
        uint8_t f = exc ? (RF_AMPA | RF_NMDA) : (RF_GABA_A | RF_GABA_B);
        if (ff) f |= RF_FF;
        n.flags.push_back(f);
        n.u0.push_back(ff ? 0.02f : (exc ? 0.2f : 0.05f));
        float r = pm_div(fabsf(w), 1.5f);
        if (r > 0.999f) r = 0.999f;
        n.alpha.push_back(pm_mul(r, 0.1f));
        n.beta.push_back(pm_mul(pm_sub(1.0f, r), 0.1f));
    };
    // flow rules L4->L2/3, L2/3->{L2/3,L5}, L5->{L6,L2/3}, L6->{L4,L6}
    auto target_layer = [&](int L) -> int {
        switch (L) {
            case L4: return L23;
            case L23: return (rng.next() & 1) ? L23 : L5;
            case L5: return (rng.next() & 1) ? L6 : L23;
            default: return (rng.next() & 1) ? L4 : L6;
        }
    };
    for (int pre = 0; pre < N; ++pre) {
        int64_t k = gen_ptr[pre];
        const int64_t kend = gen_ptr[pre + 1];
        const bool pf = pre >= NA;
        const int col = pf ? -1 : pre / NPC;
        const int L = pf ? (int)PF : layer_of(pre % NPC);
        const bool exc = n.type[pre] == 0;
        auto intra = [&](bool any_pf) {
            int post;
            bool ff = false;
            if (pf) {
                if (any_pf) post = NA + rng.range(0, N_pf);
                else post = NA + ((pre - NA) / sp.pf_group_size) * sp.pf_group_size +
                            rng.range(0, sp.pf_group_size);
            } else {
                int T = target_layer(L);
                post = col * NPC + lbase[T] + rng.range(0, lsize[T]);
                ff = (L == L4 && T == L23) || (L == L23 && T == L5) || (L == L5 && T == L6);
            }
            if (post == pre) post = (post + 1) % N;
            float lo = ff ? 2.5f : 0.4f, hi = ff ? 3.5f : 1.0f;
            float w = exc ? pm_mul(rng.uniform(lo, hi), w_scale) : pm_mul(rng.uniform(-hi, -lo), w_scale);
            int d = rng.range(1, 4);
            put(k++, post, w, d, exc, ff);
        };
        const int n_intra = pf ? sp.deg_pf_self : sp.deg_intra;
        const int n_inter = (L == L23) ? sp.deg_inter : 0;
        const int n_pf = pf ? sp.deg_pf_assoc : (L == L5 ? sp.deg_l5_pf : 0);
        for (int j = 0; j < n_intra && k < kend; ++j) intra(false);
        for (int j = 0; j < n_inter && k < kend; ++j) {
            int tc = rng.range(0, sp.n_columns);
            if (tc == col) tc = (tc + 1) % sp.n_columns;
            int post = tc * NPC + lbase[L23] + rng.range(0, sp.l23);
            float w = exc ? pm_mul(rng.uniform(0.05f, 0.15f), w_scale)
                          : pm_mul(rng.uniform(-0.15f, -0.05f), w_scale);
            int d = rng.range(5, 11);
            put(k++, post, w, d, exc, false);
        }
        for (int j = 0; j < n_pf && k < kend; ++j) {
            int post;
            if (pf) post = rng.range(0, NA);
            else {
                int g = rng.range(0, sp.pf_groups);
                post = NA + g * sp.pf_group_size + rng.range(0, sp.pf_group_size);
            }
            int d = rng.range(15, 21);
            float w = exc ? pm_mul(rng.uniform(0.6f, 1.2f), w_scale)
                          : pm_mul(rng.uniform(-1.2f, -0.6f), w_scale);
            put(k++, post, w, d, exc, false);
        }
        while (k < kend) intra(true);
        n.row_ptr[pre + 1] = (int32_t)n.post.size();
    }
    n.S = (int64_t)n.post.size();
}

void build_layout(const HostNet& net, Layout& lay) {
    const int N = net.N;
    const int64_t S = net.S;
    // groups: keys (d_eff, ff) per pre, ascending
    lay.gbeg.assign(N + 1, 0);
    std::vector<uint32_t> gid(S);
    lay.gmeta.clear(); lay.gsize.clear(); lay.gu0.clear(); lay.gpre.clear();
    for (int pre = 0; pre < N; ++pre) {
        int slot[40];
        for (int q = 0; q < 40; ++q) slot[q] = -1;
        const int64_t b = net.row_ptr[pre], e = net.row_ptr[pre + 1];
        for (int64_t s = b; s < e; ++s) {
            int key = eff_delay(net.delay[s]) * 2 + ((net.flags[s] & RF_FF) ? 1 : 0);
            slot[key] = 0;
        }
        lay.gbeg[pre] = (int32_t)lay.gmeta.size();
        for (int key = 0; key < 40; ++key) {
            if (slot[key] < 0) continue;
            slot[key] = (int)lay.gmeta.size();
            uint32_t exc = net.type[pre] == 0 ? 1u : 0u;
            lay.gmeta.push_back((uint32_t)(key >> 1) | ((uint32_t)(key & 1) << 5) | (exc << 6));
            lay.gsize.push_back(0);
            float u0 = (key & 1) ? 0.02f : (exc ? 0.2f : 0.05f);
            lay.gu0.push_back(u0);
            lay.gpre.push_back(pre);
        }
        for (int64_t s = b; s < e; ++s) {
            int key = eff_delay(net.delay[s]) * 2 + ((net.flags[s] & RF_FF) ? 1 : 0);
            gid[s] = (uint32_t)slot[key];
            lay.gsize[slot[key]]++;
        }
    }
    lay.gbeg[N] = (int32_t)lay.gmeta.size();
    lay.G = (int64_t)lay.gmeta.size();
    SNN_REQUIRE(lay.G < (1ll << 30), SNN_ERR_ARG, "too many synapse groups for 30-bit ids");
    // post-major permutation, stable in synapse id
    lay.in_ptr.assign(N + 1, 0);
    for (int64_t s = 0; s < S; ++s) lay.in_ptr[net.post[s] + 1]++;
    for (int i = 0; i < N; ++i) lay.in_ptr[i + 1] += lay.in_ptr[i];
    lay.perm.resize(S);
    lay.gid_pm.resize(S);
    std::vector<int32_t> fill(lay.in_ptr.begin(), lay.in_ptr.end() - 1);
    for (int64_t s = 0; s < S; ++s) {
        int32_t p = fill[net.post[s]]++;
        lay.perm[p] = (int32_t)s;
        const uint32_t meta = lay.gmeta[gid[s]];
        lay.gid_pm[p] = gid[s] | (((meta >> 5) & 1u) << 30) | (((meta >> 6) & 1u) << 31);
    }
}

}  // namespace snn2e
