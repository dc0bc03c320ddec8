// net2e.h - host-side Stage 2e network: generator output and device layout.
#pragma once
#include <cstdint>
#include <vector>
#include "common.h"

namespace snn2e {

enum : uint8_t { L4 = 0, L23 = 1, L5 = 2, L6 = 3, PF = 4 };
enum : uint8_t { RF_AMPA = 0x01, RF_NMDA = 0x02, RF_GABA_A = 0x04, RF_GABA_B = 0x08, RF_FF = 0x10 };

// Pre-major network as the reference generator produces it.
struct HostNet {
    int32_t N = 0, N_assoc = 0, NPC = 0, ncol = 0, l4 = 0, l23 = 0, l5 = 0, l6 = 0;
    int32_t pf_groups = 0, pf_size = 0;
    int64_t S = 0;
    std::vector<int32_t> row_ptr;  // N+1
    std::vector<int32_t> post;     // S
    std::vector<uint8_t> delay;    // S, raw delay steps
    std::vector<uint8_t> flags;    // S, receptor flags
    std::vector<float> w0, alpha, beta, u0;  // S
    // per neuron: type (0 exc / 1 inh), region (REGION), subtype, column (-1 = PF)
    std::vector<uint8_t> type, region, subtype;
    std::vector<int32_t> column;
};

// Column sharding: rank r of `world` owns the columns [c0, c1) and the
// prefrontal groups [p0, p1) (even split), i.e. the neurons [a0, a1) and
// [pf0, pf1); its local neuron order is the first range, then the second.
struct Shard {
    int rank = 0, world = 1;
    int c0 = 0, c1 = 0, p0 = 0, p1 = 0;
    int a0 = 0, a1 = 0, pf0 = 0, pf1 = 0;
    int n_local() const { return (a1 - a0) + (pf1 - pf0); }
    bool owns(int g) const { return (g >= a0 && g < a1) || (g >= pf0 && g < pf1); }
    int local_of(int g) const { return g < a1 ? g - a0 : (a1 - a0) + (g - pf0); }
    int global_of(int j) const { return j < a1 - a0 ? a0 + j : pf0 + (j - (a1 - a0)); }
};
Shard make_shard(const snn_topology_spec& spec, int rank, int world);

// Reference rules (src/stage2e/network_init.cu:38-127, 158-473).  With a
// shard, the full random sequence is drawn but only the synapses onto the
// shard's neurons are kept (in generation order, so that the canonical
// ascending-id order of every kept neuron's incoming list is unchanged);
// row_ptr then spans all N pres over the kept synapses.
void generate_reference(const snn_topology_spec& spec, HostNet& net, const Shard* shard = nullptr);

// Group / post-major layout.
//   group  = distinct (pre, effective delay, feed-forward flag) of a pre's
//            out-synapses; STP resources, utilisation, NMDA conductance and
//            the pre trace of every synapse in a group stay identical.
//   post-major order = incoming synapses of each neuron in ascending
//            reference synapse id (the canonical accumulation order).
struct Layout {
    int64_t G = 0;
    std::vector<int32_t> gbeg;     // N+1, groups of pre i are [gbeg[i], gbeg[i+1])
    std::vector<uint32_t> gmeta;   // G: d_eff | ff<<5 | exc<<6
    std::vector<int32_t> gsize;    // G: synapses in the group
    std::vector<float> gu0;        // G: initial utilisation
    std::vector<int32_t> gpre;     // G: pre-synaptic neuron of the group
    std::vector<int32_t> in_ptr;   // N+1
    std::vector<int32_t> perm;     // S: post-major position -> reference synapse id
    std::vector<uint32_t> gid_pm;  // S: group of each post-major synapse | FF << 30 | EXC << 31
};
void build_layout(const HostNet& net, Layout& lay);

inline int eff_delay(int d) { return d < 1 ? 1 : (d >= 20 ? 19 : d); }

}  // namespace snn2e
