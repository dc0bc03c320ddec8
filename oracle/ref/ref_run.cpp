// ref_run.cpp - drives the reference Stage 2e engine (stage2e::MemoryAllocator,
// stage2e::init_network, stage2e::BioMechanismScheduler, compiled unmodified
// from the reference tree) on one GPU.
//
// Modes:
//   ref_run --steps K [--corpus F] --dump OUT.txt [--state OUT.bin]
//       after every step: "step count fnv64(spiking indices)" to OUT.txt; at
//       the end, V / w / fire-rate of every neuron and the summed alpha/beta
//       to OUT.bin.  Used to pin the CPU oracle against the reference itself.
//   ref_run --steps K [--corpus F] --stats OUT.bin
//       K steps, then i32 N, i32 S, i32 K, per-neuron spike counts over the
//       run (i32[N]), fire rates (f32[N]), alpha (f32[S]), beta (f32[S]),
//       receptor flags (u8[S]) and the neuron x byte counts (i32[N*256]):
//       the long-run statistics the tests compare with this library's engine.
//   ref_run --steps K [--corpus F] --time W [--step0 T0]
//       W untimed warm-up steps, then K timed steps of the reference's own
//       host loop (src/stage2e/main.cpp:679-743, without CSV); prints
//       REF_STEPS_PER_SEC and REF_EVENTS_PER_SEC.  The scheduler is given
//       the step numbers T0, T0 + 1, ... (default 0): its phase table is a
//       function of the step number, so T0 = 5010 runs a fresh network in
//       the SYNAPTOGENIC phase with the injection (t % 3) and the 10-step
//       schedules aligned with steps 0, 1, ... of a network whose phase is
//       offset by 5000.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cstdint>
#include <chrono>
#include <vector>
#include <cuda_runtime.h>
#include "config.h"
#include "types.h"
#include "memory_allocator.cuh"
#include "network_init.cuh"
#include "input_encoding.cuh"
#include "scheduler.cuh"

static uint64_t fnv(const void* p, size_t n, uint64_t h = 1469598103934665603ull) {
    const unsigned char* b = (const unsigned char*)p;
    for (size_t i = 0; i < n; ++i) { h ^= b[i]; h *= 1099511628211ull; }
    return h;
}

int main(int argc, char** argv) {
    int steps = 100, warm = -1, step0 = 0;
    const char* corpus = nullptr;
    const char* dump = nullptr;
    const char* state = nullptr;
    const char* stats = nullptr;
    for (int i = 1; i < argc; ++i) {
        if (!strcmp(argv[i], "--steps") && i + 1 < argc) steps = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--corpus") && i + 1 < argc) corpus = argv[++i];
        else if (!strcmp(argv[i], "--dump") && i + 1 < argc) dump = argv[++i];
        else if (!strcmp(argv[i], "--state") && i + 1 < argc) state = argv[++i];
        else if (!strcmp(argv[i], "--stats") && i + 1 < argc) stats = argv[++i];
        else if (!strcmp(argv[i], "--time") && i + 1 < argc) warm = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--step0") && i + 1 < argc) step0 = atoi(argv[++i]);
    }
    int dev_count = 0;
    if (cudaGetDeviceCount(&dev_count) != cudaSuccess || dev_count == 0) {
        fprintf(stderr, "ref_run: no CUDA device\n");
        return 2;
    }
    cudaSetDevice(0);
    stage2e::MemoryAllocator alloc;
    if (alloc.allocate_all() == 0) { fprintf(stderr, "ref_run: allocation failed\n"); return 3; }
    stage2e::init_network(&alloc);
    if (corpus && stage2e::load_text_corpus(corpus) == 0) {
        fprintf(stderr, "ref_run: cannot load corpus %s\n", corpus);
        return 4;
    }
    stage2e::BioMechanismScheduler sched(&alloc);
    const int N = N_TOTAL_NEURONS_2E;
    if (warm >= 0) {
        for (int s = 0; s < warm; ++s) sched.step(step0 + s);
        cudaDeviceSynchronize();
        long long arr0 = sched.arrived_events_accum();
        auto t0 = std::chrono::steady_clock::now();
        for (int s = warm; s < warm + steps; ++s) sched.step(step0 + s);
        cudaDeviceSynchronize();
        auto t1 = std::chrono::steady_clock::now();
        double sec = std::chrono::duration<double>(t1 - t0).count();
        long long arr = sched.arrived_events_accum() - arr0;
        printf("REF_STEPS_PER_SEC %.3f\n", steps / sec);
        printf("REF_EVENTS_PER_SEC %.3f\n", arr / sec);
        printf("REF_TIMED_STEPS %d REF_SECONDS %.6f REF_ARRIVALS %lld\n", steps, sec, arr);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? 0 : 5;
    }
    FILE* f = dump ? fopen(dump, "w") : nullptr;
    std::vector<uint8_t> flags(N);
    std::vector<int32_t> idx;
    std::vector<int32_t> counts(stats ? N : 0, 0);
    for (int s = 0; s < steps; ++s) {
        sched.step(s);
        if (stats) {
            cudaMemcpy(flags.data(), alloc.buffers().d_spike_flags, N, cudaMemcpyDeviceToHost);
            for (int i = 0; i < N; ++i) counts[i] += flags[i] ? 1 : 0;
        }
        if (f) {
            cudaMemcpy(flags.data(), alloc.buffers().d_spike_flags, N, cudaMemcpyDeviceToHost);
            idx.clear();
            for (int i = 0; i < N; ++i) if (flags[i]) idx.push_back(i);
            fprintf(f, "%d %zu %016llx\n", s, idx.size(),
                    (unsigned long long)fnv(idx.data(), idx.size() * 4));
        }
    }
    if (f) fclose(f);
    if (state) {
        std::vector<NeuronStateAdEx> h(N);
        cudaMemcpy(h.data(), alloc.buffers().d_neurons, N * sizeof(NeuronStateAdEx),
                   cudaMemcpyDeviceToHost);
        std::vector<float> out(3 * (size_t)N);
        for (int i = 0; i < N; ++i) {
            out[i] = h[i].membrane_potential;
            out[N + i] = h[i].adaptive_conductance;
            out[2 * N + i] = h[i].fire_rate;
        }
        std::vector<float> a(N_TOTAL_SYNAPSES_2E), b(N_TOTAL_SYNAPSES_2E);
        cudaMemcpy(a.data(), alloc.buffers().d_synapse_alpha, a.size() * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(b.data(), alloc.buffers().d_synapse_beta, b.size() * 4, cudaMemcpyDeviceToHost);
        double sa = 0, sb = 0;
        for (size_t i = 0; i < a.size(); ++i) { sa += a[i]; sb += b[i]; }
        FILE* g = fopen(state, "wb");
        if (g) {
            fwrite(out.data(), 4, out.size(), g);
            fwrite(&sa, 8, 1, g);
            fwrite(&sb, 8, 1, g);
            fclose(g);
        }
    }
    if (stats) {
        const int S = N_TOTAL_SYNAPSES_2E;
        std::vector<NeuronStateAdEx> h(N);
        cudaMemcpy(h.data(), alloc.buffers().d_neurons, N * sizeof(NeuronStateAdEx), cudaMemcpyDeviceToHost);
        std::vector<float> fr(N), a(S), b(S);
        for (int i = 0; i < N; ++i) fr[i] = h[i].fire_rate;
        cudaMemcpy(a.data(), alloc.buffers().d_synapse_alpha, (size_t)S * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(b.data(), alloc.buffers().d_synapse_beta, (size_t)S * 4, cudaMemcpyDeviceToHost);
        std::vector<BioSynapse> syn(S);
        cudaMemcpy(syn.data(), alloc.buffers().d_synapses, (size_t)S * sizeof(BioSynapse), cudaMemcpyDeviceToHost);
        std::vector<uint8_t> rf(S);
        for (int q = 0; q < S; ++q) rf[q] = syn[q].receptor_flags;
        std::vector<int32_t> nbc((size_t)N * 256);
        cudaMemcpy(nbc.data(), alloc.buffers().d_neuron_byte_counts, nbc.size() * 4, cudaMemcpyDeviceToHost);
        FILE* g = fopen(stats, "wb");
        if (!g) { fprintf(stderr, "ref_run: cannot write %s\n", stats); return 7; }
        const int32_t hdr[3] = {N, S, steps};
        fwrite(hdr, 4, 3, g);
        fwrite(counts.data(), 4, N, g);
        fwrite(fr.data(), 4, N, g);
        fwrite(a.data(), 4, S, g);
        fwrite(b.data(), 4, S, g);
        fwrite(rf.data(), 1, S, g);
        fwrite(nbc.data(), 4, nbc.size(), g);
        fclose(g);
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { fprintf(stderr, "ref_run: %s\n", cudaGetErrorString(e)); return 6; }
    printf("REF_RUN_OK steps=%d total_spikes=%d arrived=%lld dropped=%lld\n", steps,
           sched.total_spikes_accum(), sched.arrived_events_accum(), sched.dropped_events_accum());
    return 0;
}
