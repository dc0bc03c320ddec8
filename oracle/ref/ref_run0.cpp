// ref_run0.cpp - times the reference Stage 0 / Stage 2 engine (SNNNetwork,
// src/host/network.cpp, and its kernels in src/cuda/, compiled unmodified
// from the reference tree) on one GPU, through its own per-step host API.
//
// Built twice by the recipe in this directory:
//   ref_run0   the Stage 0 build: SNNNetwork::initialize() (its own fixed
//              in-degree topology, src/cuda/network_init.cu), input vector of
//              N_SENSORY floats with 1.5 at the step's byte (the first 256
//              sensory neurons), as configuration 0 states;
//   ref_run2   the Stage 2 build (SNN_STAGE2_BUILD): allocate_only() +
//              init_columnar_synapses (src/stage2/columnar_topology.cu, 10
//              columns x 1,000, 80 intra + 20 inter, seed 123 as
//              src/stage2/main.cpp), input vector of N floats with 5.0 at the
//              step's byte (column 0's first 256 neurons,
//              src/stage2/unsupervised_trainer.cu:96-171).
// Bytes: a seeded xorshift32 uniform stream (seed 42), one per step.
//
//   ref_run0 --steps K --time W
//       W untimed warm-up steps, then K timed steps of SNNNetwork::step
//       (host wall clock, cudaDeviceSynchronize on both sides); then K more
//       untimed steps reading the spike flags back each step to count the
//       events (out-edges of spiking neurons, from the CSR's column indices).
//       Prints REF_STEPS_PER_SEC, REF_EVENTS_PER_STEP, REF_EVENTS_PER_SEC.
//
//   ref_run0 --dump DIR --steps K
//       Pinning fixtures of the reference's own deterministic step (fixed
//       256-wide shared-memory tree in the propagation, one thread per
//       synapse in the STDP): DIR/net.snn2, the freshly initialised network
//       in the reference's SNN2 v1 checkpoint layout
//       (src/stage2/unsupervised_trainer.cu:176-262: header, Synapse records,
//       row_ptr, col_idx, weights); DIR/bytes.bin, the K input bytes;
//       DIR/spikes.txt, one line per step "t count fnv64(spiking indices)";
//       after the K steps DIR/final_V.bin, final_I.bin, final_fr.bin
//       (float[N]), final_off.bin (int8[N] threshold offsets) and
//       final_w.bin (float[S], d_weights in CSR order).
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <string>
#include <cuda_runtime.h>
#include "config.h"
#include "types.h"
#include "network.h"
#ifdef SNN_STAGE2_BUILD
#include "columnar_topology.cuh"
#endif

static uint64_t fnv64(const void* p, size_t n) {
    uint64_t h = 1469598103934665603ull;
    const unsigned char* b = (const unsigned char*)p;
    for (size_t i = 0; i < n; ++i) { h ^= b[i]; h *= 1099511628211ull; }
    return h;
}

static bool write_file(const std::string& path, const void* p, size_t n) {
    FILE* f = fopen(path.c_str(), "wb");
    if (!f) return false;
    const bool ok = fwrite(p, 1, n, f) == n;
    return fclose(f) == 0 && ok;
}

int main(int argc, char** argv) {
    int steps = 1000, warm = 100;
    const char* dump = nullptr;
    for (int i = 1; i < argc; ++i) {
        if (!strcmp(argv[i], "--steps") && i + 1 < argc) steps = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--time") && i + 1 < argc) warm = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--dump") && i + 1 < argc) dump = argv[++i];
    }
    int dev_count = 0;
    if (cudaGetDeviceCount(&dev_count) != cudaSuccess || dev_count == 0) {
        fprintf(stderr, "ref_run0: no CUDA device\n");
        return 2;
    }
    cudaSetDevice(0);
    const int N = N_TOTAL_NEURONS, S = N_TOTAL_SYNAPSES;
#ifdef SNN_STAGE2_BUILD
    SNNNetwork net(123);
    net.allocate_only();
    init_columnar_synapses(net.get_d_synapses(), net.get_d_row_ptr(), net.get_d_col_idx(),
                           net.get_d_weights(), N, 1000, 80, 20, SYNAPSES_PER_NEURON, 123);
    const int in_len = N;
    const float in_val = 5.0f;
#else
    SNNNetwork net(42);
    net.initialize();
    const int in_len = N_SENSORY_NEURONS;
    const float in_val = 1.5f;
#endif
    cudaDeviceSynchronize();
    // out-degree of every pre from the post-major CSR's column indices
    std::vector<int> col((size_t)S);
    cudaMemcpy(col.data(), net.get_d_col_idx(), (size_t)S * 4, cudaMemcpyDeviceToHost);
    std::vector<long long> outdeg((size_t)N, 0);
    for (int x : col)
        if (x >= 0 && x < N) outdeg[x]++;
    std::vector<float> buf((size_t)in_len, 0.0f);
    uint32_t rng = 42u;
    auto next_byte = [&]() {
        rng ^= rng << 13;
        rng ^= rng >> 17;
        rng ^= rng << 5;
        return (int)(rng & 255u);
    };
    int prev = -1;
    auto one_step = [&](int t) {
        if (prev >= 0) buf[prev] = 0.0f;
        prev = next_byte();
        buf[prev] = in_val;
        net.step(buf.data(), t);
    };
    if (dump) {
        const std::string dir(dump);
        std::vector<unsigned char> file;
        auto put = [&](const void* p, size_t n) {
            const unsigned char* b = (const unsigned char*)p;
            file.insert(file.end(), b, b + n);
        };
        const uint32_t magic = 0x534E4E32u, version = 1u;
        const int64_t step0 = 0;
        const uint64_t pos0 = 0;
        const int32_t nn = N, ns = S;
        put(&magic, 4); put(&version, 4); put(&step0, 8); put(&pos0, 8); put(&nn, 4); put(&ns, 4);
        std::vector<Synapse> syn((size_t)S);
        std::vector<int> rp((size_t)N + 1);
        std::vector<float> wts((size_t)S);
        cudaMemcpy(syn.data(), net.get_d_synapses(), (size_t)S * sizeof(Synapse), cudaMemcpyDeviceToHost);
        cudaMemcpy(rp.data(), net.get_d_row_ptr(), ((size_t)N + 1) * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(wts.data(), net.get_d_weights(), (size_t)S * 4, cudaMemcpyDeviceToHost);
        put(syn.data(), (size_t)S * sizeof(Synapse));
        put(rp.data(), ((size_t)N + 1) * 4);
        put(col.data(), (size_t)S * 4);
        put(wts.data(), (size_t)S * 4);
        if (!write_file(dir + "/net.snn2", file.data(), file.size())) {
            fprintf(stderr, "ref_run0: cannot write %s/net.snn2\n", dump);
            return 3;
        }
        std::vector<unsigned char> bytes;
        std::vector<unsigned char> sp((size_t)N);
        std::vector<int> idx;
        FILE* fs = fopen((dir + "/spikes.txt").c_str(), "w");
        if (!fs) return 3;
        for (int t = 0; t < steps; ++t) {
            one_step(t);
            bytes.push_back((unsigned char)prev);
            cudaMemcpy(sp.data(), net.get_d_spikes(), (size_t)N, cudaMemcpyDeviceToHost);
            idx.clear();
            for (int j = 0; j < N; ++j)
                if (sp[j]) idx.push_back(j);
            fprintf(fs, "%d %zu %llu\n", t, idx.size(),
                    (unsigned long long)fnv64(idx.data(), idx.size() * 4));
        }
        fclose(fs);
        std::vector<NeuronState> neu((size_t)N);
        cudaMemcpy(neu.data(), net.get_d_neurons(), (size_t)N * sizeof(NeuronState), cudaMemcpyDeviceToHost);
        cudaMemcpy(wts.data(), net.get_d_weights(), (size_t)S * 4, cudaMemcpyDeviceToHost);
        std::vector<float> V((size_t)N), I((size_t)N), fr((size_t)N);
        std::vector<signed char> off((size_t)N);
        for (int j = 0; j < N; ++j) {
            V[j] = neu[j].membrane_potential;
            I[j] = neu[j].synaptic_current;
            fr[j] = neu[j].fire_rate;
            off[j] = neu[j].threshold_offset;
        }
        const cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess) {
            fprintf(stderr, "ref_run0: %s\n", cudaGetErrorString(err));
            return 5;
        }
        bool ok = write_file(dir + "/bytes.bin", bytes.data(), bytes.size()) &&
                  write_file(dir + "/final_V.bin", V.data(), (size_t)N * 4) &&
                  write_file(dir + "/final_I.bin", I.data(), (size_t)N * 4) &&
                  write_file(dir + "/final_fr.bin", fr.data(), (size_t)N * 4) &&
                  write_file(dir + "/final_off.bin", off.data(), (size_t)N) &&
                  write_file(dir + "/final_w.bin", wts.data(), (size_t)S * 4);
        if (!ok) return 3;
        printf("REF_DUMP %d steps N %d S %d\n", steps, N, S);
        return 0;
    }
    int t = 0;
    for (; t < warm; ++t) one_step(t);
    cudaDeviceSynchronize();
    auto t0 = std::chrono::steady_clock::now();
    for (int k = 0; k < steps; ++k, ++t) one_step(t);
    cudaDeviceSynchronize();
    auto t1 = std::chrono::steady_clock::now();
    const double sec = std::chrono::duration<double>(t1 - t0).count();
    // events of the same number of further steps (untimed: spike flags read back)
    std::vector<unsigned char> sp((size_t)N);
    long long events = 0, spikes = 0;
    for (int k = 0; k < steps; ++k, ++t) {
        one_step(t);
        cudaMemcpy(sp.data(), net.get_d_spikes(), (size_t)N, cudaMemcpyDeviceToHost);
        for (int j = 0; j < N; ++j)
            if (sp[j]) { events += outdeg[j]; spikes++; }
    }
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        fprintf(stderr, "ref_run0: %s\n", cudaGetErrorString(err));
        return 5;
    }
    printf("REF_STEPS_PER_SEC %.3f\n", steps / sec);
    printf("REF_EVENTS_PER_STEP %.3f\n", (double)events / steps);
    printf("REF_SPIKES_PER_STEP %.3f\n", (double)spikes / steps);
    printf("REF_EVENTS_PER_SEC %.3f\n", (double)events / steps * (steps / sec));
    printf("REF_TIMED_STEPS %d REF_SECONDS %.6f\n", steps, sec);
    return 0;
}
