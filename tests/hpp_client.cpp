// A caller of the header-only C++ API (include/snn_b200.hpp), written the way
// a user of the reference's host classes would: stage2e::BioMechanismScheduler
// stepped with step(t), and SNNNetwork with initialize / step / save_weights /
// load_weights.  Built and run by tests/test_cpp_header.py.
//
//   hpp_client nogpu            construction must throw SnnException(7)
//   hpp_client gpu DIR          runs both classes, prints key=value lines
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "snn_b200.hpp"

static int no_gpu() {
    try {
        snnb::stage2e::BioMechanismScheduler s(50);
        std::printf("constructed\n");
        return 1;
    } catch (const snnb::SnnException& e) {
        std::printf("scheduler_code=%d\n", e.code);
    }
    try {
        snnb::SNNNetwork n(42);
        std::printf("constructed\n");
        return 1;
    } catch (const snnb::SnnException& e) {
        std::printf("network_code=%d\n", e.code);
    }
    return 0;
}

static int gpu(const std::string& dir) {
    snnb::stage2e::BioMechanismScheduler s(50);
    const char* text = "The quick brown fox\r\njumps\tover the lazy dog.";
    std::vector<uint8_t> corpus(text, text + std::strlen(text));
    corpus.push_back(0x00);  // dropped by load_text_corpus
    std::printf("corpus_bytes=%zu\n", s.load_text_corpus(corpus));
    for (int t = 0; t < 40; ++t) s.step(t);
    s.run(24);
    std::printf("steps=%d\n", s.total_steps_executed());
    std::printf("spikes=%lld\n", s.total_spikes_accum());
    std::printf("arrived=%lld\n", s.arrived_events_accum());
    std::printf("dispatched=%lld\n", s.dispatched_events_accum());
    std::vector<float> w = s.state<float>(SNN_STATE_WEIGHT, (size_t)s.counters().n_synapses);
    if (FILE* f = std::fopen((dir + "/weights2e.f32").c_str(), "wb")) {
        std::fwrite(w.data(), sizeof(float), w.size(), f);
        std::fclose(f);
    }
    std::printf("ckpt_rc=%d\n", s.save_checkpoint(64, dir.c_str()));
    // a directory that does not exist: 2, no exception (the reference prints and returns)
    std::printf("ckpt_bad_rc=%d\n", s.save_checkpoint(64, (dir + "/missing/sub").c_str()));

    snnb::SNNNetwork net(42);
    net.initialize();
    std::printf("n_neurons=%d\n", net.n_neurons());
    for (int t = 0; t < 30; ++t) net.step(t % 3 == 0 ? 'a' + t % 26 : -1, t);
    net.set_dopamine(0.5f);
    for (int t = 30; t < 60; ++t) net.step(-1, t);
    const std::string wpath = dir + "/weights.bin";
    net.save_weights(wpath);
    net.load_weights(wpath);
    try {
        net.load_weights(dir + "/no_such_file.bin");
        std::printf("load_missing=ok\n");
    } catch (const snnb::SnnException& e) {
        std::printf("load_missing_code=%d\n", e.code);
    }
    snn_counters c;
    if (snn_get_counters(net.handle(), &c) != SNN_OK) return 3;
    std::printf("s0_spikes=%lld\n", (long long)c.total_spikes);
    return 0;
}

int main(int argc, char** argv) {
    if (argc >= 2 && std::strcmp(argv[1], "nogpu") == 0) return no_gpu();
    if (argc >= 3 && std::strcmp(argv[1], "gpu") == 0) {
        try {
            return gpu(argv[2]);
        } catch (const snnb::SnnException& e) {
            std::printf("error code=%d %s\n", e.code, e.what());
            return 4;
        }
    }
    std::fprintf(stderr, "usage: hpp_client nogpu | gpu DIR\n");
    return 2;
}
