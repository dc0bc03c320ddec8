"""Long-run statistical parity with the reference itself: the reference's
Stage 2e scheduler (compiled unmodified from its sources into
oracle/_ref/ref_run by oracle/ref/Makefile) and this library's engine run the
reference network for 20,000 steps (15,000 of them with plasticity) on the
same synthetic byte stream, on a B200.  Their spike rasters part ways after a
few hundred steps (CUDA expf and float-atomic order in the reference), so the
bar is statistical: per-layer firing rates, fire-rate traces, the excitatory
weight distribution and the columns' mean Jensen-Shannon divergence (js_mean)
within 2 %.  Skipped where the reference binary was not built."""
import os
import subprocess

import numpy as np
import pytest

import longrun_stats as ls
import snn_b200 as snn

HERE = os.path.dirname(os.path.abspath(__file__))
REF_RUN = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "ref_run")
STEPS = 20000


@pytest.mark.gpu
@pytest.mark.skipif(not os.path.exists(REF_RUN), reason="reference binary not built")
def test_long_run_statistics_match_the_reference(tmp_path):
    corpus = snn.stream(200000, seed=7)
    corpus.tofile(tmp_path / "corpus.bin")
    r = subprocess.run([REF_RUN, "--steps", str(STEPS), "--corpus", str(tmp_path / "corpus.bin"),
                        "--stats", str(tmp_path / "ref.bin")], capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    k, counts, fr, alpha, beta, flags, nbc = ls.read_reference_stats(str(tmp_path / "ref.bin"))
    assert k == STEPS
    ref = ls.summarize(counts, fr, alpha, beta, flags, nbc, k)

    net = snn.Network(raster_steps=1000)
    net.build_columns(snn.topology(n_columns=50))
    net.set_corpus(corpus)
    mine = np.zeros(net.N, np.int64)
    for _ in range(STEPS // 1000):
        ras, _ = net.run(1000, raster=True)
        bits = np.unpackbits(ras.view(np.uint8), axis=1, bitorder="little")[:, : net.N]
        mine += bits.sum(axis=0).astype(np.int64)
    ours = ls.summarize(mine, net.state("fr"), net.state("alpha"), net.state("beta"),
                        net.state("flags"), net.state("neuron_byte_counts"), STEPS)
    net.close()

    assert ref["rate_all"] > 0.005 and ref["js_mean"] > 0.05  # an active, learning run
    for key, want in ref.items():
        got = ours[key]
        if key == "w_hist":
            tv = 0.5 * np.abs(got - want).sum()
            assert tv < 0.02, f"weight histogram: total variation {tv:.4f}"
        elif want == 0:
            assert got == 0, key
        else:
            rel = abs(got - want) / abs(want)
            assert rel < 0.02, f"{key}: ours {got:.6g} reference {want:.6g} ({100 * rel:.2f} %)"
