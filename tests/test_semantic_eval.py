"""Semantic evaluation of the Stage 2e network (snn_semantic_eval, the
reference's BioMechanismScheduler::run_semantic_eval): the library's device
reductions + host arithmetic against the oracle's restatement
(pyoracle.semantic_eval) on the same counts, and the restatement itself
against closed-form cases and an independent JS implementation."""
import math

import numpy as np
import pytest

import pyoracle as po
from longrun_stats import column_js_mean

NCOL, NPC = 8, 1000


def regions(n_columns, n_total, sizes=(200, 350, 200, 250)):
    off = np.arange(n_columns * NPC) % NPC
    bounds = np.cumsum(sizes)
    reg = np.searchsorted(bounds, off, side="right").astype(np.uint8)
    return np.concatenate([reg, np.full(n_total - n_columns * NPC, 4, np.uint8)])


def test_restatement_closed_forms():
    n = 2 * NPC
    nbc = np.zeros((n, 256), np.int32)
    nbc[:NPC, :128] = 1        # column 0 answers bytes 0..127 only
    nbc[NPC:, 128:] = 1        # column 1 answers bytes 128..255 only
    last = np.full(n, -1, np.int32)
    r = po.semantic_eval(nbc, last, regions(2, n), 2, NPC, 10)
    assert abs(r["js_mean"] - math.log(2.0)) < 1e-12 and r["js_max"] == r["js_mean"]
    assert r["column_ratio"] == 1.0 and r["nonzero_columns"] == 2
    assert r["layer_delay"] == [-1.0] * 5 and r["layer_delay_n"] == [0] * 5
    # every row has 128 spikes on half the bytes: chi2 = 256 * 128 / 256 ... per row
    # (observed 1 on 128 bytes, 0 on the rest, expected 0.5): 256 * 0.25 / 0.5 = 128
    assert r["layer_act"][:4] == [400, 700, 400, 500]
    assert all(abs(x - 128.0) < 1e-6 for x in r["layer_chi2_mean"][:4])
    same = np.ones((n, 256), np.int32)
    assert po.semantic_eval(same, last, regions(2, n), 2, NPC, 10)["js_mean"] == 0.0


def test_restatement_matches_an_independent_js():
    rng = np.random.default_rng(3)
    n = 6 * NPC + 300
    nbc = (rng.random((n, 256)) < 0.02).astype(np.int32) * rng.integers(1, 4, (n, 256)).astype(np.int32)
    nbc[2 * NPC:3 * NPC] = 0  # an empty column counts as uniform
    last = rng.integers(-1, 500, n).astype(np.int32)
    r = po.semantic_eval(nbc, last, regions(6, n), 6, NPC, 500)
    assert abs(r["js_mean"] - column_js_mean(nbc, 6, NPC)) < 1e-12
    assert r["nonzero_columns"] == 5
    li = ((500 - 1) // 3) * 3
    reg = regions(6, n)
    for k in range(5):
        sel = (reg == k) & (last >= li)
        assert r["layer_delay_n"][k] == int(sel.sum())


@pytest.mark.gpu
def test_library_matches_the_restatement():
    import snn_b200 as snn
    net = snn.Network(device=0, phase_offset=5000)
    net.build_columns(snn.topology(n_columns=NCOL))
    net.set_corpus(snn.stream(20000, seed=11))
    net.run(900)
    got = net.semantic_eval()
    want = po.semantic_eval(net.state("neuron_byte_counts").reshape(-1, 256), net.state("last"),
                            regions(NCOL, net.N), NCOL, NPC, net.counters()["step"])
    assert got["grand_total"] > 0
    for k in ("js_mean", "js_max", "silhouette", "column_ratio", "grand_total", "nonzero_columns",
              "n_columns", "layer_delay", "layer_delay_n", "layer_sig", "layer_act", "layer_chi2_mean"):
        assert got[k] == want[k], k
    assert list(got["assign"]) == want["assign"]
    # an explicit step moves the injection window
    assert net.semantic_eval(step=450)["layer_delay_n"] != got["layer_delay_n"]
    net.close()


@pytest.mark.gpu
def test_other_models_refuse():
    import snn_b200 as snn
    net = snn.Network(device=0, model=snn.MODEL_STAGE0)
    net.build_columns(snn.topology(snn.MODEL_STAGE0))
    with pytest.raises(snn.SnnError) as e:
        net.semantic_eval()
    assert "Stage 2e" in str(e.value)
    net.close()
