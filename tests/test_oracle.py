"""CPU tests of the oracle: pinned against the reference's own topology
generator, its exponential, its determinism, and the exact invariants that
the CUDA layout relies on (checked here on the oracle's per-synapse state)."""
import json
import os

import numpy as np
import pytest

import pyoracle as po

HERE = os.path.dirname(os.path.abspath(__file__))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_exp_within_one_ulp_of_libm():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.uniform(-103.9, 88.7, 2_000_000),
        rng.uniform(-12, 12, 1_000_000),           # AdEx / Mg block / sigmoid range
        np.linspace(-1e-6, 1e-6, 10001),
        np.array([0.0, -0.0, 1.0, -1.0, 88.72, -103.97, -87.3, -100.0]),
    ]).astype(np.float32)
    got = po.expf_array(x)
    want = np.exp(x.astype(np.float64)).astype(np.float32)
    gi = got.view(np.int32).astype(np.int64)
    wi = want.view(np.int32).astype(np.int64)
    assert np.max(np.abs(gi - wi)) <= 1
    # constant decay factors used by the step
    for tau in (3.0, 5.0, 10.0, 20.0, 50.0, 150.0, 200.0, 500.0):
        a = np.float32(-1.0) / np.float32(tau)
        assert abs(int(po.expf_array(np.array([a]))[0].view(np.int32)) -
                   int(np.float32(np.exp(np.float64(a))).view(np.int32))) <= 1


def test_topology_pinned_to_reference_generator():
    """The oracle's generator reproduces, bit for bit, the arrays of the
    reference's own host generator (hashes in tests/golden, produced by
    compiling src/stage2e/network_init.cu unmodified)."""
    with open(os.path.join(HERE, "golden", "topology_ref_hashes.json")) as f:
        ref = json.load(f)
    o = po.Oracle2e(po.ref_params(50))
    assert o.S == ref["n_synapses"] == 10_700_000 and o.N == 55_000
    rp, post, d, fl = o.topology()
    w, a, b = o.init_weights()
    mine = {"row_ptr": rp, "post": post, "weights": w, "delay": d, "alpha": a, "beta": b,
            "flags": fl, "utilization": o.synapse("u")}
    for k, arr in mine.items():
        assert "%016x" % po.fnv64(arr) == ref[k], k
    for item in ref["sample"]:
        i, pre, p, wv, dv = item.split(":")
        i = int(i)
        assert post[i] == int(p) and d[i] == int(dv)
        assert np.float32(wv) == w[i]
        assert rp[int(pre)] <= i < rp[int(pre) + 1]
    o.close()


def test_oracle_deterministic_across_thread_counts():
    corpus = bytes(range(256)) * 20
    out = []
    for th in (1, 4):
        o = po.Oracle2e(po.ref_params(2, phase_offset=5000, n_threads=th), corpus)
        o.run(150)
        out.append([o.neuron("V"), o.synapse("alpha"), o.synapse("beta"), o.synapse("ca"),
                    o.neuron("nmda_cur"), o.neuron("input")])
        o.close()
    for x, y in zip(*out):
        assert np.array_equal(bits(x), bits(y))


@pytest.fixture(scope="module")
def ran_oracle():
    corpus = bytes((i * 37 + 11) % 256 for i in range(5000))
    o = po.Oracle2e(po.ref_params(3, phase_offset=5000), corpus)
    o.run(620)
    yield o
    o.close()


def test_invariant_post_trace_is_per_neuron(ran_oracle):
    o = ran_oracle
    _, post, _, _ = o.topology()
    xp = o.synapse("x_post")
    ref = np.zeros(o.N, np.float32)
    ref[post] = xp
    assert np.array_equal(bits(xp), bits(ref[post]))


def test_invariant_group_state(ran_oracle):
    """R, u, NMDA conductance and x_pre are identical for all synapses with the
    same (pre, effective delay, feed-forward flag)."""
    o = ran_oracle
    rp, post, d, fl = o.topology()
    pre = np.repeat(np.arange(o.N), np.diff(rp))
    de = np.clip(d.astype(np.int64), 1, 19)
    key = pre * 64 + de * 2 + ((fl & 0x10) > 0)
    order = np.argsort(key, kind="stable")
    ks = key[order]
    first = np.r_[True, ks[1:] != ks[:-1]]
    gidx = np.cumsum(first) - 1
    for f in ("R", "u", "nmda", "x_pre"):
        v = bits(o.synapse(f))[order]
        rep = v[first][gidx]
        assert np.array_equal(v, rep), f
    assert np.count_nonzero(o.synapse("nmda")) > 0 and np.count_nonzero(o.synapse("x_pre")) > 0


def test_invariant_weight_and_inhibitory_zeros(ran_oracle):
    o = ran_oracle
    _, _, _, fl = o.topology()
    a, b, w = o.synapse("alpha"), o.synapse("beta"), o.synapse("weight")
    m = (np.float32(1.5) * a) / (a + b)
    exc = (fl & 0x03) > 0
    assert np.array_equal(bits(w), bits(np.where(exc, m, -m)))
    assert a.min() >= np.float32(1e-4) and b.min() >= np.float32(1e-4)
    inh = ~exc
    for f in ("ca", "nmda", "camkii_act", "autophos"):
        assert not np.any(o.synapse(f)[inh]), f
    assert np.count_nonzero(o.synapse("ca")[exc]) > 0


def test_modulators_uniform_and_bounded(ran_oracle):
    _, m, bh = ran_oracle.control()
    assert np.all(m >= 0) and np.all(m <= 2) and m[0] > 0
    assert bh.sum() > 0


def test_activity_in_reference_range():
    """Liveness ranges of the reference's own criteria
    (src/stage2e/main.cpp:775-1396): spikes vary across steps and the delay
    ring drops nothing."""
    o = po.Oracle2e(po.ref_params(4), bytes(range(256)) * 10)
    counts = []
    for _ in range(120):
        o.run(1)
        counts.append(o.counters().last_spikes)
    c = o.counters()
    assert max(counts) - min(counts) > 10
    assert c.dropped == 0 and c.arrived > 0 and c.dispatched >= c.arrived
    o.close()


def test_oracle_reproduces_reference_engine_on_b200():
    """Pin against the reference itself: its Stage 2e scheduler, compiled
    unmodified and run on a B200 (tests/golden/make_ref_gpu_pin.sh), fed the
    same byte stream.  The oracle's spike raster matches the reference's at
    every one of the 300 steps; fire rates are bit-identical and the PSW
    evidence sums are identical; V and w agree to the reference's own
    float-atomic rounding noise."""
    import snn_b200 as snn
    corpus = snn.stream(200000, seed=7).tobytes()
    ref = [l.split() for l in open(os.path.join(HERE, "golden", "ref_b200_stage2e_seed7_spikes.txt"))]
    st = np.load(os.path.join(HERE, "golden", "ref_b200_stage2e_seed7_state.npz"))
    o = po.Oracle2e(po.ref_params(50), corpus)
    for t in range(300):
        o.run(1)
        idx = np.nonzero(o.spikes())[0].astype(np.int32)
        assert idx.size == int(ref[t][1]), f"step {t}: spike count"
        assert "%016x" % po.fnv64(idx) == ref[t][2], f"step {t}: spike set"
    sel = st["idx"]
    assert np.array_equal(o.neuron("fr")[sel], st["fr"])
    assert o.synapse("alpha").astype(np.float64).sum() == float(st["alpha_sum"])
    assert o.synapse("beta").astype(np.float64).sum() == float(st["beta_sum"])
    assert np.max(np.abs(o.neuron("V")[sel] - st["V"])) < 5e-4
    assert np.max(np.abs(o.neuron("w")[sel] - st["w"])) < 5e-6
    o.close()
