"""CPU checks of the propagation-microbench oracle (oracle/oracle4.cpp).

The reference has no such microbench, so the model is pinned by independent
restatements: the seeded generator and the forced-spike rule re-derived here
in numpy uint64 arithmetic, the exact integer push sum, the first LIF step in
closed form, and thread-count determinism of the OpenMP oracle.
"""
import numpy as np
import pytest

import pyoracle as po

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def mix64(z):
    """SplitMix64 output function on a numpy uint64 array (wrapping)."""
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def np_topology(n, fanout, seed, w_max):
    s = np.arange(n * fanout, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = mix64(np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15) + s)
    post = (((h >> np.uint64(32)) * np.uint64(n)) >> np.uint64(32)).astype(np.int32)
    u = (h & np.uint64(0xFFFFFF)).astype(np.float32) * np.float32(2.0 ** -24)
    w = (u * np.float32(w_max)).astype(np.float32)
    exc = (np.arange(n * fanout) // fanout) < (n * 4) // 5
    return post, np.where(exc, w, -w).astype(np.float32)


def np_spikes(n, t, seed, rate):
    key = mix64(np.array([seed + 1], np.uint64))[0]
    i = np.arange(n, dtype=np.uint64)
    h = mix64(((np.uint64(t) << np.uint64(32)) | i) ^ key)
    thr = np.uint64(min(int(float(np.float32(rate)) * 2.0 ** 32), 0xFFFFFFFF))
    return (h >> np.uint64(32)) < thr


def test_generator_matches_restatement():
    p = po.prop_params(n=3000, fanout=40, seed=7, rate=0.05)
    o = po.Oracle4(p)
    post, w = np_topology(3000, 40, 7, p.w_max)
    assert np.array_equal(o.post(), post)
    assert np.array_equal(o.weights().view(np.uint32), w.view(np.uint32))
    # uniform targets: every post reachable, in-degree mean = fan-out
    deg = np.bincount(post, minlength=3000)
    assert deg.mean() == 40 and deg.min() > 10


def test_forced_spikes_match_restatement():
    n, rate = 5000, 0.03
    p = po.prop_params(n=n, fanout=8, seed=11, rate=rate)
    o = po.Oracle4(p)
    last = np.full(n, -1, np.int64)
    total = 0
    for t in range(25):
        o.run(1)
        sp = np_spikes(n, t, 11, rate)
        last[sp] = t
        total += int(sp.sum())
    assert np.array_equal(o.neuron("last_pre"), last.astype(np.int32))
    c = o.counters()
    assert c["pre_spikes"] == total and c["events"] == total * 8
    assert abs(total / (25 * n) - rate) < 0.005


def test_exact_push_closed_form():
    rng = np.random.default_rng(1)
    n_pre, fanout, n_post = 3000, 50, 5000
    post = rng.integers(0, n_post, size=n_pre * fanout).astype(np.int32)
    w = rng.uniform(-1, 1, size=n_pre * fanout).astype(np.float32)
    sp = (rng.random(n_pre) < 0.1).astype(np.uint8)
    for fb in (0, 12, 24):
        acc = po.propagate(post, w, fanout, sp, n_post, frac_bits=fb)
        q = np.rint(w.astype(np.float64) * 2.0 ** fb).astype(np.int64)
        m = np.repeat(sp, fanout).astype(bool)
        ref = np.zeros(n_post, np.int64)
        np.add.at(ref, post[m], q[m])
        assert np.array_equal(acc.astype(np.int64), ref)


def test_first_step_closed_form():
    n, fanout, rate = 4000, 100, 0.05
    p = po.prop_params(n=n, fanout=fanout, seed=3, rate=rate, w_max=0.2)
    o = po.Oracle4(p)
    post, w = np_topology(n, fanout, 3, p.w_max)
    o.run(1)
    sp = np_spikes(n, 0, 3, rate).astype(np.uint8)
    acc = po.propagate(post, w, fanout, sp, n, frac_bits=24)
    x = (acc.astype(np.float32) * np.float32(2.0 ** -24)).astype(np.float32)
    v = np.maximum(x, np.float32(0))
    fired = v >= 1.0
    assert np.array_equal(o.neuron("I"), x)
    assert np.array_equal(o.neuron("V"), np.where(fired, np.float32(0), v))
    assert np.array_equal(o.neuron("ref"), np.where(fired, 2, 0).astype(np.int32))
    assert fired.sum() > 0


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_thread_determinism(mode):
    runs = []
    for nt in (1, 4):
        p = po.prop_params(n=6000, fanout=200, seed=5, rate=0.02, mode=mode, n_threads=nt)
        o = po.Oracle4(p)
        r = o.run(80, raster=True)
        runs.append((r, o.neuron("V"), o.weights(), o.neuron("R"), o.counters()))
        o.close()
    a, b = runs
    assert np.array_equal(a[0], b[0])
    assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    assert np.array_equal(a[2].view(np.uint32), b[2].view(np.uint32))
    assert np.array_equal(a[3].view(np.uint32), b[3].view(np.uint32))
    assert a[4] == b[4]


def test_plasticity_and_stp_invariants():
    p = po.prop_params(n=8000, fanout=250, seed=9, rate=0.01, mode=3)
    o = po.Oracle4(p)
    o.run(120)
    w = o.weights()
    n_exc = (8000 * 4) // 5
    we = w[: n_exc * 250]
    assert we.min() >= 0 and we.max() <= np.float32(p.w_max)
    w0 = np_topology(8000, 250, 9, p.w_max)[1]
    assert np.array_equal(w[n_exc * 250:], w0[n_exc * 250:])  # inhibitory weights frozen
    assert not np.array_equal(we, w0[: n_exc * 250])           # excitatory ones learn
    u, R = o.neuron("u"), o.neuron("R")
    assert u.min() >= 0.5 and u.max() <= 1.0
    assert R.min() >= 0.0 and R.max() <= 1.0
    c = o.counters()
    assert c["ltp_visits"] > 0 and c["total_spikes"] > 0
