"""Propagation microbench (1 M LIF neurons x 1,000 random targets, forced
Poisson pre-spikes) and the standalone push entry point snn_propagate: the
CUDA path through the C ABI against the CPU oracle (oracle/oracle4.cpp),
bit-exact: LIF spike raster every step, V / I / refractory / last spike,
weights (STDP) and the per-neuron STP state at the end."""
import numpy as np
import pytest

import pyoracle as po
import snn_b200 as snn


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def run_pair(n, fanout, rate, mode, steps, chunk=None, seed=42, learn=True, dopamine=None,
             oracle_mode=None, push=0):
    orc = po.Oracle4(po.prop_params(n=n, fanout=fanout, seed=seed, rate=rate,
                                    mode=mode if oracle_mode is None else oracle_mode))
    net = snn.Network(model=snn.MODEL_PROP, prop_mode=mode, prop_rate=rate, prop_push=push)
    net.build_columns(snn.topology(snn.MODEL_PROP, l4=n, deg_intra=fanout, seed=seed))
    assert (net.N, net.S) == (n, n * fanout)
    chunk = chunk or steps
    done = 0
    while done < steps:
        k = min(chunk, steps - done)
        if dopamine is not None and done > 0:
            net.set_dopamine(dopamine)
            orc.set_dopamine(dopamine)
        raster, counts = net.run(k, learn=learn, raster=True, counts=True)
        want = orc.run(k, raster=True)
        if not np.array_equal(raster, want):
            bad = np.nonzero((raster != want).any(axis=1))[0]
            raise AssertionError(f"raster differs first at step {done + bad[0]}")
        assert np.array_equal(counts, np.unpackbits(want.view(np.uint8), axis=1).sum(axis=1))
        done += k
    for mine, theirs in (("V", "V"), ("s", "I")):
        assert np.array_equal(bits(net.state(mine)), bits(orc.neuron(theirs))), mine
    assert np.array_equal(net.state("ref"), orc.neuron("ref"))
    assert np.array_equal(net.state("last"), orc.neuron("last_post"))
    assert np.array_equal(bits(net.state("weight")), bits(orc.weights())), "weights"
    if mode & snn.PROP_STP:
        assert np.array_equal(bits(net.state("u")), bits(orc.neuron("u")))
        assert np.array_equal(bits(net.state("R")), bits(orc.neuron("R")))
    c, oc = net.counters(), orc.counters()
    assert c["total_spikes"] == oc["total_spikes"]
    assert c["arrivals"] == oc["events"] and c["dispatched"] == oc["pre_spikes"]
    if learn:
        assert c["ltp_visits"] == oc["ltp_visits"]
    assert c["last_spikes"] == oc["last_spikes"]
    net.close()
    orc.close()
    return oc


@pytest.mark.gpu
@pytest.mark.parametrize("push", [1, 2])
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
@pytest.mark.parametrize("rate", [0.001, 0.01, 0.1])
def test_microbench_small(mode, rate, push):
    """40,000 neurons (3 post buckets) x 1,000 out-edges, 300 steps across
    graph chunks, with the L2-atomic push (1) and the bucketed push (2)."""
    oc = run_pair(40000, 1000, rate, mode, 300, chunk=120, push=push)
    assert oc["total_spikes"] > 0 or mode & snn.PROP_STP


@pytest.mark.gpu
def test_microbench_ragged_fanout():
    """Fan-out 99 (not a multiple of 4: the scalar push) with STDP + STP,
    and the same through the bucketed push."""
    run_pair(7001, 99, 0.02, 3, 200, chunk=75, push=1)
    run_pair(7001, 99, 0.02, 3, 200, chunk=75, push=2)


@pytest.mark.gpu
def test_microbench_learn_off_and_dopamine():
    # learn = 0 freezes STDP: identical to the plain model
    run_pair(12000, 400, 0.01, 1, 150, learn=False, oracle_mode=0)
    # dopamine scales both LTD and LTP from the second chunk on
    run_pair(12000, 400, 0.01, 1, 150, chunk=50, dopamine=0.25)


@pytest.mark.gpu
def test_microbench_full_size():
    """1,000,000 neurons x 1,000 targets (1.0 B synapses) with STDP at the
    1 % rate (bucketed push): the benchmark network itself, 40 steps bit-exact
    (LIF spikes, and so LTP, start after about 25 steps)."""
    oc = run_pair(1_000_000, 1000, 0.01, 1, 40, chunk=20)
    assert oc["total_spikes"] > 0 and oc["ltp_visits"] > 0


@pytest.mark.gpu
@pytest.mark.parametrize("fanout,offset", [(1000, 0), (37, 0), (64, 1)])
def test_snn_propagate(fanout, offset):
    """snn_propagate on torch tensors against the exact closed form; a
    post index out of range is skipped; a misaligned view takes the scalar
    path."""
    import torch
    rng = np.random.default_rng(fanout)
    n_pre, n_post = 5000, 7000
    post = rng.integers(0, n_post, size=n_pre * fanout + offset).astype(np.int32)
    w = rng.uniform(-0.5, 0.5, size=n_pre * fanout + offset).astype(np.float32)
    post[offset + 17] = n_post + 5  # out of range: skipped
    post[offset + 18] = -3
    sp = (rng.random(n_pre) < 0.05).astype(np.uint8)
    sp[0] = 1
    dev = torch.device("cuda:0")
    tp = torch.from_numpy(post).to(dev)[offset:]
    tw = torch.from_numpy(w).to(dev)[offset:]
    ts = torch.from_numpy(sp).to(dev)
    acc = torch.zeros(n_post, dtype=torch.int32, device=dev)
    for call in range(2):
        snn.propagate(tp, tw, fanout, ts, acc, frac_bits=20)
    torch.cuda.synchronize()
    p, ww = post[offset:], w[offset:]
    q = np.rint(ww.astype(np.float64) * 2.0 ** 20).astype(np.int64)
    m = np.repeat(sp, fanout).astype(bool) & (p >= 0) & (p < n_post)
    want = np.zeros(n_post, np.int64)
    np.add.at(want, p[m], 2 * q[m])
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), want)
