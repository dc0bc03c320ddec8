"""Stage 2e parity: the CUDA path (through the C ABI) against the CPU oracle.

Bar: bit-exact.  Spike rasters are compared every step; at the end every
neuron field, every synapse field (in the reference's pre-major order,
including the group-factored R / u / NMDA g / x_pre, the derived weight and
the per-neuron x_post) and the control state are compared with
np.array_equal on the raw float32 bits.  Small column counts keep the oracle
fast enough to cover the 10 / 100 / 1000-step schedules; the full reference
network (55,000 neurons / 10,700,000 synapses) is checked for 1,000 steps.
"""
import numpy as np
import pytest

import pyoracle as po
import snn_b200 as snn

SYN_FIELDS = ["alpha", "beta", "weight", "x_pre", "nmda", "ca", "R", "u", "elig",
              "camkii_act", "autophos", "e1", "e2", "ampa", "last_pre"]
NEU_FIELDS = [("V", "V"), ("w", "w"), ("s", "s"), ("fr", "fr"), ("ca_neuron", "ca"),
              ("nmda_cur", "nmda_cur")]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def unpack(raster_row, n):
    return np.unpackbits(raster_row.view(np.uint8), bitorder="little")[:n]


def compare_state(net, orc, tag):
    for mine, theirs in NEU_FIELDS:
        a, b = net.state(mine), orc.neuron(theirs)
        bad = np.nonzero(bits(a) != bits(b))[0]
        assert bad.size == 0, f"{tag}: neuron field {mine} differs at {bad[:5]} ({a[bad[:3]]} vs {b[bad[:3]]})"
    # the device input buffer already holds the next step's arrival sum
    a, b = net.state("input"), orc.next_input()
    bad = np.nonzero(bits(a) != bits(b))[0]
    assert bad.size == 0, f"{tag}: next-step input differs at {bad[:5]} ({a[bad[:3]]} vs {b[bad[:3]]})"
    last = net.state("last").astype(np.float32)
    assert np.array_equal(last, orc.neuron("last")), f"{tag}: last spike"
    # x_post of every synapse equals its post neuron's trace
    xp = net.state("x_post")
    post = net.state("post")
    assert np.array_equal(bits(xp[post]), bits(orc.synapse("x_post"))), f"{tag}: x_post"
    for f in SYN_FIELDS:
        a, b = net.state(f), orc.synapse(f)
        bad = np.nonzero(bits(a) != bits(b))[0]
        assert bad.size == 0, f"{tag}: synapse field {f} differs at {bad.size} synapses, first {bad[:5]} ({a[bad[:3]]} vs {b[bad[:3]]})"
    g, m, bh = orc.control()
    assert np.array_equal(bits(net.state("gates")), bits(g)), f"{tag}: gates"
    assert np.array_equal(bits(net.state("modulators")), bits(m)), f"{tag}: modulators"
    assert np.array_equal(net.state("byte_hist"), bh), f"{tag}: byte histogram"


def run_pair(ncol, steps, corpus_seed=7, phase_offset=0, e0=False, chunk=None, threads=0,
             check_state_every=None, preset=0, corpus_bytes=20000, p_cjk=0.452):
    corpus = snn.stream(corpus_bytes, seed=corpus_seed, p_cjk=p_cjk)
    orc = po.Oracle2e(po.ref_params(ncol, e0=int(e0), phase_offset=phase_offset,
                                    n_threads=threads, preset=preset), corpus)
    net = snn.Network(e0=e0, phase_offset=phase_offset,
                      preset=snn.PRESET_BASELINE if preset else snn.PRESET_REF)
    net.build_columns(snn.topology(n_columns=ncol))
    net.set_corpus(corpus)
    assert (net.N, net.S) == (orc.N, orc.S)
    chunk = chunk or steps
    done = 0
    while done < steps:
        n = min(chunk, steps - done)
        raster, counts = net.run(n, raster=True, counts=True)
        for k in range(n):
            orc.run(1)
            sp = orc.spikes()
            got = unpack(raster[k], net.N)
            if not np.array_equal(got, sp):
                diff = np.nonzero(got != sp)[0]
                raise AssertionError(f"raster differs at step {done + k}: neurons {diff[:10]}")
            assert counts[k] == int(sp.sum())
        done += n
        if check_state_every and done % check_state_every == 0:
            compare_state(net, orc, f"step {done}")
    compare_state(net, orc, f"end ({steps} steps)")
    c, oc = net.counters(), orc.counters()
    assert c["total_spikes"] == oc.total_spikes
    assert c["arrivals"] == oc.arrived
    assert c["dispatched"] == oc.dispatched
    assert c["ltp_visits"] == oc.ltp_visits
    assert c["dropped_ref"] == oc.dropped
    assert c["burst_spikes"] == oc.burst_spikes
    net.close()
    orc.close()
    return c


@pytest.mark.gpu
def test_topology_matches_oracle():
    """The product's generator gives the oracle's (reference-pinned) network."""
    orc = po.Oracle2e(po.ref_params(50))
    net = snn.Network()
    net.build_columns(snn.topology(n_columns=50))
    rp, post, d, fl = orc.topology()
    assert np.array_equal(net.state("row_ptr"), rp)
    assert np.array_equal(net.state("post"), post)
    assert np.array_equal(net.state("delay"), d)
    assert np.array_equal(net.state("flags"), fl)
    _, a, b = orc.init_weights()
    assert np.array_equal(bits(net.state("alpha")), bits(a))
    assert np.array_equal(bits(net.state("beta")), bits(b))


@pytest.mark.gpu
def test_parity_small_embryonic_1200_steps():
    """2 columns, 1,200 steps from step 0 (gain 0 phase): covers the 10-, 100-
    and 1000-step schedules, the delay ring and every state field."""
    run_pair(2, 1200, chunk=300, check_state_every=600)


@pytest.mark.gpu
def test_parity_small_learning_phase():
    """Phase table shifted into SYNAPTOGENIC (gain 1): LTP / LTD / rebound
    change alpha and beta from the first step."""
    run_pair(3, 1100, phase_offset=5000, chunk=550, check_state_every=550)


@pytest.mark.gpu
def test_parity_critical_and_pruning_phases():
    """gain 3 (CRITICAL) and PRUNING (evidence reset threshold 0.05)."""
    run_pair(2, 400, phase_offset=200000)
    run_pair(2, 1001, phase_offset=800000, chunk=1001)


@pytest.mark.gpu
def test_parity_e0_ablation():
    run_pair(2, 600, e0=True, phase_offset=5000)


@pytest.mark.gpu
def test_parity_baseline_preset():
    """The benchmark's AdEx / STP constants (SNN_PRESET_BASELINE) in the
    SYNAPTOGENIC phase, rasters every step and the full state twice."""
    run_pair(4, 400, phase_offset=5000, chunk=100, check_state_every=200, preset=1)


@pytest.mark.gpu
def test_parity_single_step_api():
    """snn_step with explicit bytes equals the oracle fed the same bytes."""
    corpus = snn.stream(400, seed=11)
    orc = po.Oracle2e(po.ref_params(2), corpus)
    net = snn.Network()
    net.build_columns(snn.topology(n_columns=2))
    pos = 0
    for t in range(150):
        b = -1
        if t % 3 == 0:
            b = int(corpus[pos])
            pos += 1
        net.step(t, inject_byte=b)
        orc.run(1)
        assert np.array_equal(net.spikes(), orc.spikes()), f"step {t}"
    compare_state(net, orc, "single-step api")


@pytest.mark.gpu
def test_parity_full_reference_network_1000_steps():
    """55,000 neurons / 10,700,000 synapses (the reference network), 1,000
    steps: rasters bit-identical every step, all state bit-identical at the end."""
    c = run_pair(50, 1000, chunk=250, threads=0, check_state_every=500)
    assert c["n_synapses"] == 10_700_000 and c["n_neurons"] == 55_000


@pytest.mark.gpu
def test_parity_benchmarked_configuration_1000_steps():
    """The configuration the throughput line is quoted on: the reference
    network (50 columns), phase table shifted into SYNAPTOGENIC (phase offset
    5000, plasticity gain 1), the `ref45` stream (seed 42, 1 MiB), 1,000
    steps: rasters bit-identical every step, all state bit-identical at steps
    500 and 1,000, counters equal."""
    c = run_pair(50, 1000, corpus_seed=42, phase_offset=5000, chunk=250, threads=0,
                 check_state_every=500, corpus_bytes=1 << 20, p_cjk=0.452)
    assert c["n_synapses"] == 10_700_000 and c["ltp_visits"] > 0
