"""Stage 0 / Stage 2 parity (configurations 0 and 1): the CUDA path through the
C ABI against the CPU oracle (oracle/oracle0.cpp), bit-exact: spike raster
every step, membrane state, weights and eligibility traces at the end."""
import numpy as np
import pytest

import pyoracle as po
import snn_b200 as snn


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def run_pair(columnar, baseline, steps, bytes_, chunk=None, dopamine=None):
    orc = po.Oracle0(po.stage0_params(columnar=columnar, baseline=baseline))
    net = snn.Network(model=snn.MODEL_STAGE0,
                      preset=snn.PRESET_BASELINE if baseline else snn.PRESET_REF)
    net.build_columns(snn.topology(snn.MODEL_STAGE0, n_columns=10 if columnar else 0))
    assert (net.N, net.S) == (orc.N, orc.S)
    net.set_corpus(bytes(bytes_.astype(np.uint8)))
    pre, post = orc.topology()
    assert np.array_equal(net.state("post"), post)
    chunk = chunk or steps
    done = 0
    while done < steps:
        n = min(chunk, steps - done)
        if dopamine is not None and done > 0:
            net.set_dopamine(dopamine)
            orc.set_dopamine(dopamine)
        raster, counts = net.run(n, raster=True, counts=True)
        for k in range(n):
            orc.run(1, [int(bytes_[(done + k) % len(bytes_)])])
            sp = orc.spikes()
            got = np.unpackbits(raster[k].view(np.uint8), bitorder="little")[: net.N]
            if not np.array_equal(got, sp):
                raise AssertionError(f"raster differs at step {done + k}: {np.nonzero(got != sp)[0][:10]}")
            assert counts[k] == sp.sum()
        done += n
    for mine, theirs in (("V", "V"), ("s", "I"), ("fr", "fr")):
        assert np.array_equal(bits(net.state(mine)), bits(orc.neuron(theirs))), mine
    assert np.array_equal(bits(net.state("weight")), bits(orc.synapse("w"))), "weights"
    assert np.array_equal(bits(net.state("elig")), bits(orc.synapse("elig"))), "eligibility"
    c = net.counters()
    assert c["total_spikes"] == int(orc.sizes()[3])
    # the last step's spike count, and the arrivals: every dispatch but the last step's
    assert c["last_spikes"] == int(orc.sizes()[4]) == counts[-1]
    deg = net.S // net.N
    assert c["dispatched"] == c["total_spikes"] * deg
    assert c["arrivals"] == (c["total_spikes"] - c["last_spikes"]) * deg
    net.close()
    orc.close()


@pytest.mark.gpu
def test_stage0_block_network_uniform_bytes():
    """Configuration 0: 10,000 LIF / 1,000,000 synapses, uniform random bytes."""
    rng = np.random.default_rng(42)
    run_pair(False, True, 600, rng.integers(0, 256, 4000), chunk=200)


@pytest.mark.gpu
def test_stage2_columnar_stream_with_reset():
    """Configuration 1: 10 columns x 1,000, synthetic UTF-8 stream, reference
    Stage 2 constants, across a periodic reset (every 10,000 steps)."""
    b = snn.stream(30000, seed=9)
    run_pair(True, False, 10150, b, chunk=1015)


@pytest.mark.gpu
def test_stage0_dopamine_change():
    rng = np.random.default_rng(3)
    run_pair(False, True, 300, rng.integers(0, 256, 300), chunk=100, dopamine=0.25)
