"""The propagation microbench sharded by post bucket over 2 GPUs (one process
per GPU, no exchange during the run) against the CPU oracle of the whole
network (plain, STDP, STDP + STP): every rank's spike raster on its own
neurons, bit-exact at every step; its neuron state, the STP / spike-time state
of every pre and the weights of the synapses onto its neurons at the end
(with STDP: LTD in the push and LTP over the reverse CSR of local spikes);
event counts that add up to the oracle's.  Needs two GPUs; skipped
otherwise."""
import json
import os

import numpy as np
import pytest

import pyoracle as po
import snn_b200 as snn

N, FANOUT, RATE, STEPS = 30011, 200, 0.02, 240


def two_gpus():
    try:
        import torch
        return torch.cuda.device_count() >= 2
    except Exception:
        return False


def w_max_of(mode):
    # with STP the releases u * R are a fraction of 1: a larger weight bound
    # keeps the posts firing, so that LTP and the post-spike lists are covered
    return 4.0 * po.prop_w_max(RATE, FANOUT) if mode & snn.PROP_STP else 0.0


def rank_main(rank, world, mode, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for sub in ("pure-snn-language_b200", "oracle"):
        sys.path.insert(0, os.path.join(os.path.dirname(here), sub))
    import snn_b200 as snn
    net = snn.Network(device=rank, model=snn.MODEL_PROP, prop_mode=mode, prop_rate=RATE,
                      prop_w_max=w_max_of(mode))
    net.set_shard(rank, world)
    net.build_columns(snn.topology(snn.MODEL_PROP, l4=N, deg_intra=FANOUT, seed=42))
    raster = np.concatenate([net.run(100, raster=True)[0], net.run(STEPS - 100, raster=True)[0]])
    np.save(os.path.join(out_dir, f"raster{rank}.npy"), raster)
    fields = ["V", "s", "ref", "last", "weight", "post"]
    if mode & snn.PROP_STP:
        fields += ["u", "R"]
    for f in fields:
        np.save(os.path.join(out_dir, f"{f}{rank}.npy"), net.state(f))
    with open(os.path.join(out_dir, f"counters{rank}.json"), "w") as fh:
        json.dump(net.counters(), fh)
    net.close()


@pytest.mark.gpu
@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", [0, 1, 3])
def test_two_rank_post_bucket_shards_match_the_oracle(tmp_path, mode):
    import torch.multiprocessing as mp
    mp.start_processes(rank_main, args=(2, mode, str(tmp_path)), nprocs=2, start_method="spawn")
    orc = po.Oracle4(po.prop_params(n=N, fanout=FANOUT, seed=42, rate=RATE, mode=mode,
                                    w_max=w_max_of(mode)))
    want = np.unpackbits(orc.run(STEPS, raster=True).view(np.uint8), axis=1, bitorder="little")[:, :N]
    cs = [json.load(open(tmp_path / f"counters{r}.json")) for r in range(2)]
    assert cs[0]["local_lo"] == 0 and cs[0]["local_hi"] == cs[1]["local_lo"] and cs[1]["local_hi"] == N
    post = orc.post()
    for r, c in enumerate(cs):
        lo, hi = c["local_lo"], c["local_hi"]
        got = np.unpackbits(np.load(tmp_path / f"raster{r}.npy").view(np.uint8), axis=1,
                            bitorder="little")[:, :N]
        bad = np.nonzero((got[:, lo:hi] != want[:, lo:hi]).any(axis=1))[0]
        assert bad.size == 0, f"rank {r}: raster differs first at step {bad[:1]}"
        assert not got[:, :lo].any() and not got[:, hi:].any(), f"rank {r}: spikes outside its range"
        for mine, theirs in (("V", "V"), ("s", "I"), ("ref", "ref"), ("last", "last_post")):
            a = np.load(tmp_path / f"{mine}{r}.npy")[lo:hi]
            b = orc.neuron(theirs)[lo:hi]
            assert np.array_equal(a.view(np.uint32), np.asarray(b, a.dtype).view(np.uint32)), \
                f"rank {r}: {mine}"
        if mode & snn.PROP_STP:  # the pres' STP state is replicated on every rank
            for f in ("u", "R"):
                assert np.array_equal(np.load(tmp_path / f"{f}{r}.npy").view(np.uint32),
                                      orc.neuron(f).view(np.uint32)), f"rank {r}: {f}"
        assert np.array_equal(np.load(tmp_path / f"post{r}.npy"), post)
        mine = (post >= lo) & (post < hi)
        w = np.load(tmp_path / f"weight{r}.npy")
        assert np.array_equal(w[mine].view(np.uint32), orc.weights()[mine].view(np.uint32)), \
            f"rank {r}: weights onto its neurons"
    oc = orc.counters()
    assert sum(c["total_spikes"] for c in cs) == oc["total_spikes"]
    assert oc["total_spikes"] > 0
    assert sum(c["arrivals"] for c in cs) == oc["events"]
    assert all(c["dispatched"] == oc["pre_spikes"] for c in cs)  # every rank draws every pre-spike
    if mode & snn.PROP_STDP:
        assert oc["ltp_visits"] > 0
        assert sum(c["ltp_visits"] for c in cs) == oc["ltp_visits"]
    orc.close()
