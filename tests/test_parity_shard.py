"""Column sharding over 2 GPUs (one process per GPU, NCCL all-gather of the
step's spike bitmask and counts) against the CPU oracle of the whole network:
every rank's spike raster, bit-exact at every step, and its neuron state at
the end.  Needs two GPUs; skipped otherwise."""
import json
import os

import numpy as np
import pytest

import pyoracle as po
import snn_b200 as snn

NCOL, STEPS, PHASE = 8, 300, 5000


def two_gpus():
    try:
        import torch
        return torch.cuda.device_count() >= 2
    except Exception:
        return False


def rank_main(rank, world, uid, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for sub in ("pure-snn-language_b200", "oracle"):
        sys.path.insert(0, os.path.join(os.path.dirname(here), sub))
    import snn_b200 as snn
    net = snn.Network(device=rank, phase_offset=PHASE)
    net.set_shard(rank, world, uid)
    net.build_columns(snn.topology(n_columns=NCOL))
    net.set_corpus(snn.stream(20000, seed=7))
    raster, counts = net.run(STEPS, raster=True, counts=True)
    np.save(os.path.join(out_dir, f"raster{rank}.npy"), raster)
    for f in ("V", "w", "fr", "nmda_cur", "input"):
        np.save(os.path.join(out_dir, f"{f}{rank}.npy"), net.state(f))
    with open(os.path.join(out_dir, f"counters{rank}.json"), "w") as fh:
        json.dump(net.counters(), fh)
    net.close()


@pytest.mark.gpu
@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
def test_two_rank_column_shards_match_the_oracle(tmp_path):
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    uid = snn.nccl_unique_id()
    mp.start_processes(rank_main, args=(2, uid, str(tmp_path)), nprocs=2, start_method="spawn")
    spec = snn.topology(n_columns=NCOL)
    plans = [snn.shard_plan(spec, r, 2) for r in range(2)]
    rasters = [np.load(tmp_path / f"raster{r}.npy") for r in range(2)]
    corpus = snn.stream(20000, seed=7)
    orc = po.Oracle2e(po.ref_params(NCOL, phase_offset=PHASE), corpus)
    total = 0
    for k in range(STEPS):
        orc.run(1)
        sp = orc.spikes()
        total += int(sp.sum())
        for r, p in enumerate(plans):
            want = np.concatenate([sp[p["a0"]:p["a1"]], sp[p["pf0"]:p["pf1"]]])
            got = np.unpackbits(rasters[r][k].view(np.uint8), bitorder="little")[: p["n_local"]]
            if not np.array_equal(got, want):
                raise AssertionError(f"rank {r}: raster differs at step {k}: "
                                     f"{np.nonzero(got != want)[0][:10]}")
    assert total > 0
    names = {"V": "V", "w": "w", "fr": "fr", "nmda_cur": "nmda_cur"}
    for r, p in enumerate(plans):
        for mine, theirs in names.items():
            full = orc.neuron(theirs)
            want = np.concatenate([full[p["a0"]:p["a1"]], full[p["pf0"]:p["pf1"]]])
            got = np.load(tmp_path / f"{mine}{r}.npy")
            assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32)), \
                f"rank {r}: {mine}"
        nxt = orc.next_input()
        want = np.concatenate([nxt[p["a0"]:p["a1"]], nxt[p["pf0"]:p["pf1"]]])
        assert np.array_equal(np.load(tmp_path / f"input{r}.npy").view(np.uint32),
                              want.astype(np.float32).view(np.uint32)), f"rank {r}: next input"
        with open(tmp_path / f"counters{r}.json") as fh:
            c = json.load(fh)
        assert c["total_spikes"] == total  # global on every rank
    oc = orc.counters()
    cs = [json.load(open(tmp_path / f"counters{r}.json")) for r in range(2)]
    assert sum(c["arrivals"] for c in cs) == oc.arrived
    # every (pre spike, synapse) dispatch is counted once, on the rank of the synapse's post
    assert sum(c["dispatched"] for c in cs) == oc.dispatched
