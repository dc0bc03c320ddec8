"""Host logic of column sharding, on CPU with world_size-2 gloo ranks: each
rank computes its partition plan of a Stage 2e topology (snn_shard_plan, the
same code the engine runs before building its shard) and the ranks check
together that the plans tile the network exactly."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_main(rank, world, port, ncol, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import snn_b200 as snn
    spec = snn.topology(n_columns=ncol)
    p = snn.shard_plan(spec, rank, world)
    full = snn.shard_plan(spec, 0, 1)
    v = torch.tensor([p["n_local"], p["synapses"], p["groups_local"] + p["groups_mirror"]],
                     dtype=torch.int64)
    dist.all_reduce(v)
    ranges = [None] * world
    dist.all_gather_object(ranges, (p["a0"], p["a1"], p["pf0"], p["pf1"]))
    # neurons and synapses are split exactly; a (pre, delay, class) group whose
    # synapses land on several ranks exists once per rank (local or mirror)
    ok = (int(v[0]) == full["n_local"] and int(v[1]) == full["synapses"]
          and int(v[2]) >= full["groups_local"] and p["mirror_pres"] > 0)
    # the neuron ranges of the ranks tile [0, N) without overlap
    covered = np.zeros(full["n_local"], np.int32)
    for a0, a1, pf0, pf1 in ranges:
        covered[a0:a1] += 1
        covered[pf0:pf1] += 1
    ok = ok and bool((covered == 1).all())
    np.save(os.path.join(out_dir, f"ok{rank}.npy"), np.array([int(ok), p["remote_short_delay"]]))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,ncol", [(2, 8), (2, 11)])
def test_shard_plans_tile_the_network(tmp_path, world, ncol):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "pure-snn-language_b200"))
    mp.start_processes(rank_main, args=(world, free_port(), ncol, str(tmp_path)), nprocs=world,
                       start_method="spawn")
    for r in range(world):
        ok, short = np.load(tmp_path / f"ok{r}.npy")
        assert ok == 1, f"rank {r}: plan does not tile the network"
