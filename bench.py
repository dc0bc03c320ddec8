#!/usr/bin/env python3
"""Stage 2e simulation throughput on B200 (55,000 AdEx neurons / 10,700,000
synapses, the reference network), as one JSON line.

A step is one full simulate -> inject-byte -> learn step of the network
(AdEx + NMDA/Ca + STP + dual-trace PSW STDP + CaMKII / eligibility + delays +
gate / modulators / inhibition), on a seeded synthetic Chinese-like UTF-8
stream (p_CJK = 0.452, the `ref45` preset), with the phase table shifted into
the SYNAPTOGENIC phase (plasticity gain 1) so that learning is active.

  value      synaptic events / s (delivered pre-spike x synapse arrivals),
             device-timed with CUDA events on the engine's stream, inputs
             resident in HBM
  e2e        the same metric through the C ABI (snn_run) with host buffers:
             every step's input bytes copied from pinned host memory and every
             step's spike raster + spike count copied back, wall clock
  roofline   the synapse pass (dominant kernel): algorithmic bytes per launch
             / its mean CUDA-event duration, against MEASURED_PEAKS.json

--impl reference times the CPU oracle (the reference has no CPU path; the
oracle is the restatement of its step) on the host cores.

Multi-GPU: one process per GPU; Stage 2e at this size runs one independent
network replica per GPU ("replicas", weak scaling), value = sum over ranks,
time = max over ranks.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "pure-snn-language_b200"))

METRIC = "synaptic events/sec (SOPS) and sim steps/sec, Stage-2e 55k/10.7M, 1–8 B200"
UNIT = "events/s"
PHASE_OFFSET = 5000      # SYNAPTOGENIC: plasticity gain 1
STREAM_SEED = 42
P_CJK = 0.452


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()  # let the sampler start before the timed region
            while not self.rows and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.02)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for k, n in enumerate(names):
                    if r[5 + k].lower().startswith("active"):
                        reasons.add(n)
            except (ValueError, IndexError):
                pass
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def profile_traffic(name, key="traffic_bytes_per_launch"):
    """A DRAM traffic figure (read + write) recorded from an ncu capture in
    profiles/<name> as `<key> = N`, or None."""
    import re
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    m = re.search(key + r"\s*=\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


def synapse_pass_bytes(S, S_exc, d_arr, d_disp, d_ltp, steps, first_step):
    """Algorithmic HBM bytes of the synapse pass over `steps` steps (see
    DESIGN.md, 'Byte model'): group id 4*S + Ca read/write 8*S_exc every
    step; per dispatched edge 12 (alpha, beta read; value write), per arrival
    36 (value read; plasticity record read/write), per LTP visit 32; every 10
    steps eligibility 8*S + e1/e2 16*S + CaMKII 16*S_exc; every 1000 steps
    alpha/beta 16*S."""
    n10 = sum(1 for t in range(first_step, first_step + steps) if t % 10 == 0)
    n1000 = sum(1 for t in range(first_step, first_step + steps) if t % 1000 == 0)
    dense = steps * (4.0 * S + 8.0 * S_exc)
    periodic = n10 * (24.0 * S + 16.0 * S_exc) + n1000 * 16.0 * S
    events = 12.0 * d_disp + 36.0 * d_arr + 32.0 * d_ltp
    return dense + periodic + events


def make_net(snn, device, raster_steps=1024):
    net = snn.Network(device=device, phase_offset=PHASE_OFFSET, raster_steps=raster_steps)
    net.build_columns(snn.topology(n_columns=50))
    return net


def cpu_baseline(warmup, budget_s=12.0, threads=0):
    """CPU oracle on a bounded sample of the same workload (all host cores)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    import snn_b200 as snn
    corpus = snn.stream(1 << 20, seed=STREAM_SEED, p_cjk=P_CJK)
    cores = threads or os.cpu_count()
    o = po.Oracle2e(po.ref_params(50, phase_offset=PHASE_OFFSET, n_threads=cores), corpus)
    o.run(warmup)
    c0 = o.counters()
    t0 = time.perf_counter()
    n = 0
    while n < 5 or time.perf_counter() - t0 < budget_s:
        o.run(1)
        n += 1
    dt = time.perf_counter() - t0
    c1 = o.counters()
    o.close()
    ev = c1.arrived - c0.arrived
    return {"value": ev / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "steps_per_sec": n / dt,
            "sample": f"{n} steps (after {warmup} warm-up) of the 55k/10.7M network, "
                      f"CPU oracle, {cores} OpenMP threads"}


PROP_RATES = (0.001, 0.01, 0.03, 0.1)
PROP_MODES = ((0, "STDP off"), (1, "STDP on"), (2, "STP on"))


def prop_push_bytes(events, pre_spikes, mode):
    """Algorithmic HBM bytes of the push kernel: post + weight streams (8 B
    per event), the spike list (4 B per spiker, +4 release with STP), the
    LTD weight write-back (4 B per event of the 80 % excitatory pres)."""
    b = 8.0 * events + 4.0 * pre_spikes
    if mode & 2:
        b += 4.0 * pre_spikes
    if mode & 1:
        b += 4.0 * 0.8 * events
    return b


def prop_cpu_baseline(rate, budget_s=10.0):
    """CPU oracle of the microbench (plain propagation, 1 M x 1,000) timed on
    all host cores for a bounded number of steps."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    cores = os.cpu_count()
    o = po.Oracle4(po.prop_params(n=1_000_000, fanout=1000, rate=rate, mode=0, n_threads=cores))
    o.run(3)
    c0 = o.counters()
    t0 = time.perf_counter()
    n = 0
    while n < 5 or time.perf_counter() - t0 < budget_s:
        o.run(1)
        n += 1
    dt = time.perf_counter() - t0
    ev = o.counters()["events"] - c0["events"]
    o.close()
    return {"value": ev / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} steps of the 1M x 1,000 microbench at rate {rate} (STDP off), "
                      f"CPU oracle, {cores} OpenMP threads"}


def prop_main(args):
    """Propagation microbench: one JSON line per (mode, rate).  Under torchrun
    the network is sharded by post bucket over the ranks (one GPU each; the
    forced pre-spikes are drawn on every rank, so nothing is exchanged during
    the run): strong scaling, device time max over ranks, events summed."""
    import datetime
    import snn_b200 as snn
    import torch
    import torch.distributed as tdist
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        tdist.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    torch.cuda.set_device(local)
    warm = max(args.warmup, 3)
    peak, peak_kind = measured_peaks()
    cb = None if args.no_cpu_baseline or world > 1 else prop_cpu_baseline(0.01)
    rates = [float(x) for x in args.prop_rates.split(",")] if args.prop_rates else PROP_RATES
    modes = [m for m in PROP_MODES if not args.prop_modes or str(m[0]) in args.prop_modes.split(",")]
    n_neu = args.prop_neurons
    # ncu: DRAM bytes per event of the bucketed push (plain propagation)
    traffic_per_event = profile_traffic("k4_push_b_propagation_1M.md", "traffic_bytes_per_event")
    for mode, mname in modes:
        for rate in rates:
            net = snn.Network(device=local, model=snn.MODEL_PROP, prop_mode=mode, prop_rate=rate)
            if world > 1:
                net.set_shard(rank, world)
            net.build_columns(snn.topology(snn.MODEL_PROP, l4=n_neu))
            net.run(warm)
            net.synchronize()
            c0 = net.counters()
            torch.cuda.synchronize()
            net.set_profiling(True)
            if world > 1:
                tdist.barrier()
            with ClockSampler(local) as clk:
                net.run(args.steps)
                net.synchronize()
            prof = net.profile()
            net.set_profiling(False)
            c1 = net.counters()
            ev = c1["arrivals"] - c0["arrivals"]
            pre = c1["dispatched"] - c0["dispatched"]
            dev_s = prof["step_ms"] / 1000.0
            pname = next(k for k in prof["kernels"] if k.startswith("k4_push"))
            push = prof["kernels"][pname]
            push_s = push["ms"] / push["launches"] / 1000.0
            pb = prop_push_bytes(ev, pre, mode) / args.steps
            achieved = pb / push_s / 1e9
            # end to end: snn_run with the spike raster copied to pinned host memory
            raster = torch.empty((args.steps, net.words), dtype=torch.int32, pin_memory=True)
            ce0 = net.counters()
            torch.cuda.synchronize()
            if world > 1:
                tdist.barrier()
            t0 = time.perf_counter()
            net._check(net.L.snn_run(net.h, args.steps, None, 0, 1, raster.data_ptr(), None))
            net.synchronize()
            wall = time.perf_counter() - t0
            e2e_ev = net.counters()["arrivals"] - ce0["arrivals"]
            post_sp = c1["total_spikes"] - c0["total_spikes"]
            ltp_v = c1["ltp_visits"] - c0["ltp_visits"]
            if world > 1:  # device time and wall time: max over ranks; events: sum
                tv = torch.tensor([dev_s, wall, push_s], dtype=torch.float64)
                te = torch.tensor([ev, e2e_ev, post_sp, ltp_v], dtype=torch.float64)
                tdist.all_reduce(tv, op=tdist.ReduceOp.MAX)
                tdist.all_reduce(te, op=tdist.ReduceOp.SUM)
                dev_s, wall, push_s = (float(x) for x in tv)
                ev, e2e_ev, post_sp, ltp_v = (float(x) for x in te)
                pb = prop_push_bytes(ev, pre * world, mode) / args.steps / world  # per rank
                achieved = pb / push_s / 1e9
            if rank != 0:
                net.close()
                continue
            line = {
                "metric": f"synaptic events/sec (SOPS), propagation microbench {n_neu:,} x 1,000",
                "value": ev / dev_s, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": warm, "ms_per_step": dev_s * 1000.0 / args.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f32 weights, int32 fixed-point sums",
                "data": "synthetic (seeded forced Poisson pre-spikes)",
                "config": {"workload": f"propagation microbench, {n_neu:,} LIF x fan-out 1,000 "
                                       f"({n_neu * 1000 / 1e9:.1f}B synapses), rate {rate}, {mname}",
                           "rate": rate, "mode": mname,
                           "events_per_step": ev / args.steps,
                           "post_spikes_per_step": post_sp / args.steps,
                           "ltp_visits_per_step": ltp_v / args.steps,
                           "parallelism": f"post-bucket shards x{world}" if world > 1 else "1 GPU",
                           "exchange": "none during the run (forced pre-spikes drawn on every rank)",
                           "l2": f"inputs larger than L2 ({n_neu * 8e-6:.1f} GB of synapse streams)"},
                "e2e": {"value": e2e_ev / wall, "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": net.words * 4},
                "gpu_launches": int(sum(v["launches"] for v in prof["kernels"].values())),
                "kernels_ms_per_step": {k: v["ms"] / max(v["launches"], 1)
                                        for k, v in prof["kernels"].items()},
                "roofline": {"bound": "hbm", "kernel": pname, "achieved": achieved,
                             "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                             "peak_kind": peak_kind, "bytes_per_launch": pb,
                             "traffic": traffic_per_event * ev / args.steps / world
                             if pname == "k4_push_b" and mode == 0 and traffic_per_event else None},
                "clocks": clk.summary(),
            }
            if cb:
                line["cpu_baseline"] = cb
            print(json.dumps(line), flush=True)
            net.close()
    if world > 1:
        tdist.barrier()
        tdist.destroy_process_group()


def stage0_main(args):
    """Configurations 0 and 1 (Stage 0 block network, Stage 2A columnar
    network), benchmark constants: one JSON line each."""
    import snn_b200 as snn
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    warm = max(args.warmup, 3)
    for columnar in (False, True):
        name = ("stage2A columnar 10 x 1,000 LIF / 1M synapses, synthetic UTF-8 (p_CJK 0.85)"
                if columnar else "stage0 10,000 LIF / 1M synapses, uniform random bytes")
        if columnar:
            data = snn.stream(1 << 20, seed=STREAM_SEED, p_cjk=0.85)
        else:
            data = np.random.default_rng(STREAM_SEED).integers(0, 256, 1 << 20).astype(np.uint8)
        net = snn.Network(model=snn.MODEL_STAGE0, preset=snn.PRESET_BASELINE)
        net.build_columns(snn.topology(snn.MODEL_STAGE0, n_columns=10 if columnar else 0))
        net.set_corpus(data.tobytes())
        net.run(warm)
        net.synchronize()
        c0 = net.counters()
        net.set_profiling(True)
        with ClockSampler(0) as clk:
            net.run(args.steps)
            net.synchronize()
        prof = net.profile()
        net.set_profiling(False)
        c1 = net.counters()
        ev = c1["dispatched"] - c0["dispatched"]
        dev_s = prof["step_ms"] / 1000.0
        # e2e: the input bytes copied from pinned host memory with the call
        pin = torch.empty(args.steps, dtype=torch.uint8, pin_memory=True)
        pin.numpy()[:] = data[: args.steps]
        ce0 = net.counters()
        t0 = time.perf_counter()
        net._check(net.L.snn_run(net.h, args.steps, pin.data_ptr(), args.steps, 1, None, None))
        net.synchronize()
        wall = time.perf_counter() - t0
        e2e_ev = net.counters()["dispatched"] - ce0["dispatched"]
        line = {
            "metric": "synaptic events/sec (SOPS) and sim steps/sec, " + name,
            "value": ev / dev_s, "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": warm,
            "ms_per_step": prof["step_ms"] / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "steps_per_sec": args.steps / dev_s,
            "config": {"workload": name, "constants": "benchmark (baseline preset)",
                       "events_per_step": ev / args.steps,
                       "l2": "L2-resident (1M synapses)"},
            "e2e": {"value": e2e_ev / wall, "unit": UNIT, "h2d_bytes_per_step": 1,
                    "d2h_bytes_per_step": 0, "steps_per_sec": args.steps / wall},
            "gpu_launches": int(sum(v["launches"] for v in prof["kernels"].values())),
            "kernels_ms_per_step": {k: v["ms"] / max(v["launches"], 1) for k, v in prof["kernels"].items()},
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline:
            cores = os.cpu_count()
            o = po.Oracle0(po.stage0_params(columnar=columnar, baseline=True, n_threads=cores))
            o.run(warm, data[:warm])
            s0 = o.sizes()
            t0, n = time.perf_counter(), 0
            while n < 50 or time.perf_counter() - t0 < 8.0:
                o.run(10, data[warm + n: warm + n + 10])
                n += 10
            dt = time.perf_counter() - t0
            s1 = o.sizes()
            deg = int(s1[1] // s1[0])
            line["cpu_baseline"] = {"value": float(s1[3] - s0[3]) * deg / dt, "unit": UNIT,
                                    "cores": cores, "kind": "port",
                                    "sample": f"{n} steps, CPU oracle, {cores} OpenMP threads"}
            o.close()
        print(json.dumps(line), flush=True)
        net.close()


def shard_main(args):
    """Configuration 3: the Stage 2e network scaled to --columns columns
    (5,000: 5.5 M neurons / 1.07 B synapses), sharded by column over the
    torchrun ranks (one GPU each), NCCL all-gather of the spike bitmask every
    step.  Strong scaling: the network is the same at every rank count."""
    import datetime
    import torch
    import torch.distributed as tdist
    import snn_b200 as snn
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    warm = max(args.warmup, 3)
    if world > 1:
        tdist.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    torch.cuda.set_device(local)
    uid = [snn.nccl_unique_id() if rank == 0 else None]
    if world > 1:
        tdist.broadcast_object_list(uid, src=0)
    t_build = time.perf_counter()
    net = snn.Network(device=local, phase_offset=PHASE_OFFSET, raster_steps=256)
    net.set_shard(rank, world, uid[0] if world > 1 else None)
    net.build_columns(snn.topology(n_columns=args.columns))
    net.set_corpus(snn.stream(1 << 20, seed=STREAM_SEED, p_cjk=P_CJK))
    build_s = time.perf_counter() - t_build
    net.run(warm)
    net.synchronize()
    c0 = net.counters()
    if world > 1:
        tdist.barrier()
    net.set_profiling(True)
    with ClockSampler(local) as clk:
        net.run(args.steps)
        net.synchronize()
    prof = net.profile()
    net.set_profiling(False)
    c1 = net.counters()
    arr = float(c1["arrivals"] - c0["arrivals"])
    dev_ms = prof["step_ms"]
    # e2e: snn_run with the rank's raster rows copied to pinned host memory
    e2e_steps = min(args.e2e_steps, 200)
    raster = torch.empty((e2e_steps, net.words), dtype=torch.int32, pin_memory=True)
    net.run(50)  # untimed: re-instantiates the step graph after profiling
    net.synchronize()
    ce0 = net.counters()
    if world > 1:
        tdist.barrier()
    t0 = time.perf_counter()
    net._check(net.L.snn_run(net.h, e2e_steps, None, 0, 1, raster.data_ptr(), None))
    net.synchronize()
    wall = time.perf_counter() - t0
    e2e_arr = float(net.counters()["arrivals"] - ce0["arrivals"])
    v = torch.tensor([dev_ms, wall, build_s], dtype=torch.float64)
    e = torch.tensor([arr, e2e_arr, float(net.S)], dtype=torch.float64)
    if world > 1:
        tdist.all_reduce(v, op=tdist.ReduceOp.MAX)
        tdist.all_reduce(e, op=tdist.ReduceOp.SUM)
    dev_ms, wall, build_s = (float(x) for x in v)
    arr_all, e2e_all, syn_all = (float(x) for x in e)
    if rank == 0:
        peak, peak_kind = measured_peaks()
        line = {
            "metric": "synaptic events/sec (SOPS) and sim steps/sec, Stage-2e 5.5M/1.07B column-sharded",
            "value": arr_all / (dev_ms / 1000.0), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded UTF-8 stream, ref45 preset)",
            "steps_per_sec": args.steps / (dev_ms / 1000.0),
            "config": {"workload": f"stage2e {args.columns:,} columns ({args.columns * 1100:,} neurons / "
                                   f"{int(syn_all):,} synapses), column-sharded over {world} GPU(s), "
                                   "SYNAPTOGENIC phase",
                       "columns": args.columns, "parallelism": f"column shards x{world}",
                       "exchange": "NCCL all-gather of spike words + counts every step",
                       "events_per_step": arr_all / args.steps, "build_s": build_s,
                       "l2": "inputs larger than L2"},
            "e2e": {"value": e2e_all / wall, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": net.words * 4},
            "gpu_launches": int(sum(k["launches"] for n, k in prof["kernels"].items() if "@" not in n)),
            "kernels_ms_per_step_rank0": {k: x["ms"] / max(x["launches"], 1)
                                          for k, x in prof["kernels"].items()},
            "clocks": clk.summary(),
            "peak_hbm_gbs": peak, "peak_kind": peak_kind,
        }
        print(json.dumps(line), flush=True)
    net.close()
    if world > 1:
        tdist.barrier()
        tdist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=1000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="stage2e", choices=["stage2e", "prop", "shard", "stage0"],
                    help="stage2e: the 55k/10.7M network (one line); prop: the 1M x 1,000 "
                         "propagation microbench (one line per mode and rate; post-bucket shards over the "
                         "torchrun ranks); shard: "
                         "the 100x network column-sharded over the torchrun ranks; stage0: "
                         "configurations 0 and 1 (one line each, 1 GPU)")
    ap.add_argument("--columns", type=int, default=5000, help="shard workload: columns")
    ap.add_argument("--prop-neurons", type=int, default=1_000_000)
    ap.add_argument("--prop-rates", default="", help="comma list, default 0.001,0.01,0.03,0.1")
    ap.add_argument("--prop-modes", default="", help="comma list of 0 (STDP off), 1 (STDP on), 2 (STP on)")
    args = ap.parse_args()
    warm = max(args.warmup, 3)
    if args.workload == "prop":
        prop_main(args)
        return
    if args.workload == "shard":
        shard_main(args)
        return
    if args.workload == "stage0":
        stage0_main(args)
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import torch
        import torch.distributed as tdist
        import datetime
        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local))
        dist = tdist

    if args.impl == "reference":
        if rank == 0:
            cb = cpu_baseline(warm)
            line = {"metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus,
                    "steps": args.steps, "warmup": warm,
                    "ms_per_step": 1000.0 / cb["steps_per_sec"], "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                    "data": "synthetic (seeded UTF-8 stream, ref45)", "impl": "reference",
                    "config": {"workload": "stage2e 55k neurons / 10.7M synapses, ref constants",
                               "phase": "SYNAPTOGENIC (gain 1)"},
                    "cpu_baseline": cb,
                    "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        if dist:
            dist.destroy_process_group()
        return

    import snn_b200 as snn
    import torch
    torch.cuda.set_device(local)
    corpus = snn.stream(1 << 20, seed=STREAM_SEED + rank, p_cjk=P_CJK)
    net = make_net(snn, local)
    net.set_corpus(corpus)
    # warm-up (also fills the network with activity)
    net.run(warm)
    net.synchronize()
    c0 = net.counters()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    # timed region: one CUDA event pair on the engine stream around the K steps
    net.set_profiling(2)
    with ClockSampler(local) as clk:
        net.run(args.steps)
        net.synchronize()
    torch.cuda.synchronize()
    dev_ms = net.profile()["step_ms"]
    net.set_profiling(False)
    c1 = net.counters()
    arr = c1["arrivals"] - c0["arrivals"]
    # per-kernel breakdown (events around every kernel) on the next steps, for
    # the roofline of the synapse pass
    kp_steps = min(args.steps, 1000)
    first = c1["step"]
    net.set_profiling(True)
    net.run(kp_steps)
    net.synchronize()
    prof = net.profile()
    net.set_profiling(False)
    c2 = net.counters()
    kp_arr = c2["arrivals"] - c1["arrivals"]
    disp = c2["dispatched"] - c1["dispatched"]
    ltp = c2["ltp_visits"] - c1["ltp_visits"]
    # max over ranks of the device time, sum of events
    if dist:
        t = torch.tensor([dev_ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e = torch.tensor([float(arr)], device="cuda", dtype=torch.float64)
        dist.all_reduce(e, op=dist.ReduceOp.SUM)
        dev_ms_max, arr_all = float(t.item()), float(e.item())
    else:
        dev_ms_max, arr_all = dev_ms, float(arr)
    value = arr_all / (dev_ms_max / 1000.0)
    steps_per_sec = args.steps / (dev_ms_max / 1000.0)

    # roofline of the synapse pass
    flags = net.state("flags")
    S = net.S
    S_exc = int(np.count_nonzero(flags & 0x03))
    k4 = prof["kernels"]["k_synapses"]
    k4_bytes = synapse_pass_bytes(S, S_exc, kp_arr, disp, ltp, kp_steps, first) / kp_steps
    k4_ms = k4["ms"] / k4["launches"]
    peak, peak_kind = measured_peaks()
    achieved = k4_bytes / (k4_ms / 1000.0) / 1e9
    traffic = profile_traffic("k_synapses_stage2e_55k.md")

    # end to end through the C ABI, host buffers
    e2e_steps = args.e2e_steps
    n_bytes = (e2e_steps + 2) // 3
    pin = torch.empty(n_bytes, dtype=torch.uint8, pin_memory=True)
    pin.numpy()[:] = snn.stream(n_bytes, seed=STREAM_SEED + 1000 + rank, p_cjk=P_CJK)
    raster = torch.empty((e2e_steps, net.words), dtype=torch.int32, pin_memory=True)
    counts = torch.empty(e2e_steps, dtype=torch.int32, pin_memory=True)
    ce0 = net.counters()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = net.L.snn_run(net.h, e2e_steps, pin.data_ptr(), n_bytes, 1, raster.data_ptr(),
                       counts.data_ptr())
    net._check(rc)
    net.synchronize()
    wall = time.perf_counter() - t0
    ce1 = net.counters()
    e2e_arr = ce1["arrivals"] - ce0["arrivals"]
    if dist:
        t = torch.tensor([wall], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e = torch.tensor([float(e2e_arr)], device="cuda", dtype=torch.float64)
        dist.all_reduce(e, op=dist.ReduceOp.SUM)
        wall, e2e_arr = float(t.item()), float(e.item())
    e2e = {"value": e2e_arr / wall, "unit": UNIT,
           "h2d_bytes_per_step": n_bytes / e2e_steps,
           "d2h_bytes_per_step": net.words * 4 + 4,
           "steps_per_sec": e2e_steps / wall}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": warm, "ms_per_step": dev_ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded UTF-8 stream, ref45 preset)",
            "steps_per_sec": steps_per_sec,
            "config": {"workload": "stage2e 55k neurons / 10.7M synapses (reference network), "
                                   "ref constants, SYNAPTOGENIC phase",
                       "n_neurons": net.N, "n_synapses": S,
                       "parallelism": "replicas" if world > 1 else "single",
                       "l2": "inputs larger than L2 (synapse state ~0.73 GB per GPU)",
                       "events_per_step": arr / args.steps},
            "e2e": e2e,
            # kernels per step (the "@" slot repeats k_synapses) x timed steps
            "gpu_launches": sum(1 for n in prof["kernels"] if "@" not in n) * args.steps,
            "kernels_ms_per_step": {k: v["ms"] / max(v["launches"], 1)
                                    for k, v in prof["kernels"].items()},
            "roofline": {"bound": "hbm", "kernel": "k_synapses", "achieved": achieved,
                         "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "bytes_per_launch": k4_bytes,
                         "traffic": traffic},
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(warm)
        print(json.dumps(line), flush=True)
    net.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
