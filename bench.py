#!/usr/bin/env python3
"""Throughput of the B200 spiking-network core, one JSON line per run.

Workloads (selected automatically, or with --workload):

  stage2e  (plain `python bench.py`, one GPU) the reference's Stage 2e network:
           55,000 AdEx neurons / 10,700,000 synapses in 50 columns, reference
           constants, phase table shifted into SYNAPTOGENIC (plasticity gain
           1), seeded synthetic Chinese-like UTF-8 stream (`ref45` preset,
           seed 42).  A step is one full simulate -> inject-byte -> learn step
           (AdEx + NMDA/Ca + STP + dual-trace PSW STDP + CaMKII / eligibility
           + delays + gate / modulators / inhibition).
  shard    (under torchrun, every N including 1, or --gpus N > 1) the same
           layering scaled to 5,000 columns (5,500,000 neurons / 1.07 B
           synapses), sharded by column over the ranks, one GPU each, with an
           NCCL all-gather of the spike words every step (strong scaling).
  prop     the 1 M x 1,000 propagation microbench (one line per mode / rate).
  stage0   the Stage 0 / Stage 2A networks (one line each).

Every timed quantity of a line covers the same steps: a fresh network, W
warm-up steps, then the window of K steps.

  value      synaptic events / s (delivered pre-spike x synapse arrivals) over
             the window, device time (one CUDA event pair on the engine's
             stream), inputs resident in HBM
  e2e        the same window through the C ABI (snn_run) from a checkpoint of
             the state after the warm-up: every step's input byte copied from
             pinned host memory, every step's spike raster and count read
             back, wall clock (stage2e; the shard workload times the K steps
             after the window)
  roofline   the synapse pass (dominant kernel): algorithmic bytes per launch
             over the window / its mean CUDA-event duration over the window,
             against MEASURED_PEAKS.json
  cpu_baseline  the CPU oracle (the reference has no CPU path; the oracle is
             the restatement of its step) on the host cores, over the window
             (bounded), plus a bounded single-thread leg
  reference_gpu  the reference's own Stage 2e scheduler, compiled unmodified
             for sm_100a (oracle/_ref/ref_run), timed on the same GPU

--impl reference times the CPU oracle over the same window and prints the
same config; it loads no library of the product.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "pure-snn-language_b200")
ORACLE = os.path.join(ROOT, "oracle")

METRIC = "synaptic events/sec (SOPS) and sim steps/sec, Stage-2e 55k/10.7M, 1–8 B200"
UNIT = "events/s"
PHASE_OFFSET = 5000      # SYNAPTOGENIC: plasticity gain 1
STREAM_SEED = 42
STREAMS = {"ref45": 0.452, "b85": 0.85}
CORPUS_BYTES = 1 << 20
SHARD_COLUMNS = 5000
SHARD_SAMPLE_COLUMNS = 250   # CPU oracle sample of the sharded network (host memory)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torchrun = "TORCHELASTIC_RUN_ID" in os.environ or "LOCAL_WORLD_SIZE" in os.environ
    return rank, world, local, torchrun


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


def host_cpu_info():
    """CPU model, sockets, physical cores, logical CPUs, NUMA nodes and the
    CPUs this process may run on."""
    model, phys = None, set()
    sock, core = None, None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                k, _, v = line.partition(":")
                k, v = k.strip(), v.strip()
                if k == "model name" and model is None:
                    model = v
                elif k == "physical id":
                    sock = v
                elif k == "core id":
                    core = v
                elif not k and sock is not None:
                    phys.add((sock, core))
                    sock = core = None
        if sock is not None:
            phys.add((sock, core))
    except OSError:
        pass
    numa = 0
    try:
        numa = len([d for d in os.listdir("/sys/devices/system/node") if d.startswith("node")
                    and d[4:].isdigit()])
    except OSError:
        pass
    try:
        usable = len(os.sched_getaffinity(0))
    except AttributeError:
        usable = os.cpu_count()
    return {"model": model, "sockets": len({s for s, _ in phys}) or None,
            "physical_cores": len(phys) or None, "logical_cpus": os.cpu_count(),
            "numa_nodes": numa or None, "usable_cpus": usable}


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
    """Algorithmic HBM bytes of the Stage 2e synapse pass over `steps` steps
    from `first_step`: group id 4*S + Ca read/write 8*S_exc every step; per
    dispatched edge 12 (alpha, beta read; value write), per arrival 36 (value
    read; plasticity record read/write), per LTP visit 32; every 10 steps
    eligibility 8*S + e1/e2 16*S + CaMKII 16*S_exc; every 1000 steps
    alpha/beta 16*S."""
    n10 = sum(1 for t in range(first_step, first_step + steps) if t % 10 == 0)
    n1000 = sum(1 for t in range(first_step, first_step + steps) if t % 1000 == 0)
    dense = steps * (4.0 * S + 8.0 * S_exc)
    periodic = n10 * (24.0 * S + 16.0 * S_exc) + n1000 * 16.0 * S
    events = 12.0 * d_disp + 36.0 * d_arr + 32.0 * d_ltp
    return dense + periodic + events


def window_bytes(corpus, warm, steps, interval=3):
    """The corpus bytes that the window [warm, warm + steps) injects (one byte
    per step with t % interval == 0, read in order from the start)."""
    pos = (warm + interval - 1) // interval
    n = sum(1 for t in range(warm, warm + steps) if t % interval == 0)
    idx = (pos + np.arange(n)) % corpus.size
    return np.ascontiguousarray(corpus[idx])


def stream_label(name, classes):
    return (f"synthetic UTF-8 stream `{name}` (seed {STREAM_SEED}, p_CJK {STREAMS[name]}): "
            f"ASCII {classes['ascii']:.4f}, lead {classes['head']:.4f}, "
            f"continuation {classes['continuation']:.4f} of its bytes")


def stage2e_config(warm, steps, stream_name, world=1):
    return {"workload": "stage2e 55,000 neurons / 10,700,000 synapses (reference network, "
                        "50 columns), ref constants, SYNAPTOGENIC phase (phase offset 5000)",
            "n_neurons": 55000, "n_synapses": 10700000, "stream": stream_name,
            "window": f"steps {warm}..{warm + steps - 1} of a fresh network",
            "parallelism": f"replicas x{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (synapse state ~0.73 GB)"}


def shard_config(warm, steps, columns, world):
    return {"workload": f"stage2e {columns:,} columns ({columns * 1100:,} neurons / "
                        f"{10_700_000 * columns // 50:,} synapses), column-sharded, "
                        "SYNAPTOGENIC phase (phase offset 5000)",
            "columns": columns, "stream": "ref45",
            "window": f"steps {warm}..{warm + steps - 1} of a fresh network",
            "parallelism": f"column shards x{world}",
            "exchange": "NCCL all-gather of spike words + counts every step",
            "l2": "inputs larger than L2"}


# ---------------------------------------------------------------------------
# CPU oracle legs (test infrastructure: the oracle library only)
# ---------------------------------------------------------------------------
def oracle_window(columns, warm, steps, stream_name, threads, budget_s=None, min_steps=3):
    """The CPU oracle of the Stage 2e network run for `warm` steps, then timed
    over up to `steps` steps (fewer once `budget_s` seconds are spent, at least
    `min_steps`).  Returns (events, seconds, steps timed, build seconds)."""
    sys.path.insert(0, ORACLE)
    import pyoracle as po
    corpus = po.stream(CORPUS_BYTES, seed=STREAM_SEED, p_cjk=STREAMS[stream_name])
    t_b = time.perf_counter()
    o = po.Oracle2e(po.ref_params(columns, phase_offset=PHASE_OFFSET, n_threads=threads), corpus)
    build_s = time.perf_counter() - t_b
    o.run(warm)
    c0 = o.counters()
    t0 = time.perf_counter()
    n = 0
    while n < steps:
        o.run(1)
        n += 1
        if budget_s is not None and n >= min_steps and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    ev = o.counters().arrived - c0.arrived
    o.close()
    return ev, dt, n, build_s


def cpu_baseline_stage2e(warm, steps, stream_name, columns=50, budget_s=20.0, st_budget_s=15.0):
    """OpenMP leg over the window (bounded) and a single-thread leg over its
    first steps (bounded)."""
    info = host_cpu_info()
    cores = info["usable_cpus"] or 1
    ev, dt, n, _ = oracle_window(columns, warm, steps, stream_name, cores, budget_s)
    ev1, dt1, n1, _ = oracle_window(columns, warm, steps, stream_name, 1, st_budget_s, 2)
    return {"value": ev / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "steps_per_sec": n / dt, "events_per_step": ev / n,
            "sample": f"steps {warm}..{warm + n - 1} of the window ({n} of {steps}), "
                      f"CPU oracle of the {columns}-column network, {cores} OpenMP threads",
            "single_thread": {"value": ev1 / dt1, "unit": UNIT, "cores": 1,
                              "steps_per_sec": n1 / dt1,
                              "sample": f"steps {warm}..{warm + n1 - 1}, one thread"},
            "host": info}


def reference_main(args, workload):
    """--impl reference: the CPU oracle on the host cores (all of them) over
    the same window and config as the product's line; loads no product
    library.  Under torchrun rank 0 alone runs it."""
    rank, world, _, _ = dist_env()
    if rank != 0:
        return
    warm = max(args.warmup, 3)
    info = host_cpu_info()
    cores = info["usable_cpus"] or 1
    if workload == "shard":
        cfg = shard_config(warm, args.steps, args.columns, world)
        sample_cols = min(SHARD_SAMPLE_COLUMNS, args.columns)
        ev, dt, n, build_s = oracle_window(sample_cols, warm, min(args.steps, 200), "ref45",
                                           cores, budget_s=60.0)
        sample = (f"steps {warm}..{warm + n - 1} of a {sample_cols}-column network built by the "
                  f"same rule ({sample_cols / args.columns:.0%} of the columns; the full "
                  f"{args.columns:,}-column oracle needs ~130 B of host memory per synapse), "
                  f"CPU oracle, {cores} OpenMP threads")
        metric = ("synaptic events/sec (SOPS) and sim steps/sec, Stage-2e 5.5M/1.07B "
                  "column-sharded")
        scaling, data = "strong", "synthetic UTF-8 stream `ref45`"
    else:
        cfg = stage2e_config(warm, args.steps, args.stream, world)
        ev, dt, n, build_s = oracle_window(50, warm, min(args.steps, 3000), args.stream, cores)
        sample = (f"steps {warm}..{warm + n - 1} of the 55k/10.7M network (the window), "
                  f"CPU oracle, {cores} OpenMP threads")
        metric, scaling = METRIC, "weak"
        sys.path.insert(0, ORACLE)
        import pyoracle as po
        data = stream_label(args.stream, po.byte_classes(
            po.stream(CORPUS_BYTES, seed=STREAM_SEED, p_cjk=STREAMS[args.stream])))
    value = ev / dt
    line = {"metric": metric, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": warm, "ms_per_step": dt * 1000.0 / n,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
            "data": data, "impl": "reference", "config": cfg,
            "steps_per_sec": n / dt, "events_per_step": ev / n,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample, "build_s": build_s, "host": info},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the reference's own GPU engine (speed bar on the same GPU)
# ---------------------------------------------------------------------------
def reference_gpu(warm, steps, corpus, gpu):
    exe = os.path.join(ORACLE, "_ref", "ref_run")
    if not os.path.exists(exe):
        return {"unavailable": "oracle/_ref/ref_run was not built (needs the reference sources)"}
    with tempfile.TemporaryDirectory() as td:
        cp = os.path.join(td, "corpus.bin")
        corpus.tofile(cp)
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(gpu))
        try:
            r = subprocess.run([exe, "--steps", str(steps), "--time", str(warm), "--step0",
                                str(PHASE_OFFSET + 10), "--corpus", cp],
                               capture_output=True, text=True, timeout=600, env=env, cwd=td)
        except subprocess.TimeoutExpired:
            return {"unavailable": "ref_run did not finish within 600 s"}
    vals = {}
    for line in r.stdout.splitlines():
        parts = line.split()
        if parts and parts[0] in ("REF_STEPS_PER_SEC", "REF_EVENTS_PER_SEC"):
            vals[parts[0]] = float(parts[1])
    if r.returncode != 0 or len(vals) < 2:
        return {"unavailable": f"ref_run exited {r.returncode}: {r.stderr.strip()[-200:]}"}
    return {"steps_per_sec": vals["REF_STEPS_PER_SEC"], "value": vals["REF_EVENTS_PER_SEC"],
            "unit": UNIT, "timed_steps": steps, "warmup": warm,
            "how": "the reference's BioMechanismScheduler::step host loop "
                   "(src/stage2e/scheduler.cu:485-676), sources compiled unmodified for sm_100a, "
                   f"fresh network, step numbers from {PHASE_OFFSET + 10} (SYNAPTOGENIC), same "
                   "corpus; its own dynamics (float atomics), so events per step differ slightly"}


# ---------------------------------------------------------------------------
# Stage 2e, one GPU (the headline)
# ---------------------------------------------------------------------------
def stage2e_main(args):
    sys.path.insert(0, PKG)
    import snn_b200 as snn
    import torch
    rank, world, local, _ = dist_env()
    dist = None
    if world > 1:  # replicas: one independent network per GPU
        import datetime
        import torch.distributed as tdist
        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local))
        dist = tdist
    torch.cuda.set_device(local)
    warm, K = max(args.warmup, 3), args.steps
    corpus = snn.stream(CORPUS_BYTES, seed=STREAM_SEED, p_cjk=STREAMS[args.stream])
    net = snn.Network(device=local, phase_offset=PHASE_OFFSET, raster_steps=1024)
    net.build_columns(snn.topology(n_columns=50))
    net.set_corpus(corpus)
    net.run(warm)
    net.synchronize()
    tmpdir = tempfile.mkdtemp(prefix="snnbench_", dir="/dev/shm" if os.path.isdir("/dev/shm") else None)
    ckpt = os.path.join(tmpdir, f"warm{rank}.ckpt")
    net.save(ckpt)
    c0 = net.counters()
    try:
        # (1) value: the window, one CUDA event pair on the engine stream
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        net.set_profiling(2)
        with ClockSampler(local) as clk:
            net.run(K)
            net.synchronize()
        torch.cuda.synchronize()
        dev_ms = net.profile()["step_ms"]
        net.set_profiling(False)
        c1 = net.counters()
        arr = c1["arrivals"] - c0["arrivals"]
        # (2) the same window again with events around every kernel
        net.load(ckpt)
        net.set_profiling(True)
        net.run(K)
        net.synchronize()
        prof = net.profile()
        net.set_profiling(False)
        c2 = net.counters()
        kp = {k: c2[k] - c0[k] for k in ("arrivals", "dispatched", "ltp_visits")}
        # (3) e2e: the same window through snn_run with host buffers
        wb = window_bytes(corpus, warm, K)
        pin = torch.empty(max(wb.size, 1), dtype=torch.uint8, pin_memory=True)
        pin.numpy()[: wb.size] = wb
        raster = torch.empty((K, net.words), dtype=torch.int32, pin_memory=True)
        counts = torch.empty(K, dtype=torch.int32, pin_memory=True)
        walls, e2e_arr = [], None
        for rep in range(args.e2e_repeats + 1):  # the first call is an untimed warm-up
            net.load(ckpt)
            ce0 = net.counters()
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            rc = net.L.snn_run(net.h, K, pin.data_ptr(), wb.size, 1, raster.data_ptr(),
                               counts.data_ptr())
            net._check(rc)
            net.synchronize()
            wall = time.perf_counter() - t0
            if rep:
                walls.append(wall)
            e2e_arr = net.counters()["arrivals"] - ce0["arrivals"]
    finally:
        try:
            os.remove(ckpt)
            os.rmdir(tmpdir)
        except OSError:
            pass
    wall = float(np.median(walls))
    # max over ranks of the times, sum of the events
    if dist:
        t = torch.tensor([dev_ms, wall], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e = torch.tensor([float(arr), float(e2e_arr)], device="cuda", dtype=torch.float64)
        dist.all_reduce(e, op=dist.ReduceOp.SUM)
        dev_ms_max, wall = float(t[0]), float(t[1])
        arr_all, e2e_all = float(e[0]), float(e[1])
    else:
        dev_ms_max, arr_all, e2e_all = dev_ms, float(arr), float(e2e_arr)
    value = arr_all / (dev_ms_max / 1000.0)
    # roofline of the synapse pass over the window
    flags = net.state("flags")
    S = net.S
    S_exc = int(np.count_nonzero(flags & 0x03))
    ks = prof["kernels"]["k_synapses"]
    syn_bytes = synapse_pass_bytes(S, S_exc, kp["arrivals"], kp["dispatched"], kp["ltp_visits"],
                                   K, warm) / K
    syn_ms = ks["ms"] / ks["launches"]
    peak, peak_kind = measured_peaks()
    achieved = syn_bytes / (syn_ms / 1000.0) / 1e9
    traffic = profile_traffic("k_synapses_stage2e_55k.md")
    if rank == 0:
        classes = snn.byte_classes(corpus)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": K, "warmup": warm, "ms_per_step": dev_ms_max / K,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": stream_label(args.stream, classes),
            "config": stage2e_config(warm, K, args.stream, world),
            "steps_per_sec": K / (dev_ms_max / 1000.0),
            "events_per_step": arr / K,
            "e2e": {"value": e2e_all / wall, "unit": UNIT,
                    "h2d_bytes_per_step": wb.size / K,
                    "d2h_bytes_per_step": net.words * 4 + 4,
                    "steps_per_sec": K / wall, "events_per_step": e2e_arr / K,
                    "repeats": args.e2e_repeats,
                    "how": "snn_run over the window from the warm-up checkpoint, median wall time"},
            # two kernels per step (the "@" slot repeats k_synapses)
            "gpu_launches": sum(1 for n in prof["kernels"] if "@" not in n) * K,
            "kernels_ms_per_step": {k: v["ms"] / max(v["launches"], 1)
                                    for k, v in prof["kernels"].items()},
            "roofline": {"bound": "hbm", "kernel": "k_synapses", "achieved": achieved,
                         "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "bytes_per_launch": syn_bytes,
                         "launch_us": syn_ms * 1000.0, "traffic": traffic},
            "clocks": clk.summary(),
        }
        if arr != kp["arrivals"] or arr != e2e_arr:
            line["window_mismatch"] = {"value": arr, "kernels": kp["arrivals"], "e2e": e2e_arr}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_stage2e(warm, K, args.stream)
            line["reference_gpu"] = reference_gpu(warm, K, corpus, local)
        print(json.dumps(line), flush=True)
    net.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# configuration 3: the 5,000-column network, column-sharded (strong scaling)
# ---------------------------------------------------------------------------
def shard_main(args):
    import datetime
    sys.path.insert(0, PKG)
    import torch
    import torch.distributed as tdist
    import snn_b200 as snn
    rank, world, local, _ = dist_env()
    warm, K = max(args.warmup, 3), args.steps
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
    corpus = snn.stream(CORPUS_BYTES, seed=STREAM_SEED, p_cjk=STREAMS["ref45"])
    net.set_corpus(corpus)
    build_s = time.perf_counter() - t_build
    net.run(warm)
    net.synchronize()
    c0 = net.counters()
    if world > 1:
        tdist.barrier()
    torch.cuda.synchronize()
    net.set_profiling(2)
    with ClockSampler(local) as clk:
        net.run(K)
        net.synchronize()
    dev_ms = net.profile()["step_ms"]
    net.set_profiling(False)
    c1 = net.counters()
    arr = float(c1["arrivals"] - c0["arrivals"])
    # e2e: the next K steps through snn_run, this rank's raster rows and the
    # spike counts copied to pinned host memory, the input bytes from it
    wb = window_bytes(corpus, warm + K, K)
    pin = torch.empty(max(wb.size, 1), dtype=torch.uint8, pin_memory=True)
    pin.numpy()[: wb.size] = wb
    raster = torch.empty((K, net.words), dtype=torch.int32, pin_memory=True)
    counts = torch.empty(K, dtype=torch.int32, pin_memory=True)
    ce0 = net.counters()
    if world > 1:
        tdist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    net._check(net.L.snn_run(net.h, K, pin.data_ptr(), wb.size, 1, raster.data_ptr(),
                             counts.data_ptr()))
    net.synchronize()
    wall = time.perf_counter() - t0
    e2e_arr = float(net.counters()["arrivals"] - ce0["arrivals"])
    # per-kernel split on the following steps (events around every kernel)
    net.set_profiling(True)
    net.run(min(K, 50))
    net.synchronize()
    prof = net.profile()
    net.set_profiling(False)
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
            "metric": "synaptic events/sec (SOPS) and sim steps/sec, Stage-2e 5.5M/1.07B "
                      "column-sharded",
            "value": arr_all / (dev_ms / 1000.0), "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": warm, "ms_per_step": dev_ms / K, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic UTF-8 stream `ref45`",
            "config": shard_config(warm, K, args.columns, world),
            "steps_per_sec": K / (dev_ms / 1000.0),
            "events_per_step": arr_all / K, "synapses": syn_all, "build_s": build_s,
            "e2e": {"value": e2e_all / wall, "unit": UNIT, "h2d_bytes_per_step": wb.size / K,
                    "d2h_bytes_per_step": net.words * 4 + 4, "steps_per_sec": K / wall,
                    "events_per_step": e2e_all / K,
                    "how": "snn_run over the K steps after the window (wall clock, max over ranks)"},
            # k_neurons + k_synapses per step; sharded also k_mirror_groups and k_mirror_hist
            "gpu_launches": (4 if world > 1 else 2) * K,
            "kernels_ms_per_step_rank0": {k: x["ms"] / max(x["launches"], 1)
                                          for k, x in prof["kernels"].items()},
            "clocks": clk.summary(),
            "peak_hbm_gbs": peak, "peak_kind": peak_kind,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_stage2e(
                warm, K, "ref45", columns=min(SHARD_SAMPLE_COLUMNS, args.columns), budget_s=30.0,
                st_budget_s=10.0)
        print(json.dumps(line), flush=True)
    net.close()
    if world > 1:
        tdist.barrier()
        tdist.destroy_process_group()


# ---------------------------------------------------------------------------
# configuration 4: the propagation microbench
# ---------------------------------------------------------------------------
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
    sys.path.insert(0, ORACLE)
    import pyoracle as po
    cores = host_cpu_info()["usable_cpus"] or 1
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
    sys.path.insert(0, PKG)
    import snn_b200 as snn
    import torch
    import torch.distributed as tdist
    rank, world, local, _ = dist_env()
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


# ---------------------------------------------------------------------------
# configurations 0 and 1
# ---------------------------------------------------------------------------
def stage0_main(args):
    """Configurations 0 and 1 (Stage 0 block network, Stage 2A columnar
    network), benchmark constants: one JSON line each."""
    sys.path.insert(0, PKG)
    import snn_b200 as snn
    import torch
    sys.path.insert(0, ORACLE)
    import pyoracle as po
    warm = max(args.warmup, 3)
    for columnar in (False, True):
        name = ("stage2A columnar 10 x 1,000 LIF / 1M synapses, synthetic UTF-8 (p_CJK 0.85)"
                if columnar else "stage0 10,000 LIF / 1M synapses, uniform random bytes")
        if columnar:
            data = snn.stream(CORPUS_BYTES, seed=STREAM_SEED, p_cjk=0.85)
        else:
            data = np.random.default_rng(STREAM_SEED).integers(0, 256, CORPUS_BYTES).astype(np.uint8)
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
            cores = host_cpu_info()["usable_cpus"] or 1
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-repeats", type=int, default=3,
                    help="stage2e: timed snn_run repeats of the window (median)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default=None, choices=["stage2e", "prop", "shard", "stage0"],
                    help="default: shard under torchrun (every N) or with --gpus > 1, else "
                         "stage2e.  stage2e: the 55k/10.7M network; shard: the 5,000-column "
                         "network column-sharded over the ranks; prop: the 1M x 1,000 "
                         "propagation microbench (one line per mode and rate); stage0: "
                         "configurations 0 and 1 (one line each, 1 GPU)")
    ap.add_argument("--stream", default="ref45", choices=sorted(STREAMS),
                    help="stage2e input preset (ref45: p_CJK 0.452, b85: p_CJK 0.85)")
    ap.add_argument("--columns", type=int, default=SHARD_COLUMNS, help="shard workload: columns")
    ap.add_argument("--prop-neurons", type=int, default=1_000_000)
    ap.add_argument("--prop-rates", default="", help="comma list, default 0.001,0.01,0.03,0.1")
    ap.add_argument("--prop-modes", default="", help="comma list of 0 (STDP off), 1 (STDP on), 2 (STP on)")
    args = ap.parse_args()
    _, world, _, torchrun = dist_env()
    workload = args.workload or ("shard" if (torchrun or world > 1 or args.gpus > 1) else "stage2e")
    if args.impl == "reference":
        if workload not in ("stage2e", "shard"):
            print(json.dumps({"impl": "reference", "unavailable": f"no reference arm for {workload}"}))
            return
        reference_main(args, workload)
        return
    if workload == "prop":
        prop_main(args)
    elif workload == "shard":
        shard_main(args)
    elif workload == "stage0":
        stage0_main(args)
    else:
        stage2e_main(args)


if __name__ == "__main__":
    main()
