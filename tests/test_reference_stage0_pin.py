"""Stage 0 / Stage 2 parity pinned to the reference itself.

`oracle/_ref/ref_run0` and `ref_run2` are the reference's own SNNNetwork
(src/host/network.cpp:143-191 with the kernels of src/cuda/), compiled from its
unmodified sources as the Stage 0 build and as the Stage 2 build with the
columnar topology.  Their step is deterministic (a fixed 256-wide shared-memory
tree in the propagation, one thread per synapse in the STDP pass), so a run of
the reference on the GPU gives golden rasters for its own network, whose
topology and initial weights come from device cuRAND.  With `--dump` the
harness writes that network in the reference's SNN2 v1 checkpoint layout, the
input bytes, one spike-count / FNV-1a line per step and the final state.

Checked here, for 1,000 steps from the freshly initialised network:
  * the CPU oracle built on the reference's synapse list reproduces every
    step's spike raster exactly, and its membrane potentials, fire rates and
    threshold offsets bit for bit at the end;
  * the product, loading the same SNN2 v1 file through the C ABI, reproduces
    every step's raster exactly as well (canonical build and refmath build);
  * weights: the canonical arithmetic (snn_expf, explicit fused multiply-adds)
    and the reference's (CUDA expf, the compiler's contraction) round the STDP
    terms differently, which after 1,000 steps leaves the canonical weights
    within 5e-5 of the reference's; the refmath build, which writes the STDP
    expressions as the reference does, is held to 1e-5 relative (or 1e-7
    absolute for weights near zero); the synaptic currents, sums of weights,
    follow the weights.
"""
import os
import subprocess

import numpy as np
import pytest

import pyoracle as po
import snn_b200 as snn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")
STEPS = 1000


def fnv64(idx):
    h = 1469598103934665603
    for b in np.asarray(idx, dtype="<i4").tobytes():
        h ^= b
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def ref_dump(exe, out, steps):
    r = subprocess.run([exe, "--dump", str(out), "--steps", str(steps)], capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln.split() for ln in open(os.path.join(out, "spikes.txt")).read().splitlines()]
    assert len(lines) == steps
    counts = np.array([int(x[1]) for x in lines], np.int64)
    hashes = [int(x[2]) for x in lines]
    data = np.fromfile(os.path.join(out, "bytes.bin"), np.uint8)
    final = {k: np.fromfile(os.path.join(out, f"final_{k}.bin"), np.float32)
             for k in ("V", "I", "fr", "w")}
    final["off"] = np.fromfile(os.path.join(out, "final_off.bin"), np.int8)
    return counts, hashes, data, final


def close(a, b, tol=1e-5, atol=1e-12):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.all(np.abs(a - b) <= tol * np.abs(b) + atol)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def engine_run(path, columnar, data, refmath):
    net = snn.Network(model=snn.MODEL_STAGE0, preset=snn.PRESET_REF, refmath=refmath)
    net.build_columns(snn.topology(snn.MODEL_STAGE0, n_columns=10 if columnar else 0))
    net.load(path, snn.FMT_SNN2_V1)
    net.set_corpus(data.tobytes())
    raster, _ = net.run(STEPS, raster=True, counts=True)
    out = {k: net.state(k).copy() for k in ("V", "s", "fr", "weight", "post", "row_ptr")}
    n = net.N
    net.close()
    hashes = []
    for t in range(STEPS):
        idx = np.nonzero(np.unpackbits(raster[t].view(np.uint8), bitorder="little")[:n])[0]
        hashes.append((idx.size, fnv64(idx)))
    return out, hashes


def edge_sorted(pre, post, w):
    o = np.lexsort((w, post, pre))
    return pre[o], post[o], w[o]


@pytest.mark.gpu
@pytest.mark.parametrize("columnar", [False, True], ids=["stage0_block", "stage2_columnar"])
def test_oracle_and_engine_reproduce_the_reference_engine(tmp_path, columnar):
    exe = os.path.join(REF_DIR, "ref_run2" if columnar else "ref_run0")
    if not os.path.exists(exe):
        pytest.skip("reference harness not built (needs the reference sources)")
    counts, hashes, data, final = ref_dump(exe, tmp_path, STEPS)
    assert counts.sum() > 0
    path = os.path.join(tmp_path, "net.snn2")
    f = po.read_snn2(path)
    # the reference keeps its synapses post-major: record s is CSR position s
    assert np.array_equal(f["col_idx"], f["pre"])
    assert np.array_equal(np.repeat(np.arange(f["n"]), np.diff(f["row_ptr"])), f["post"])

    # (1) the CPU oracle on the reference's synapse list
    orc = po.Oracle0(po.stage0_reference_build_params(columnar),
                     synapses=(f["pre"], f["post"], f["weight"]))
    assert orc.N == f["n"] and orc.S == f["s"]
    for t in range(STEPS):
        orc.run(1, [int(data[t])])
        idx = np.nonzero(orc.spikes())[0]
        assert idx.size == counts[t] and fnv64(idx) == hashes[t], f"oracle raster differs at step {t}"
    assert np.array_equal(bits(orc.neuron("V")), bits(final["V"])), "V"
    assert np.array_equal(bits(orc.neuron("fr")), bits(final["fr"])), "fire rate"
    assert np.array_equal(orc.neuron("off").astype(np.int8), final["off"]), "threshold offsets"
    w_orc = orc.synapse("w")
    err = np.abs(w_orc.astype(np.float64) - final["w"])
    print(f"\noracle weights: {np.count_nonzero(err)} of {err.size} differ, max |dw| {err.max():.3g}")
    assert err.max() < 5e-5, "weights"
    assert close(orc.neuron("I"), final["I"], tol=1e-3, atol=1e-3), "synaptic current"
    orc.close()

    # (2) the product through the C ABI on the reference's file, both builds
    ref_edges = edge_sorted(f["pre"], f["post"], final["w"])
    for refmath in (False, True):
        tag = "refmath" if refmath else "canonical"
        out, got = engine_run(path, columnar, data, refmath)
        for t in range(STEPS):
            assert got[t] == (counts[t], hashes[t]), f"{tag} engine raster differs at step {t}"
        assert np.array_equal(bits(out["V"]), bits(final["V"])), f"{tag}: V"
        assert np.array_equal(bits(out["fr"]), bits(final["fr"])), f"{tag}: fire rate"
        pre = np.repeat(np.arange(f["n"]), np.diff(out["row_ptr"]))
        mine = edge_sorted(pre, out["post"], out["weight"])
        assert np.array_equal(mine[0], ref_edges[0]) and np.array_equal(mine[1], ref_edges[1])
        err = np.abs(mine[2].astype(np.float64) - ref_edges[2])
        print(f"{tag} engine weights: {np.count_nonzero(err)} differ, max |dw| {err.max():.3g}")
        if refmath:
            assert close(mine[2], ref_edges[2], tol=1e-5, atol=1e-7), f"{tag}: weights"
            assert close(out["s"], final["I"], tol=1e-5, atol=1e-6), f"{tag}: synaptic current"
        else:
            assert err.max() < 5e-5, f"{tag}: weights"
