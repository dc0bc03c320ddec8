"""The header-only C++ API (include/snn_b200.hpp): a C++17 client
(tests/hpp_client.cpp) compiles against it and links the C ABI library.
Without a GPU the classes throw SnnException(SNN_ERR_NO_DEVICE); on a GPU the
client's counters, weights and checkpoint bytes equal the same session driven
through the Python binding."""
import os
import shutil
import subprocess

import numpy as np
import pytest

import snn_b200 as snn

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "pure-snn-language_b200")


def gpu_present():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    out = str(tmp_path_factory.mktemp("hpp") / "hpp_client")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"), os.path.join(HERE, "hpp_client.cpp"),
           "-L", PKG, "-lsnn_b200", "-Wl,-rpath," + PKG, "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


def run_client(exe, *args):
    r = subprocess.run([exe, *args], capture_output=True, text=True, timeout=600)
    kv = {}
    for line in r.stdout.splitlines():
        if "=" in line:
            k, v = line.split("=", 1)
            kv[k] = v
    return r.returncode, kv, r.stdout + r.stderr


@pytest.mark.skipif(gpu_present(), reason="checks the no-GPU error path")
def test_header_compiles_and_throws_without_gpu(client):
    rc, kv, out = run_client(client, "nogpu")
    assert rc == 0, out
    assert kv == {"scheduler_code": "7", "network_code": "7"}, out


@pytest.mark.gpu
def test_header_matches_python_binding(client, tmp_path):
    cdir = tmp_path / "cpp"
    cdir.mkdir()
    rc, kv, out = run_client(client, "gpu", str(cdir))
    assert rc == 0, out

    text = b"The quick brown fox\r\njumps\tover the lazy dog."
    corpus = bytes(32 if c in (13, 10, 9) else c for c in text)
    assert int(kv["corpus_bytes"]) == len(corpus)
    net = snn.Network()
    net.build_columns(snn.topology(n_columns=50))
    net.set_corpus(corpus)
    for t in range(40):
        net.step(t)
    net.run(24)
    c = net.counters()
    assert int(kv["steps"]) == c["step"] == 64
    assert int(kv["spikes"]) == c["total_spikes"]
    assert int(kv["arrived"]) == c["arrivals"]
    assert int(kv["dispatched"]) == c["dispatched"]
    w = np.fromfile(cdir / "weights2e.f32", np.float32)
    assert np.array_equal(w.view(np.uint32), net.state("weight").view(np.uint32))
    assert kv["ckpt_rc"] == "0" and kv["ckpt_bad_rc"] == "2"
    pypath = str(tmp_path / "py_ckpt.bin")
    net.save(pypath, snn.FMT_SCKP_V2)
    with open(cdir / "ckpt_step64.bin", "rb") as f, open(pypath, "rb") as g:
        assert f.read() == g.read()
    net.close()

    n0 = snn.Network(model=snn.MODEL_STAGE0, preset=snn.PRESET_BASELINE)
    n0.build_columns(snn.topology(snn.MODEL_STAGE0, 0, seed=42))
    assert int(kv["n_neurons"]) == n0.N
    for t in range(30):
        n0.step(t, (ord("a") + t % 26) if t % 3 == 0 else -1)
    n0.set_dopamine(0.5)
    for t in range(30, 60):
        n0.step(t)
    assert int(kv["s0_spikes"]) == n0.counters()["total_spikes"]
    assert kv["load_missing_code"] == "5"
    pyw = str(tmp_path / "py_w.bin")
    n0.save(pyw, snn.FMT_RAW_F32)
    with open(cdir / "weights.bin", "rb") as f, open(pyw, "rb") as g:
        assert f.read() == g.read()
    n0.close()
