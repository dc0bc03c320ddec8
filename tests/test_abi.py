"""CPU tests of the C ABI library: it loads, exports every entry point that
include/*.h declares, validates arguments, and fails loudly (no fallback)
when no GPU is present.  No compute call needs a GPU here."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import snn_b200 as snn

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def declared_functions():
    names = set()
    inc = os.path.join(ROOT, "include")
    for fn in os.listdir(inc):
        if not fn.endswith(".h") or fn in ("snn_pmath.h", "snn_prop_rules.h"):  # inline helpers
            continue
        txt = open(os.path.join(inc, fn)).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        for m in re.finditer(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b(snn_\w+)\s*\(", txt, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    L = snn.lib()
    decl = declared_functions()
    assert {"snn_create", "snn_run", "snn_step", "snn_build_columns"} <= decl
    missing = [n for n in sorted(decl) if not hasattr(L, n)]
    assert not missing, missing
    assert set(snn.EXPORTS) <= decl


def gpu_present():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(gpu_present(), reason="checks the no-GPU error path")
def test_create_without_gpu_fails_loudly():
    with pytest.raises(snn.SnnError) as e:
        snn.Network()
    assert e.value.code == 7


def test_config_and_topology_init():
    L = snn.lib()
    cfg = snn.Config()
    assert L.snn_config_init(C.byref(cfg), 0, 0) == 0 and cfg.raster_steps == 1024
    assert L.snn_config_init(C.byref(cfg), 9, 0) == 1
    assert L.snn_config_init(None, 0, 0) == 1
    spec = snn.topology(n_columns=50)
    assert (spec.l4, spec.l23, spec.l5, spec.l6) == (200, 350, 200, 250)
    assert spec.total_synapses == 10_700_000 and spec.seed == 42
    with pytest.raises(snn.SnnError):
        snn.topology(n_columns=1)


def test_null_handles_are_rejected():
    L = snn.lib()
    assert L.snn_step(None, 0, -1, 1) == 1
    assert L.snn_run(None, 1, None, 0, 1, None, None) == 1
    assert L.snn_get_counters(None, None) == 1


def test_stream_presets_byte_classes():
    b = snn.stream(600_000, seed=42, p_cjk=0.452)
    cls = snn.byte_classes(b)
    assert abs(cls["continuation"] - 0.475) < 0.01
    b85 = snn.stream(600_000, seed=42, p_cjk=0.85)
    assert snn.byte_classes(b85)["continuation"] > 0.6
    # valid UTF-8 except possibly the cut last character
    b.tobytes()[:-3].decode("utf-8", errors="strict")
    assert np.array_equal(snn.stream(1000, seed=5), snn.stream(1000, seed=5))
    assert not np.array_equal(snn.stream(1000, seed=5), snn.stream(1000, seed=6))


def test_library_does_not_link_nccl_and_torch_loads_after_it():
    """NCCL is opened at run time by sharded runs only: the library has no
    link-time libnccl dependency, so importing torch after loading it keeps
    torch's own NCCL build (a system libnccl loaded first would take the
    soname and leave torch's newer NCCL symbols unresolved)."""
    import subprocess
    import sys
    out = subprocess.run(["readelf", "-d", snn.LIB_PATH], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    needed = [ln for ln in out.stdout.splitlines() if "(NEEDED)" in ln]
    assert needed and not any("nccl" in ln for ln in needed), needed
    code = ("import sys; sys.path.insert(0, %r); import snn_b200 as snn; snn.lib(); "
            "import torch; print('ok', torch.__version__)" % os.path.dirname(snn.LIB_PATH))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stderr[-2000:]
