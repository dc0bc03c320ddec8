"""CPU tests of the benchmark's input and reference arm: the oracle's stream
and corpus filter equal the product's, and `bench.py --impl reference` runs
the CPU oracle over the same window and config as the product's line without
loading any library of the product."""
import json
import os
import subprocess
import sys

import numpy as np

import pyoracle as po
import snn_b200 as snn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_oracle_stream_equals_product_stream():
    for seed, p in ((42, 0.452), (42, 0.85), (7, 0.452), (3, 0.1)):
        a = po.stream(300_000, seed=seed, p_cjk=p)
        b = snn.stream(300_000, seed=seed, p_cjk=p)
        assert np.array_equal(a, b), (seed, p)
        assert po.byte_classes(a) == snn.byte_classes(b)


def test_stream_presets_byte_classes():
    c45 = snn.byte_classes(snn.stream(1 << 20, seed=42, p_cjk=0.452))
    c85 = snn.byte_classes(snn.stream(1 << 20, seed=42, p_cjk=0.85))
    assert abs(c45["continuation"] - 0.475) < 0.005
    assert c85["continuation"] > 0.62
    for c in (c45, c85):
        assert abs(c["ascii"] + c["head"] + c["continuation"] - 1.0) < 1e-12
        assert abs(c["continuation"] - 2 * c["head"]) < 0.002  # 3-byte characters


def test_text_filter_matches_reference_rule():
    raw = bytes([0, 65, 13, 10, 9, 0, 0xE4, 0xB8, 0x80, 32, 0, 66])
    assert po.text_filter(raw).tobytes() == bytes([65, 32, 32, 32, 0xE4, 0xB8, 0x80, 32, 66])
    assert po.text_filter(b"").size == 0


def test_reference_arm_loads_no_product_library():
    """Runs the reference arm in a child process and lists the shared objects
    it mapped: the oracle's, never libsnn_b200.so."""
    code = (
        "import sys, runpy, json\n"
        f"sys.argv = ['bench.py', '--impl', 'reference', '--steps', '3', '--warmup', '3']\n"
        f"runpy.run_path({os.path.join(ROOT, 'bench.py')!r}, run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "print('MAPS', json.dumps(sorted({l.split()[-1] for l in maps.splitlines() "
        "if l.endswith('.so') or '.so.' in l.split()[-1]})))\n")
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT,
                       env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.splitlines()
    line = json.loads(next(x for x in lines if x.startswith("{")))
    maps = json.loads(next(x for x in lines if x.startswith("MAPS "))[5:])
    assert not any("libsnn_b200" in m for m in maps), maps
    assert any(m.endswith("oracle/liboracle.so") for m in maps)
    assert line["impl"] == "reference" and line["cpu_baseline"]["kind"] == "port"
    sys.path.insert(0, ROOT)
    import bench
    assert line["config"] == bench.stage2e_config(3, 3, "ref45")
    assert line["unit"] == bench.UNIT and line["metric"] == bench.METRIC
    # the oracle over steps 3..5 of the benchmarked network delivers events
    assert line["events_per_step"] > 0
