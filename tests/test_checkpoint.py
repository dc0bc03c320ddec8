"""Checkpoints: the native full-state format resumes bit-exactly (all three
models); SCKP v2 written by the CUDA path is byte-identical to the oracle's
SCKP v2 of the same run; SNN2 v1 and raw weights round-trip; damaged or
foreign files are refused with SNN_ERR_IO before any state changes."""
import os

import numpy as np
import pytest

import pyoracle as po
import snn_b200 as snn

ERR_IO = 5


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def stage2e(ncol=4, phase=5000):
    net = snn.Network(phase_offset=phase)
    net.build_columns(snn.topology(n_columns=ncol))
    net.set_corpus(snn.stream(20000, seed=7))
    return net


@pytest.mark.gpu
def test_stage2e_native_resume_is_bit_exact(tmp_path):
    path = str(tmp_path / "s2e.snbn")
    a = stage2e()
    a.run(130)
    a.save(path, snn.FMT_NATIVE)
    ra, _ = a.run(170, raster=True)
    b = stage2e()
    b.load(path, snn.FMT_NATIVE)
    assert b.counters()["step"] == 130
    rb, _ = b.run(170, raster=True)
    assert np.array_equal(ra, rb)
    for f in ("V", "w", "input", "alpha", "beta", "ca", "R", "elig", "ampa", "last_pre"):
        assert np.array_equal(bits(a.state(f)), bits(b.state(f))), f
    assert np.array_equal(bits(a.state("gates")), bits(b.state("gates")))
    ca, cb = a.counters(), b.counters()
    for k in ("step", "total_spikes", "arrivals", "dispatched", "ltp_visits"):
        assert ca[k] == cb[k], k


@pytest.mark.gpu
def test_stage2e_sckp_v2_matches_oracle_file(tmp_path):
    steps = 120
    corpus = snn.stream(20000, seed=7)
    orc = po.Oracle2e(po.ref_params(4, phase_offset=5000), corpus)
    orc.run(steps)
    net = stage2e()
    net.run(steps)
    mine, theirs = str(tmp_path / "gpu.sckp"), str(tmp_path / "oracle.sckp")
    net.save(mine, snn.FMT_SCKP_V2)
    orc.save_sckp(theirs, steps)
    a, b = open(mine, "rb").read(), open(theirs, "rb").read()
    assert len(a) == len(b) == 20 + 80 * net.S + 4 * net.N * 256 + 8 * net.S
    if a != b:
        x = np.frombuffer(a[20:20 + 80 * net.S], np.uint8).reshape(-1, 80)
        y = np.frombuffer(b[20:20 + 80 * net.S], np.uint8).reshape(-1, 80)
        bad = np.nonzero((x != y).any(axis=0))[0]
        raise AssertionError(f"SCKP bytes differ; BioSynapse byte offsets {bad[:12]}")


@pytest.mark.gpu
def test_stage2e_raw_weights(tmp_path):
    net = stage2e()
    net.run(40)
    path = str(tmp_path / "w.f32")
    net.save(path, snn.FMT_RAW_F32)
    assert np.array_equal(np.fromfile(path, np.float32).view(np.uint32), bits(net.state("weight")))


def stage0(columnar=True):
    net = snn.Network(model=snn.MODEL_STAGE0, preset=snn.PRESET_REF if columnar else snn.PRESET_BASELINE)
    net.build_columns(snn.topology(snn.MODEL_STAGE0, n_columns=10 if columnar else 0))
    net.set_corpus(bytes(np.random.default_rng(3).integers(0, 256, 5000).astype(np.uint8)))
    return net


@pytest.mark.gpu
def test_stage0_native_resume_and_snn2_raw_round_trip(tmp_path):
    a = stage0()
    a.run(300)
    nat, snn2, raw = (str(tmp_path / n) for n in ("s0.snbn", "s0.snn2", "s0.f32"))
    a.save(nat, snn.FMT_NATIVE)
    a.save(snn2, snn.FMT_SNN2_V1)
    a.save(raw, snn.FMT_RAW_F32)
    ra, _ = a.run(200, raster=True)
    b = stage0()
    b.load(nat, snn.FMT_NATIVE)
    rb, _ = b.run(200, raster=True)
    assert np.array_equal(ra, rb)
    assert np.array_equal(bits(a.state("weight")), bits(b.state("weight")))
    # SNN2 v1: weights, eligibility and spike times come back; header fields as written
    c = stage0()
    c.load(snn2, snn.FMT_SNN2_V1)
    assert c.counters()["step"] == 300
    d = stage0()
    d.run(300)
    for f in ("weight", "elig"):
        assert np.array_equal(bits(c.state(f)), bits(d.state(f))), f
    hdr = np.fromfile(snn2, np.uint32, 2)
    assert hdr[0] == 0x534E4E32 and hdr[1] == 1
    # raw weights: f32[S] in the reference CSR order
    e = stage0()
    e.load(raw, snn.FMT_RAW_F32)
    assert np.array_equal(bits(e.state("weight")), bits(d.state("weight")))


@pytest.mark.gpu
def test_stage0_snn2_adopts_the_files_topology(tmp_path):
    """An SNN2 file written by a network of the same sizes but another CSR
    (another topology seed): loading adopts the file's CSR, and the run goes
    on exactly as on a network built with that topology; a file whose CSR is
    malformed is refused before anything changes."""
    corpus = bytes(np.random.default_rng(3).integers(0, 256, 5000).astype(np.uint8))

    def make(seed):
        net = snn.Network(model=snn.MODEL_STAGE0, preset=snn.PRESET_REF)
        net.build_columns(snn.topology(snn.MODEL_STAGE0, n_columns=10, seed=seed))
        net.set_corpus(corpus)
        return net

    a = make(1)
    a.run(250)
    path = str(tmp_path / "a.snn2")
    a.save(path, snn.FMT_SNN2_V1)
    same, other = make(1), make(9)
    assert not np.array_equal(same.state("post"), other.state("post"))
    v0 = other.state("V").copy()
    # malformed CSR (a row pointer beyond the synapse count): refused, nothing changed
    blob = bytearray(open(path, "rb").read())
    rp_off = 32 + 32 * a.S
    bad = blob[:]
    bad[rp_off + 4 * 5: rp_off + 4 * 6] = np.int32(a.S + 10).tobytes()
    bad_path = str(tmp_path / "bad.snn2")
    open(bad_path, "wb").write(bytes(bad))
    with pytest.raises(snn.SnnError) as e:
        other.load(bad_path, snn.FMT_SNN2_V1)
    assert e.value.code == ERR_IO
    assert np.array_equal(bits(other.state("V")), bits(v0))
    assert other.counters()["step"] == 0

    for n in (same, other):
        n.load(path, snn.FMT_SNN2_V1)
    r1, c1 = same.run(150, raster=True, counts=True)
    r2, c2 = other.run(150, raster=True, counts=True)
    assert np.array_equal(r1, r2) and c1.sum() > 0

    def edges(n):
        rp = n.state("row_ptr")
        pre = np.repeat(np.arange(n.N), np.diff(rp))
        post, w = n.state("post"), bits(n.state("weight"))
        o = np.lexsort((w, post, pre))
        return pre[o], post[o], w[o]

    for x, y in zip(edges(same), edges(other)):
        assert np.array_equal(x, y)
    k1, k2 = same.counters(), other.counters()
    for key in ("step", "total_spikes", "arrivals", "dispatched", "last_spikes"):
        assert k1[key] == k2[key], key
    assert k2["last_spikes"] == c2[-1]
    p1, p2 = str(tmp_path / "s.snn2"), str(tmp_path / "o.snn2")
    same.save(p1, snn.FMT_SNN2_V1)
    other.save(p2, snn.FMT_SNN2_V1)
    assert open(p1, "rb").read() == open(p2, "rb").read()


@pytest.mark.gpu
def test_microbench_native_resume(tmp_path):
    def make():
        n = snn.Network(model=snn.MODEL_PROP, prop_mode=3, prop_rate=0.02)
        n.build_columns(snn.topology(snn.MODEL_PROP, l4=30000, deg_intra=400))
        return n
    path = str(tmp_path / "p.snbn")
    a = make()
    a.run(60)
    a.save(path, snn.FMT_NATIVE)
    ra, _ = a.run(90, raster=True)
    b = make()
    b.load(path, snn.FMT_NATIVE)
    rb, _ = b.run(90, raster=True)
    assert np.array_equal(ra, rb)
    for f in ("V", "weight", "u", "R"):
        assert np.array_equal(bits(a.state(f)), bits(b.state(f))), f


@pytest.mark.gpu
def test_bad_checkpoints_are_refused_without_side_effects(tmp_path):
    good = str(tmp_path / "good.snbn")
    a = stage2e()
    a.run(30)
    a.save(good, snn.FMT_NATIVE)
    blob = open(good, "rb").read()
    cases = {
        "truncated": blob[: len(blob) // 2],
        "bad_magic": b"XXXX" + blob[4:],
        # header 16 B + host blob 64 B + section count 4 B; then the first section's name
        "other_fingerprint": blob[:60] + bytes([blob[60] ^ 0x20]) + blob[61:],
        "flipped_section_name": blob[:84] + bytes([blob[84] ^ 0x20]) + blob[85:],
    }
    b = stage2e()
    b.run(10)
    v0 = b.state("V").copy()
    for name, data in cases.items():
        p = str(tmp_path / f"{name}.snbn")
        open(p, "wb").write(data)
        with pytest.raises(snn.SnnError) as e:
            b.load(p, snn.FMT_NATIVE)
        assert e.value.code == ERR_IO, name
    with pytest.raises(snn.SnnError) as e:
        b.load(str(tmp_path / "missing.snbn"), snn.FMT_NATIVE)
    assert e.value.code == ERR_IO
    # another model's file, and another network's file
    s0 = str(tmp_path / "s0.snbn")
    stage0().save(s0, snn.FMT_NATIVE)
    with pytest.raises(snn.SnnError) as e:
        b.load(s0, snn.FMT_NATIVE)
    assert e.value.code == ERR_IO
    other = stage2e(ncol=6)
    with pytest.raises(snn.SnnError) as e:
        other.load(good, snn.FMT_NATIVE)
    assert e.value.code == ERR_IO
    assert np.array_equal(bits(b.state("V")), bits(v0))
    assert b.counters()["step"] == 10


def native_section_offset(blob, name):
    """Byte offset of a section's data in a native checkpoint (u32 magic,
    u32 version, i32 model, u32 blob bytes, blob, u32 count, then per
    section char[24] name, u64 bytes, data)."""
    hb = int(np.frombuffer(blob[12:16], np.uint32)[0])
    off = 16 + hb
    count = int(np.frombuffer(blob[off: off + 4], np.uint32)[0])
    off += 4
    for _ in range(count):
        nm = blob[off: off + 24].split(b"\0")[0].decode()
        nb = int(np.frombuffer(blob[off + 24: off + 32], np.uint64)[0])
        off += 32
        if nm == name:
            return off, nb
        off += nb
    raise KeyError(name)


@pytest.mark.gpu
def test_microbench_checkpoint_weights_out_of_range_are_refused(tmp_path):
    """A microbench checkpoint whose excitatory weight lies above w_max (or
    an inhibitory one above 0) is refused before anything reaches the
    device: the push's int32 sums and the plasticity clamps rely on the
    ranges."""
    def make():
        n = snn.Network(model=snn.MODEL_PROP, prop_mode=1, prop_rate=0.02)
        n.build_columns(snn.topology(snn.MODEL_PROP, l4=30000, deg_intra=400))
        return n
    good = str(tmp_path / "p.snbn")
    a = make()
    a.run(20)
    a.save(good, snn.FMT_NATIVE)
    blob = bytearray(open(good, "rb").read())
    off, nb = native_section_offset(bytes(blob), "w")
    w = np.frombuffer(bytes(blob[off: off + nb]), np.float32)
    w_max = float(np.abs(w).max())
    b = make()
    b.run(5)
    v0, w0 = b.state("V").copy(), b.state("weight").copy()
    for idx, val in ((3, 2.0 * w_max + 1.0), (w.size - 2, 0.5), (7, float("nan"))):
        bad = bytearray(blob)
        bad[off + 4 * idx: off + 4 * idx + 4] = np.float32(val).tobytes()
        p = str(tmp_path / f"bad{idx}.snbn")
        open(p, "wb").write(bytes(bad))
        with pytest.raises(snn.SnnError) as e:
            b.load(p, snn.FMT_NATIVE)
        assert e.value.code == ERR_IO
    assert np.array_equal(bits(b.state("V")), bits(v0))
    assert np.array_equal(bits(b.state("weight")), bits(w0))
    assert b.counters()["step"] == 5
    b.load(good, snn.FMT_NATIVE)
    assert b.counters()["step"] == 20
