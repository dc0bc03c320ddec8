"""Python binding of the B200 SNN core (libsnn_b200.so, C ABI in
include/snn_b200.h).

Mirrors the reference host API (TSOFTP-afk/pure-snn-language):
``Network`` plays the role of ``stage2e::BioMechanismScheduler`` +
``MemoryAllocator`` (src/stage2e/scheduler.cuh:66-224) and of
``SNNNetwork`` (src/include/network.h:11-95): build by columns and layers,
step / run with byte injection, read state and counters, save / load.

The library must be built (``make -C pure-snn-language_b200``); importing this
module on a machine without the built library, or creating a network without
a CUDA device, raises instead of falling back to anything else.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsnn_b200.so")
# the same core built with the reference's arithmetic (CUDA expf, compiler
# contraction of plain expressions) instead of the canonical one
REFMATH_LIB_PATH = os.path.join(HERE, "libsnn_b200_refmath.so")

SNN_OK = 0
ERRORS = {1: "SNN_ERR_ARG", 2: "SNN_ERR_CUDA", 3: "SNN_ERR_OOM", 4: "SNN_ERR_STATE",
          5: "SNN_ERR_IO", 6: "SNN_ERR_UNSUPPORTED", 7: "SNN_ERR_NO_DEVICE"}
MODEL_STAGE2E, MODEL_STAGE0, MODEL_PROP = 0, 1, 2
PROP_PLAIN, PROP_STDP, PROP_STP = 0, 1, 2
PRESET_REF, PRESET_BASELINE = 0, 1
CORPUS_TEXT_FILTER = 1
FMT_NATIVE, FMT_SNN2_V1, FMT_SCKP_V2, FMT_RAW_F32 = 0, 1, 2, 3

STATE = {
    "V": (0, np.float32, "N"), "w": (1, np.float32, "N"), "s": (2, np.float32, "N"),
    "fr": (3, np.float32, "N"), "ca_neuron": (4, np.float32, "N"),
    "input": (5, np.float32, "N"), "nmda_cur": (6, np.float32, "N"),
    "last": (7, np.int32, "N"), "ref": (8, np.int32, "N"), "x_post": (9, np.float32, "N"),
    "thresh_off": (10, np.int32, "N"),
    "alpha": (20, np.float32, "S"), "beta": (21, np.float32, "S"),
    "weight": (22, np.float32, "S"), "x_pre": (23, np.float32, "S"),
    "nmda": (24, np.float32, "S"), "ca": (25, np.float32, "S"),
    "R": (26, np.float32, "S"), "u": (27, np.float32, "S"), "elig": (28, np.float32, "S"),
    "camkii_act": (29, np.float32, "S"), "autophos": (30, np.float32, "S"),
    "e1": (31, np.float32, "S"), "e2": (32, np.float32, "S"),
    "ampa": (33, np.float32, "S"), "last_pre": (34, np.float32, "S"),
    "post": (40, np.int32, "S"), "delay": (41, np.uint8, "S"), "row_ptr": (42, np.int32, "N1"),
    "flags": (43, np.uint8, "S"), "gates": (50, np.float32, "G4"),
    "modulators": (51, np.float32, "4"), "byte_hist": (52, np.int32, "256"),
    "neuron_byte_counts": (53, np.int32, "N256"),
}


class SnnError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [("model", C.c_int32), ("preset", C.c_int32), ("device", C.c_int32),
                ("e0", C.c_int32), ("phase_offset", C.c_int32), ("raster_steps", C.c_int32),
                ("prop_mode", C.c_int32), ("prop_rate", C.c_float), ("prop_w_max", C.c_float),
                ("prop_push", C.c_int32), ("reserved", C.c_int32 * 6)]


class TopologySpec(C.Structure):
    _fields_ = [("n_columns", C.c_int32), ("l4", C.c_int32), ("l23", C.c_int32),
                ("l5", C.c_int32), ("l6", C.c_int32), ("pf_groups", C.c_int32),
                ("pf_group_size", C.c_int32), ("deg_intra", C.c_int32), ("deg_inter", C.c_int32),
                ("deg_l5_pf", C.c_int32), ("deg_pf_self", C.c_int32),
                ("deg_pf_assoc", C.c_int32), ("total_synapses", C.c_int64),
                ("seed", C.c_uint32), ("rule", C.c_int32), ("reserved", C.c_int32 * 8)]


class Counters(C.Structure):
    _fields_ = [("step", C.c_int64), ("total_spikes", C.c_int64), ("arrivals", C.c_int64),
                ("dispatched", C.c_int64), ("dropped_ref", C.c_int64),
                ("ltp_visits", C.c_int64), ("burst_spikes", C.c_int64),
                ("n_neurons", C.c_int64), ("n_synapses", C.c_int64), ("n_groups", C.c_int64),
                ("last_spikes", C.c_int32), ("last_byte", C.c_int32),
                ("modeled_bytes", C.c_double), ("local_lo", C.c_int64), ("local_hi", C.c_int64),
                ("reserved", C.c_int64 * 4)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_ if k != "reserved"}


class Semantic(C.Structure):
    _fields_ = [("silhouette", C.c_double), ("js_mean", C.c_double), ("js_max", C.c_double),
                ("column_ratio", C.c_double), ("grand_total", C.c_double),
                ("n_columns", C.c_int32), ("nonzero_columns", C.c_int32),
                ("layer_delay", C.c_double * 5), ("layer_delay_n", C.c_int32 * 5),
                ("layer_sig", C.c_int32 * 5), ("layer_act", C.c_int32 * 5),
                ("layer_chi2_mean", C.c_double * 5), ("reserved", C.c_int32 * 8)]

    def as_dict(self):
        out = {}
        for k, _ in self._fields_:
            if k == "reserved":
                continue
            v = getattr(self, k)
            out[k] = list(v) if hasattr(v, "__len__") else v
        return out


class Profile(C.Structure):
    _fields_ = [("steps", C.c_int64), ("n_kernels", C.c_int32), ("reserved0", C.c_int32),
                ("kernel_ms", C.c_double * 8), ("launches", C.c_int64 * 8),
                ("step_ms", C.c_double), ("names", (C.c_char * 32) * 8)]

    def as_dict(self):
        k = self.n_kernels
        return {"steps": self.steps, "step_ms": self.step_ms,
                "kernels": {self.names[i].value.decode(): {"ms": self.kernel_ms[i],
                                                           "launches": self.launches[i]}
                            for i in range(k)}}


EXPORTS = ["snn_config_init", "snn_topology_init", "snn_create", "snn_destroy",
           "snn_last_error", "snn_version", "snn_build_columns", "snn_set_corpus", "snn_step",
           "snn_run", "snn_synchronize", "snn_get_spikes", "snn_get_state", "snn_get_counters",
           "snn_set_dopamine", "snn_set_e0", "snn_save", "snn_load", "snn_stream_generate",
           "snn_set_profiling", "snn_get_profile", "snn_propagate", "snn_propagate_static",
           "snn_nccl_unique_id", "snn_set_shard", "snn_shard_plan", "snn_semantic_eval",
           "snn_set_corpus_ex", "snn_load_text_corpus", "snn_byte_classes"]

_lib = None
_lib_refmath = None


def lib(refmath=False):
    """Load libsnn_b200.so, or with refmath=True libsnn_b200_refmath.so
    (raises if it was not built)."""
    global _lib, _lib_refmath
    if refmath:
        if _lib_refmath is None:
            _lib_refmath = _load(REFMATH_LIB_PATH)
        return _lib_refmath
    if _lib is None:
        _lib = _load(LIB_PATH)
    return _lib


def _load(path):
    if not os.path.exists(path):
        raise OSError(f"{path} is missing: build it with `make -C {HERE}`")
    L = C.CDLL(path)
    vp = C.c_void_p
    L.snn_config_init.argtypes = [C.POINTER(Config), C.c_int32, C.c_int32]
    L.snn_topology_init.argtypes = [C.POINTER(TopologySpec), C.c_int32, C.c_int32]
    L.snn_create.argtypes = [C.POINTER(Config), C.POINTER(vp)]
    L.snn_destroy.argtypes = [vp]
    L.snn_destroy.restype = None
    L.snn_last_error.argtypes = [vp]
    L.snn_last_error.restype = C.c_char_p
    L.snn_version.restype = C.c_char_p
    L.snn_build_columns.argtypes = [vp, C.POINTER(TopologySpec)]
    L.snn_set_corpus.argtypes = [vp, vp, C.c_int64]
    L.snn_set_corpus_ex.argtypes = [vp, vp, C.c_int64, C.c_int32, vp]
    L.snn_load_text_corpus.argtypes = [vp, C.c_char_p, vp]
    L.snn_byte_classes.argtypes = [vp, C.c_int64, vp, C.c_int32]
    L.snn_step.argtypes = [vp, C.c_int32, C.c_int32, C.c_int32]
    L.snn_run.argtypes = [vp, C.c_int32, vp, C.c_int64, C.c_int32, vp, vp]
    L.snn_synchronize.argtypes = [vp]
    L.snn_get_spikes.argtypes = [vp, vp, C.c_int64]
    L.snn_get_state.argtypes = [vp, C.c_int32, vp, C.c_int64]
    L.snn_get_counters.argtypes = [vp, C.POINTER(Counters)]
    L.snn_semantic_eval.argtypes = [vp, C.c_int64, C.POINTER(Semantic), vp, C.c_int64]
    L.snn_set_dopamine.argtypes = [vp, C.c_float]
    L.snn_set_e0.argtypes = [vp, C.c_int32]
    L.snn_save.argtypes = [vp, C.c_char_p, C.c_int32]
    L.snn_load.argtypes = [vp, C.c_char_p, C.c_int32]
    L.snn_stream_generate.argtypes = [vp, C.c_int64, C.c_uint64, C.c_double, C.c_double]
    L.snn_set_profiling.argtypes = [vp, C.c_int32]
    L.snn_get_profile.argtypes = [vp, C.POINTER(Profile)]
    L.snn_propagate.argtypes = [vp, vp, C.c_int64, C.c_int32, vp, vp, C.c_int64, C.c_int32, vp]
    L.snn_propagate_static.argtypes = L.snn_propagate.argtypes
    L.snn_nccl_unique_id.argtypes = [vp, C.c_int64]
    L.snn_set_shard.argtypes = [vp, C.c_int32, C.c_int32, vp, C.c_int64]
    L.snn_shard_plan.argtypes = [C.POINTER(TopologySpec), C.c_int32, C.c_int32, vp, C.c_int32]
    return L


def propagate(post, w, fanout, spikes, acc, frac_bits=24, stream=None, static=False):
    """snn_propagate on torch CUDA tensors (int32 post[n_pre*fanout],
    float32 w[...], uint8 spikes[n_pre], int32 acc[n_post], accumulated in
    place) on `stream` (a torch.cuda.Stream, default: the current stream).
    static=True calls snn_propagate_static (no allocation, n_pre <= 2^20)."""
    import torch
    for t_, dt in ((post, torch.int32), (w, torch.float32), (spikes, torch.uint8), (acc, torch.int32)):
        if not (t_.is_cuda and t_.dtype == dt and t_.is_contiguous()):
            raise SnnError(1, "propagate wants contiguous CUDA tensors int32/float32/uint8/int32")
    st = stream if stream is not None else torch.cuda.current_stream(acc.device)
    fn = lib().snn_propagate_static if static else lib().snn_propagate
    rc = fn(post.data_ptr(), w.data_ptr(), spikes.numel(), fanout, spikes.data_ptr(),
            acc.data_ptr(), acc.numel(), frac_bits, st.cuda_stream)
    if rc:
        raise SnnError(rc, lib().snn_last_error(None).decode())


def nccl_unique_id():
    """128-byte NCCL unique id (bytes) for snn_set_shard; make it on one rank
    and share it with the others."""
    buf = (C.c_uint8 * 128)()
    rc = lib().snn_nccl_unique_id(buf, 128)
    if rc:
        raise SnnError(rc, lib().snn_last_error(None).decode())
    return bytes(buf)


def shard_plan(spec, rank, world):
    """Host-only partition plan of a Stage 2e topology (no GPU needed)."""
    out = np.zeros(10, np.int64)
    rc = lib().snn_shard_plan(C.byref(spec), rank, world, out.ctypes.data, 10)
    if rc:
        raise SnnError(rc, lib().snn_last_error(None).decode())
    keys = ["n_local", "a0", "a1", "pf0", "pf1", "synapses", "groups_local", "groups_mirror",
            "mirror_pres", "remote_short_delay"]
    return {k: int(v) for k, v in zip(keys, out)}


def stream(n, seed=42, p_cjk=0.452, zipf_s=1.1):
    """Seeded synthetic UTF-8 byte stream (numpy uint8[n]).  p_cjk=0.452 is
    the `ref45` preset (about 47.5 % continuation bytes), 0.85 is `b85`."""
    out = np.zeros(n, np.uint8)
    rc = lib().snn_stream_generate(out.ctypes.data, n, seed, p_cjk, zipf_s)
    if rc:
        raise SnnError(rc, "snn_stream_generate")
    return out


def byte_classes(b):
    """Fractions of ASCII (< 0x80), UTF-8 lead (0xC0..0xF7) and continuation
    (0x80..0xBF) bytes (snn_byte_classes)."""
    a = np.ascontiguousarray(np.frombuffer(bytes(b), np.uint8))
    out = np.zeros(3, np.int64)
    rc = lib().snn_byte_classes(a.ctypes.data, a.size, out.ctypes.data, 3)
    if rc:
        raise SnnError(rc, "snn_byte_classes")
    n = max(a.size, 1)
    return {"ascii": float(out[0]) / n, "head": float(out[1]) / n,
            "continuation": float(out[2]) / n}


def topology(model=MODEL_STAGE2E, n_columns=50, **overrides):
    spec = TopologySpec()
    rc = lib().snn_topology_init(C.byref(spec), model, n_columns)
    if rc:
        raise SnnError(rc, "snn_topology_init")
    for k, v in overrides.items():
        setattr(spec, k, v)
    return spec


class Network:
    """One network on one GPU (one snn_ctx)."""

    def __init__(self, model=MODEL_STAGE2E, preset=PRESET_REF, device=0, e0=False,
                 phase_offset=0, raster_steps=1024, prop_mode=0, prop_rate=0.01, prop_w_max=0.0,
                 prop_push=0, refmath=False):
        """refmath=True runs the network on the core built with the
        reference's arithmetic (libsnn_b200_refmath.so)."""
        L = lib(refmath)
        self.L = L
        cfg = Config()
        self._check(L.snn_config_init(C.byref(cfg), model, preset), None)
        cfg.device, cfg.e0, cfg.phase_offset, cfg.raster_steps = device, int(e0), phase_offset, raster_steps
        if model == MODEL_PROP:
            cfg.prop_mode, cfg.prop_rate, cfg.prop_w_max = prop_mode, prop_rate, prop_w_max
            cfg.prop_push = prop_push
        h = C.c_void_p()
        rc = L.snn_create(C.byref(cfg), C.byref(h))
        if rc:
            raise SnnError(rc, L.snn_last_error(None).decode())
        self.h = h
        self.model = model
        self.N = self.S = 0

    def _check(self, rc, h="self"):
        if rc:
            msg = self.L.snn_last_error(self.h if h == "self" else None)
            raise SnnError(rc, msg.decode() if msg else "")

    def close(self):
        if getattr(self, "h", None):
            self.L.snn_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def build_columns(self, spec):
        self._check(self.L.snn_build_columns(self.h, C.byref(spec)))
        c = self.counters()
        self.N, self.S = c["n_neurons"], c["n_synapses"]
        self.words = (self.N + 31) // 32
        self.n_columns = spec.n_columns
        return self

    def set_corpus(self, data, text_filter=False):
        """The byte stream the network reads (one byte per inject step,
        wrapping).  text_filter=True applies the reference's corpus filter
        (NUL dropped, CR / LF / TAB -> space); returns the kept length."""
        b = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8))
        kept = C.c_int64(0)
        self._check(self.L.snn_set_corpus_ex(self.h, b.ctypes.data, b.size,
                                             CORPUS_TEXT_FILTER if text_filter else 0,
                                             C.byref(kept)))
        return kept.value

    def load_text_corpus(self, path):
        """Read a text file, filter it like the reference's load_text_corpus
        and make it the corpus; returns the kept length."""
        kept = C.c_int64(0)
        self._check(self.L.snn_load_text_corpus(self.h, os.fsencode(path), C.byref(kept)))
        return kept.value

    def step(self, step, inject_byte=-1, learn=True):
        self._check(self.L.snn_step(self.h, step, inject_byte, int(learn)))

    def run(self, n_steps, data=None, learn=True, raster=False, counts=False):
        """Run n_steps; returns (raster uint32[n_steps, words] or None,
        counts int32[n_steps] or None)."""
        r = np.zeros((n_steps, self.words), np.uint32) if raster else None
        c = np.zeros(n_steps, np.int32) if counts else None
        b = None
        if data is not None:
            b = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8))
        self._check(self.L.snn_run(self.h, n_steps, b.ctypes.data if b is not None else None,
                                   b.size if b is not None else 0, int(learn),
                                   r.ctypes.data if r is not None else None,
                                   c.ctypes.data if c is not None else None))
        return r, c

    def synchronize(self):
        self._check(self.L.snn_synchronize(self.h))

    def spikes(self):
        w = np.zeros(self.words, np.uint32)
        self._check(self.L.snn_get_spikes(self.h, w.ctypes.data, w.size))
        return np.unpackbits(w.view(np.uint8), bitorder="little")[: self.N]

    def state(self, name):
        which, dt, shape = STATE[name]
        if self.model == MODEL_PROP and name in ("R", "u"):
            shape = "N"  # per pre-synaptic neuron in the microbench
        n = {"N": self.N, "S": self.S, "N1": self.N + 1, "4": 4, "256": 256,
             "N256": self.N * 256, "G4": 4 * self.n_columns}[shape]
        out = np.zeros(n, dt)
        self._check(self.L.snn_get_state(self.h, which, out.ctypes.data, out.nbytes))
        return out.reshape(-1, 4) if shape == "G4" else out

    def counters(self):
        c = Counters()
        self._check(self.L.snn_get_counters(self.h, C.byref(c)))
        return c.as_dict()

    def semantic_eval(self, step=None):
        """Semantic evaluation of a Stage 2e network (snn_semantic_eval):
        dict of the scalars and per-layer lists, plus each column's cluster
        under "assign".  step defaults to the number of executed steps."""
        out = Semantic()
        n_col = max(int(getattr(self, "n_columns", 0) or 0), 1)
        asg = np.zeros(n_col, np.int32)
        st = self.counters()["step"] if step is None else int(step)
        self._check(self.L.snn_semantic_eval(self.h, st, C.byref(out), asg.ctypes.data, asg.size))
        d = out.as_dict()
        d["assign"] = asg[: d["n_columns"]]
        return d

    def set_profiling(self, enable=True):
        """True / 1: per-kernel device times; 2: whole-run device time only
        (Stage 2e); False / 0: off."""
        self._check(self.L.snn_set_profiling(self.h, int(enable)))

    def profile(self):
        p = Profile()
        self._check(self.L.snn_get_profile(self.h, C.byref(p)))
        return p.as_dict()

    def set_shard(self, rank, world, uid=None):
        """Column sharding (before build_columns): rank of world, NCCL id."""
        b = (C.c_uint8 * 128).from_buffer_copy(uid) if uid is not None else None
        self._check(self.L.snn_set_shard(self.h, rank, world, b, 128 if b is not None else 0))
        self.rank, self.world = rank, world

    def set_dopamine(self, level):
        self._check(self.L.snn_set_dopamine(self.h, level))

    def set_e0(self, enable):
        self._check(self.L.snn_set_e0(self.h, int(enable)))

    def save(self, path, fmt=FMT_NATIVE):
        self._check(self.L.snn_save(self.h, path.encode(), fmt))

    def load(self, path, fmt=FMT_NATIVE):
        self._check(self.L.snn_load(self.h, path.encode(), fmt))
