"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, never by the product package.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


class O2eParams(C.Structure):
    _fields_ = [
        ("n_columns", C.c_int32), ("l4", C.c_int32), ("l23", C.c_int32),
        ("l5", C.c_int32), ("l6", C.c_int32), ("pf_groups", C.c_int32),
        ("pf_group_size", C.c_int32), ("deg_intra", C.c_int32),
        ("deg_inter", C.c_int32), ("deg_l5_pf", C.c_int32),
        ("deg_pf_self", C.c_int32), ("deg_pf_assoc", C.c_int32),
        ("total_synapses", C.c_int64), ("seed", C.c_uint32), ("e0", C.c_int32),
        ("phase_offset", C.c_int32), ("n_threads", C.c_int32),
    ]


class O2eCounters(C.Structure):
    _fields_ = [
        ("step", C.c_int64), ("total_spikes", C.c_int64), ("arrived", C.c_int64),
        ("dispatched", C.c_int64), ("dropped", C.c_int64), ("ltp_visits", C.c_int64),
        ("burst_spikes", C.c_int64), ("last_spikes", C.c_int32),
        ("last_arrived", C.c_int32), ("last_dispatched", C.c_int32),
        ("last_byte", C.c_int32), ("n_neurons", C.c_int32), ("ring_idx", C.c_int32),
        ("n_synapses", C.c_int64),
    ]


SYN_FIELDS = {"alpha": 0, "beta": 1, "weight": 2, "x_pre": 3, "x_post": 4, "nmda": 5,
              "ca": 6, "R": 7, "u": 8, "elig": 9, "camkii_act": 10, "autophos": 11,
              "e1": 12, "e2": 13, "ampa": 14}
NEU_FIELDS = {"V": 0, "s": 1, "w": 2, "fr": 3, "ca": 4, "input": 5, "nmda_cur": 6,
              "inh": 7, "spike": 8, "last": 9, "ref": 10}

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.o2e_create.restype = C.c_void_p
        L.o2e_create.argtypes = [C.POINTER(O2eParams)]
        L.o2e_destroy.argtypes = [C.c_void_p]
        L.o2e_set_corpus.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.o2e_run.argtypes = [C.c_void_p, C.c_int32]
        L.o2e_counters.argtypes = [C.c_void_p, C.POINTER(O2eCounters)]
        L.o2e_topology.argtypes = [C.c_void_p] + [C.c_void_p] * 4
        L.o2e_neuron_f32.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
        L.o2e_spikes.argtypes = [C.c_void_p, C.c_void_p]
        L.o2e_next_input.argtypes = [C.c_void_p, C.c_void_p]
        L.o2e_synapse_f32.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
        L.o2e_control.argtypes = [C.c_void_p] + [C.c_void_p] * 3
        L.o2e_neuron_byte_counts.argtypes = [C.c_void_p, C.c_void_p]
        L.o2e_init_weights.argtypes = [C.c_void_p] + [C.c_void_p] * 3
        L.o2e_expf.restype = C.c_float
        L.o2e_expf.argtypes = [C.c_float]
        L.o2e_expf_array.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.o2e_fnv64.restype = C.c_uint64
        L.o2e_fnv64.argtypes = [C.c_void_p, C.c_int64]
        _lib = L
    return _lib


def ref_params(n_columns=50, seed=42, e0=0, phase_offset=0, n_threads=0):
    """Reference topology rules (src/stage2e/network_init.cu:198-233), scaled by
    column count; n_columns=50 is the reference network (55,000 / 10,700,000)."""
    p = O2eParams()
    p.n_columns = n_columns
    p.l4, p.l23, p.l5, p.l6 = 200, 350, 200, 250
    p.pf_groups, p.pf_group_size = n_columns, 100
    p.deg_intra, p.deg_inter, p.deg_l5_pf = 150, 30, 15
    p.deg_pf_self, p.deg_pf_assoc = 100, 50
    p.total_synapses = 10_700_000 * n_columns // 50
    p.seed, p.e0, p.phase_offset, p.n_threads = seed, e0, phase_offset, n_threads
    return p


class Oracle2e:
    def __init__(self, params, corpus=None):
        self.L = lib()
        self.p = params
        self.h = self.L.o2e_create(C.byref(params))
        c = self.counters()
        self.N, self.S = c.n_neurons, c.n_synapses
        if corpus is not None:
            buf = np.ascontiguousarray(np.frombuffer(bytes(corpus), dtype=np.uint8))
            self.L.o2e_set_corpus(self.h, buf.ctypes.data, buf.size)

    def close(self):
        if self.h:
            self.L.o2e_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def run(self, n):
        self.L.o2e_run(self.h, n)

    def counters(self):
        c = O2eCounters()
        self.L.o2e_counters(self.h, C.byref(c))
        return c

    def topology(self):
        rp = np.zeros(self.N + 1, np.int32)
        post = np.zeros(self.S, np.int32)
        d = np.zeros(self.S, np.uint8)
        fl = np.zeros(self.S, np.uint8)
        self.L.o2e_topology(self.h, rp.ctypes.data, post.ctypes.data, d.ctypes.data, fl.ctypes.data)
        return rp, post, d, fl

    def init_weights(self):
        w = np.zeros(self.S, np.float32)
        a = np.zeros(self.S, np.float32)
        b = np.zeros(self.S, np.float32)
        self.L.o2e_init_weights(self.h, w.ctypes.data, a.ctypes.data, b.ctypes.data)
        return w, a, b

    def neuron(self, name):
        out = np.zeros(self.N, np.float32)
        self.L.o2e_neuron_f32(self.h, NEU_FIELDS[name], out.ctypes.data)
        return out

    def next_input(self):
        out = np.zeros(self.N, np.float32)
        self.L.o2e_next_input(self.h, out.ctypes.data)
        return out

    def spikes(self):
        out = np.zeros(self.N, np.uint8)
        self.L.o2e_spikes(self.h, out.ctypes.data)
        return out

    def synapse(self, name):
        out = np.zeros(self.S, np.float32)
        self.L.o2e_synapse_f32(self.h, SYN_FIELDS[name], out.ctypes.data)
        return out

    def control(self):
        g = np.zeros(4 * self.p.n_columns, np.float32)
        m = np.zeros(4, np.float32)
        bh = np.zeros(256, np.int32)
        self.L.o2e_control(self.h, g.ctypes.data, m.ctypes.data, bh.ctypes.data)
        return g.reshape(-1, 4), m, bh

    def neuron_byte_counts(self):
        out = np.zeros(self.N * 256, np.int32)
        self.L.o2e_neuron_byte_counts(self.h, out.ctypes.data)
        return out.reshape(self.N, 256)


def fnv64(arr):
    """FNV-1a 64 over the raw bytes of an array (same as the pin harnesses)."""
    a = np.ascontiguousarray(arr)
    return int(lib().o2e_fnv64(a.ctypes.data, a.nbytes))


def expf_array(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().o2e_expf_array(x.ctypes.data, y.ctypes.data, x.size)
    return y
