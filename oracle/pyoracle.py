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
        ("phase_offset", C.c_int32), ("n_threads", C.c_int32), ("preset", C.c_int32),
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
              "e1": 12, "e2": 13, "ampa": 14, "last_pre": 15}
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


def ref_params(n_columns=50, seed=42, e0=0, phase_offset=0, n_threads=0, preset=0):
    """Reference topology rules (src/stage2e/network_init.cu:198-233), scaled by
    column count; n_columns=50 is the reference network (55,000 / 10,700,000).
    preset 0: the reference's constants; 1: the benchmark's AdEx / STP ones."""
    p = O2eParams()
    p.n_columns = n_columns
    p.l4, p.l23, p.l5, p.l6 = 200, 350, 200, 250
    p.pf_groups, p.pf_group_size = n_columns, 100
    p.deg_intra, p.deg_inter, p.deg_l5_pf = 150, 30, 15
    p.deg_pf_self, p.deg_pf_assoc = 100, 50
    p.total_synapses = 10_700_000 * n_columns // 50
    p.seed, p.e0, p.phase_offset, p.n_threads = seed, e0, phase_offset, n_threads
    p.preset = preset
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

    def save_sckp(self, path, step):
        """SCKP v2 file of the current state (the reference scheduler's layout)."""
        L = lib()
        L.o2e_save_sckp.argtypes = [C.c_void_p, C.c_char_p, C.c_int32]
        rc = L.o2e_save_sckp(self.h, path.encode(), step)
        if rc:
            raise OSError(f"o2e_save_sckp failed ({rc})")

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


# ---------------------------------------------------------------------------
# Stage 0 / Stage 2 oracle (oracle/oracle0.cpp)
# ---------------------------------------------------------------------------
class O0Params(C.Structure):
    _fields_ = [("n_columns", C.c_int32), ("n_sens", C.c_int32), ("n_assoc", C.c_int32),
                ("n_motor", C.c_int32), ("deg_intra", C.c_int32), ("deg_inter", C.c_int32),
                ("seed", C.c_uint32), ("w_max", C.c_float), ("input_gain", C.c_float),
                ("homeo_lr", C.c_float), ("homeo_max", C.c_float), ("target_sa", C.c_float),
                ("target_m", C.c_float), ("reset_interval", C.c_int32), ("dopamine", C.c_float),
                ("n_threads", C.c_int32)]


def stage0_params(columnar=False, baseline=True, seed=42, n_threads=0, n_columns=10):
    """Stage 0 block network (configuration 0) or 10-column Stage 2 network
    (configuration 1); baseline=True uses the benchmark constants, False the
    reference Stage 2 build constants (gain 5, LR 0.005, max 0.1, 15 Hz)."""
    p = O0Params()
    if columnar:
        p.n_columns, p.n_sens, p.n_assoc, p.n_motor = n_columns, 200, 600, 200
        p.deg_intra, p.deg_inter = 80, 20
        p.reset_interval = 10000
    else:
        p.n_columns, p.n_sens, p.n_assoc, p.n_motor = 0, 2000, 6000, 2000
        p.deg_intra, p.deg_inter = 100, 0
        p.reset_interval = 0
    p.seed = seed
    if baseline:
        p.w_max, p.input_gain, p.homeo_lr, p.homeo_max = 1.0, 1.5, 1e-4, 2.0
        p.target_sa, p.target_m = 0.005, 0.030
    else:
        p.w_max, p.input_gain, p.homeo_lr, p.homeo_max = 0.3, 5.0, 0.005, 0.1
        p.target_sa, p.target_m = 0.015, 0.030
    p.dopamine = 1.0
    p.n_threads = n_threads
    return p


class Oracle0:
    def __init__(self, params):
        L = lib()
        if not hasattr(L, "_o0_ready"):
            L.o0_create.restype = C.c_void_p
            L.o0_create.argtypes = [C.POINTER(O0Params)]
            L.o0_destroy.argtypes = [C.c_void_p]
            L.o0_run.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
            L.o0_sizes.argtypes = [C.c_void_p, C.c_void_p]
            L.o0_spikes.argtypes = [C.c_void_p, C.c_void_p]
            L.o0_neuron.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
            L.o0_synapse.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
            L.o0_topology.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
            L.o0_set_dopamine.argtypes = [C.c_void_p, C.c_float]
            L._o0_ready = True
        self.L = L
        self.h = L.o0_create(C.byref(params))
        sz = self.sizes()
        self.N, self.S = int(sz[0]), int(sz[1])

    def sizes(self):
        out = np.zeros(5, np.int64)
        self.L.o0_sizes(self.h, out.ctypes.data)
        return out

    def run(self, n, bytes_=None):
        b = None
        if bytes_ is not None:
            b = np.ascontiguousarray(np.asarray(bytes_, dtype=np.int32))
        self.L.o0_run(self.h, n, b.ctypes.data if b is not None else None)

    def spikes(self):
        out = np.zeros(self.N, np.uint8)
        self.L.o0_spikes(self.h, out.ctypes.data)
        return out

    def neuron(self, which):
        idx = {"V": 0, "I": 1, "fr": 2, "input": 3, "last_spk": 4, "off": 5, "ref": 6}[which]
        out = np.zeros(self.N, np.float32)
        self.L.o0_neuron(self.h, idx, out.ctypes.data)
        return out

    def synapse(self, which):
        out = np.zeros(self.S, np.float32)
        self.L.o0_synapse(self.h, {"w": 0, "elig": 1}[which], out.ctypes.data)
        return out

    def topology(self):
        pre = np.zeros(self.S, np.int32)
        post = np.zeros(self.S, np.int32)
        self.L.o0_topology(self.h, pre.ctypes.data, post.ctypes.data)
        return pre, post

    def set_dopamine(self, da):
        self.L.o0_set_dopamine(self.h, da)

    def close(self):
        if self.h:
            self.L.o0_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# Propagation microbench oracle (oracle/oracle4.cpp)
# ---------------------------------------------------------------------------
class O4Params(C.Structure):
    _fields_ = [("n", C.c_int32), ("fanout", C.c_int32), ("seed", C.c_uint32),
                ("mode", C.c_int32), ("rate", C.c_float), ("w_max", C.c_float),
                ("dopamine", C.c_float), ("n_threads", C.c_int32)]


class O4Counters(C.Structure):
    _fields_ = [("step", C.c_int64), ("total_spikes", C.c_int64), ("events", C.c_int64),
                ("pre_spikes", C.c_int64), ("ltp_visits", C.c_int64),
                ("last_spikes", C.c_int32), ("n_exc", C.c_int32), ("n_synapses", C.c_int64)]


def prop_w_max(rate, fanout):
    """Default weight bound of the microbench: 0.01 / (rate * fan-out), as a
    float32 (the value the engine derives when prop_w_max is 0)."""
    if rate <= 0:
        return 1.0
    return float(np.float32(np.float32(0.01) / (np.float32(rate) * np.float32(fanout))))


def prop_params(n=1_000_000, fanout=1000, seed=42, mode=0, rate=0.01, w_max=0.0,
                dopamine=1.0, n_threads=0):
    p = O4Params()
    p.n, p.fanout, p.seed, p.mode, p.rate = n, fanout, seed, mode, rate
    p.w_max = w_max if w_max > 0 else prop_w_max(rate, fanout)
    p.dopamine, p.n_threads = dopamine, n_threads
    return p


class Oracle4:
    FIELDS = {"V": (0, np.float32), "I": (1, np.float32), "u": (2, np.float32),
              "R": (3, np.float32), "ref": (6, np.int32), "last_post": (7, np.int32),
              "last_pre": (8, np.int32)}

    def __init__(self, params):
        L = lib()
        if not hasattr(L, "_o4_ready"):
            L.o4_create.restype = C.c_void_p
            L.o4_create.argtypes = [C.POINTER(O4Params)]
            L.o4_destroy.argtypes = [C.c_void_p]
            L.o4_set_dopamine.argtypes = [C.c_void_p, C.c_float]
            L.o4_run.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
            L.o4_counters.argtypes = [C.c_void_p, C.POINTER(O4Counters)]
            L.o4_get.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
            L.o4_propagate.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32,
                                       C.c_void_p, C.c_void_p, C.c_int32]
            L._o4_ready = True
        self.L = L
        self.P = params
        self.h = L.o4_create(C.byref(params))
        self.N = params.n
        self.S = params.n * params.fanout

    def run(self, n, raster=False):
        r = np.zeros((n, (self.N + 31) // 32), np.uint32) if raster else None
        self.L.o4_run(self.h, n, r.ctypes.data if r is not None else None)
        return r

    def counters(self):
        c = O4Counters()
        self.L.o4_counters(self.h, C.byref(c))
        return {k: getattr(c, k) for k, _ in O4Counters._fields_}

    def neuron(self, name):
        idx, dt = self.FIELDS[name]
        out = np.zeros(self.N, dt)
        self.L.o4_get(self.h, idx, out.ctypes.data)
        return out

    def weights(self):
        out = np.zeros(self.S, np.float32)
        self.L.o4_get(self.h, 4, out.ctypes.data)
        return out

    def post(self):
        out = np.zeros(self.S, np.int32)
        self.L.o4_get(self.h, 5, out.ctypes.data)
        return out

    def set_dopamine(self, da):
        self.L.o4_set_dopamine(self.h, da)

    def close(self):
        if self.h:
            self.L.o4_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def propagate(post, w, fanout, spikes, n_post, frac_bits=24):
    """Closed-form exact push (o4_propagate) of one spike vector."""
    L = lib()
    if not hasattr(L, "_o4_prop_ready"):
        L.o4_propagate.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32,
                                   C.c_void_p, C.c_void_p, C.c_int32]
        L._o4_prop_ready = True
    post = np.ascontiguousarray(post, np.int32)
    w = np.ascontiguousarray(w, np.float32)
    spikes = np.ascontiguousarray(spikes, np.uint8)
    acc = np.zeros(n_post, np.int32)
    L.o4_propagate(post.ctypes.data, w.ctypes.data, len(spikes), fanout, spikes.ctypes.data,
                   acc.ctypes.data, frac_bits)
    return acc


def semantic_eval(nbc, last, region, n_columns, npc, step):
    """Semantic evaluation of a Stage 2e network, restated from
    BioMechanismScheduler::launch_semantic_eval (src/stage2e/scheduler.cu:
    785-1036) with the js_divergence helper (:31-40), the column response
    kernel (:294-310) and the per-neuron chi-squared kernel (:195-231).
    Plain Python loops in the reference's order of operations (math.log is
    the C library's log), the per-neuron chi-squared in float32 and each
    layer's float sum in ascending neuron order.  nbc: int32[N, 256] neuron x
    byte spike counts; last: int32[N] last spike step; region: uint8[N]
    (0 L4, 1 L2/3, 2 L5, 3 L6, 4 prefrontal)."""
    import math
    NB, K = 256, 5
    nbc = np.asarray(nbc, np.int64).reshape(-1, NB)
    resp = nbc[: n_columns * npc].reshape(n_columns, npc, NB).sum(axis=1)
    P, col_total, grand = [], [], 0.0
    for c in range(n_columns):
        s = 0.0
        for b in range(NB):
            s += float(resp[c, b])
        col_total.append(s)
        grand += s
        P.append([1.0 / NB] * NB if s < 1e-10 else [float(resp[c, b]) / s for b in range(NB)])

    def js(p, q):
        v = 0.0
        for b in range(NB):
            m = 0.5 * (p[b] + q[b])
            if p[b] > 1e-12 and m > 1e-12:
                v += 0.5 * p[b] * math.log(p[b] / m)
            if q[b] > 1e-12 and m > 1e-12:
                v += 0.5 * q[b] * math.log(q[b] / m)
        return 0.0 if v < 0.0 else v

    jm = [[0.0] * n_columns for _ in range(n_columns)]
    js_sum, js_max, js_n = 0.0, 0.0, 0
    for i in range(n_columns):
        for j in range(i + 1, n_columns):
            v = js(P[i], P[j])
            jm[i][j] = jm[j][i] = v
            js_sum += v
            js_max = max(js_max, v)
            js_n += 1
    asg = [i % K for i in range(n_columns)]
    for _ in range(20):
        cnt, sp = [0] * K, [[0.0] * NB for _ in range(K)]
        for i in range(n_columns):
            cnt[asg[i]] += 1
            for b in range(NB):
                sp[asg[i]][b] += P[i][b]
        cen = []
        for k in range(K):
            if cnt[k] > 0:
                ck, s = [], 0.0
                for b in range(NB):
                    ck.append(sp[k][b] / cnt[k])
                    s += ck[b]
                cen.append([1.0 / NB] * NB if s < 1e-12 else [x / s for x in ck])
            else:
                cen.append([1.0 / NB] * NB)
        changed = False
        for i in range(n_columns):
            best, bk = float("inf"), 0
            for k in range(K):
                d = js(P[i], cen[k])
                if d < best:
                    best, bk = d, k
            if bk != asg[i]:
                asg[i], changed = bk, True
        if not changed:
            break
    sil, sil_n = 0.0, 0
    for i in range(n_columns):
        a, an, bmin = 0.0, 0, float("inf")
        for k in range(K):
            if k == asg[i]:
                for j in range(n_columns):
                    if j != i and asg[j] == k:
                        a += jm[i][j]
                        an += 1
                if an > 0:
                    a /= an
            else:
                ds, dn = 0.0, 0
                for j in range(n_columns):
                    if asg[j] == k:
                        ds += jm[i][j]
                        dn += 1
                if dn > 0 and ds / dn < bmin:
                    bmin = ds / dn
        if an > 0 and bmin < float("inf"):
            den = max(a, bmin)
            sil += (bmin - a) / den if den > 1e-12 else 0.0
            sil_n += 1
    nzt = [t for t in col_total if t > 0.0]
    li = max(((step - 1) // 3) * 3, 0) if step >= 1 else 0
    tot = nbc.sum(axis=1)
    expected = tot.astype(np.float32) * np.float32(1.0 / 256.0)
    chi = np.zeros(nbc.shape[0], np.float32)
    for b in range(NB):
        diff = nbc[:, b].astype(np.float32) - expected
        chi = chi + (diff * diff) / np.where(expected < 1e-10, np.float32(1), expected)
    chi = np.where(expected < 1e-10, np.float32(0), chi).astype(np.float32)
    out = {"js_mean": js_sum / js_n if js_n else 0.0, "js_max": js_max,
           "silhouette": sil / sil_n if sil_n else 0.0, "grand_total": grand,
           "nonzero_columns": len(nzt), "n_columns": n_columns,
           "column_ratio": max(nzt) / min(nzt) if len(nzt) >= 2 else 0.0, "assign": asg,
           "layer_delay": [], "layer_delay_n": [], "layer_sig": [], "layer_act": [],
           "layer_chi2_mean": []}
    region = np.asarray(region)
    last = np.asarray(last, np.int64)
    for r in range(5):
        sel = np.nonzero(region == r)[0]
        hit = sel[last[sel] >= li]
        out["layer_delay_n"].append(int(hit.size))
        d = 0.0
        for i in hit:
            d += float(last[i] - li)
        out["layer_delay"].append(d / hit.size if hit.size else -1.0)
        act = sel[tot[sel] >= 10]
        cs = np.float32(0)
        for i in act:
            cs = np.float32(cs + chi[i])
        out["layer_act"].append(int(act.size))
        out["layer_sig"].append(int((chi[act] > np.float32(293.2)).sum()))
        out["layer_chi2_mean"].append(float(cs) / act.size if act.size else 0.0)
    return out
