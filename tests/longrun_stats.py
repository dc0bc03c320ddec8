"""Long-run statistics of a Stage 2e run, shared by the comparison with the
reference engine (tests/test_longrun_reference.py): per-layer firing rates,
fire-rate traces, the excitatory weight distribution and the mean pairwise
Jensen-Shannon divergence of the columns' byte responses (the reference's
js_mean, src/stage2e/scheduler.cu:771-836, restated with natural logs)."""
import numpy as np

LAYERS = {"L4": (0, 200), "L23": (200, 550), "L5": (550, 750), "L6": (750, 1000)}


def js_divergence(p, q):
    m = 0.5 * (p + q)
    def kl(a, b):
        nz = a > 0
        return float(np.sum(a[nz] * np.log(a[nz] / b[nz])))
    return 0.5 * kl(p, m) + 0.5 * kl(q, m)


def column_js_mean(nbc, n_columns, npc=1000):
    """Mean JS divergence over all column pairs of the columns' byte-response
    distributions (neuron x byte spike counts summed per column; an empty
    column counts as uniform)."""
    nbc = np.asarray(nbc).reshape(-1, 256)
    resp = nbc[: n_columns * npc].reshape(n_columns, npc, 256).sum(axis=1).astype(np.float64)
    tot = resp.sum(axis=1, keepdims=True)
    P = np.where(tot > 0, resp / np.maximum(tot, 1e-300), 1.0 / 256)
    vals = [js_divergence(P[i], P[j]) for i in range(n_columns) for j in range(i + 1, n_columns)]
    return float(np.mean(vals))


def summarize(counts, fire_rate, alpha, beta, flags, nbc, steps, n_columns=50, npc=1000):
    counts = np.asarray(counts, np.float64)
    na = n_columns * npc
    off = np.arange(na) % npc
    out = {"rate_all": counts.sum() / (counts.size * steps)}
    for name, (lo, hi) in LAYERS.items():
        sel = np.nonzero((off >= lo) & (off < hi))[0]
        out[f"rate_{name}"] = counts[sel].sum() / (sel.size * steps)
        out[f"fr_{name}"] = float(np.mean(fire_rate[sel]))
    out["rate_PF"] = counts[na:].sum() / ((counts.size - na) * steps)
    out["fr_PF"] = float(np.mean(fire_rate[na:]))
    exc = (flags & 0x03) != 0
    a, b = alpha[exc].astype(np.float64), beta[exc].astype(np.float64)
    w = 1.5 * a / (a + b)
    out["w_mean"] = float(w.mean())
    out["w_std"] = float(w.std())
    hist, _ = np.histogram(w, bins=30, range=(0.0, 1.5))
    out["w_hist"] = hist / hist.sum()
    out["js_mean"] = column_js_mean(nbc, n_columns, npc)
    return out


def read_reference_stats(path):
    raw = np.fromfile(path, np.uint8)
    N, S, K = raw[:12].view(np.int32)
    o = 12
    def take(n, dt):
        nonlocal o
        a = raw[o:o + n * np.dtype(dt).itemsize].view(dt)
        o += n * np.dtype(dt).itemsize
        return a
    counts = take(N, np.int32)
    fr = take(N, np.float32)
    alpha = take(S, np.float32)
    beta = take(S, np.float32)
    flags = take(S, np.uint8)
    nbc = take(N * 256, np.int32)
    return int(K), counts, fr, alpha, beta, flags, nbc
