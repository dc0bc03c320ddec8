"""snn_propagate_static (the push with a file-scope device scratch, no
allocation) against snn_propagate: the same sums on two calls in a row.
Kept in its own file, collected last, so that it runs both alone and after
every other test of the session."""
import numpy as np
import pytest

import snn_b200 as snn


def arrays(n_pre, fanout, n_post, seed, rate=0.05):
    rng = np.random.default_rng(seed)
    post = rng.integers(0, n_post, size=n_pre * fanout).astype(np.int32)
    w = rng.uniform(-0.25, 0.25, size=n_pre * fanout).astype(np.float32)
    sp = (rng.random(n_pre) < rate).astype(np.uint8)
    return post, w, sp


@pytest.mark.gpu
@pytest.mark.parametrize("n_pre,fanout", [(20000, 1000), (1 << 20, 8), (3001, 37)])
def test_static_matches_allocating_entry_point(n_pre, fanout):
    import torch
    dev = torch.device("cuda:0")
    n_post = 50000
    post, w, sp = arrays(n_pre, fanout, n_post, seed=n_pre + fanout)
    tp, tw, ts = (torch.from_numpy(a).to(dev) for a in (post, w, sp))
    ref = torch.zeros(n_post, dtype=torch.int32, device=dev)
    got = torch.zeros(n_post, dtype=torch.int32, device=dev)
    for _ in range(2):  # two calls in a row, accumulating
        snn.propagate(tp, tw, fanout, ts, ref, frac_bits=22)
        snn.propagate(tp, tw, fanout, ts, got, frac_bits=22, static=True)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    # and both equal the exact closed form
    q = np.rint(w.astype(np.float64) * 2.0 ** 22).astype(np.int64)
    m = np.repeat(sp, fanout).astype(bool)
    want = np.zeros(n_post, np.int64)
    np.add.at(want, post[m], 2 * q[m])
    assert np.array_equal(got.cpu().numpy().astype(np.int64), want)


@pytest.mark.gpu
def test_static_rejects_oversize_input():
    """n_pre above the 1,048,576-entry scratch is refused before any launch."""
    import torch
    dev = torch.device("cuda:0")
    n_pre = (1 << 20) + 1
    tp = torch.zeros(n_pre, dtype=torch.int32, device=dev)
    tw = torch.zeros(n_pre, dtype=torch.float32, device=dev)
    ts = torch.zeros(n_pre, dtype=torch.uint8, device=dev)
    acc = torch.zeros(16, dtype=torch.int32, device=dev)
    with pytest.raises(snn.SnnError) as e:
        snn.propagate(tp, tw, 1, ts, acc, static=True)
    assert e.value.code == 1 and "static scratch" in str(e.value)


@pytest.mark.gpu
def test_static_calls_allocate_nothing():
    """After a warm-up call, static calls of several sizes leave the device's
    free memory exactly as it was (no cudaMalloc behind them)."""
    import torch
    dev = torch.device("cuda:0")
    n_post = 40000
    bufs = []
    for n_pre, fanout in ((5000, 64), (200000, 4), (1 << 20, 2)):
        post, w, sp = arrays(n_pre, fanout, n_post, seed=7 * n_pre + fanout)
        bufs.append([torch.from_numpy(a).to(dev) for a in (post, w, sp)] + [fanout])
    acc = torch.zeros(n_post, dtype=torch.int32, device=dev)
    tp, tw, ts, f = bufs[0]
    snn.propagate(tp, tw, f, ts, acc, static=True)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(dev)[0]
    for tp, tw, ts, f in bufs * 2:
        snn.propagate(tp, tw, f, ts, acc, static=True)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free0
