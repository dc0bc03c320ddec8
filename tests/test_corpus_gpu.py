"""GPU test of the text-corpus entry points (snn_load_text_corpus,
snn_set_corpus_ex with SNN_CORPUS_TEXT_FILTER): the network reads exactly the
bytes the reference's filter keeps (src/stage2e/input_encoding.cu:49-64)."""
import os

import numpy as np
import pytest

import pyoracle as po
import snn_b200 as snn

pytestmark = pytest.mark.gpu


def _raster(net, steps):
    r, _ = net.run(steps, raster=True)
    return r


def test_text_corpus_filter_through_the_c_abi(tmp_path):
    body = snn.stream(3000, seed=11, p_cjk=0.452).tobytes()
    raw = bytearray()
    for i in range(0, len(body), 37):  # sprinkle NUL, CR, LF and TAB through the text
        raw += body[i:i + 37] + bytes([(0, 13, 10, 9)[(i // 37) % 4]])
    path = tmp_path / "corpus.txt"
    path.write_bytes(bytes(raw))
    want = po.text_filter(bytes(raw))
    steps = 60
    nets = [snn.Network(device=0, phase_offset=5000) for _ in range(3)]
    try:
        for n in nets:
            n.build_columns(snn.topology(n_columns=2))
        assert nets[0].load_text_corpus(str(path)) == want.size
        assert nets[1].set_corpus(bytes(raw), text_filter=True) == want.size
        assert nets[2].set_corpus(want.tobytes()) == want.size
        rs = [_raster(n, steps) for n in nets]
        assert np.array_equal(rs[0], rs[2]) and np.array_equal(rs[1], rs[2])
        assert rs[2].any()
        with pytest.raises(snn.SnnError) as e:
            nets[0].load_text_corpus(str(tmp_path / "missing.txt"))
        assert e.value.code == 5
        empty = tmp_path / "empty.txt"
        empty.write_bytes(b"\x00\x00")
        with pytest.raises(snn.SnnError):
            nets[0].load_text_corpus(str(empty))
    finally:
        for n in nets:
            n.close()
