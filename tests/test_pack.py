"""CPU: the product's archive-side encoder (xksv_host_pack, compile step) is
byte-identical to the reference encoder: checked against the reference's own
golden vectors and, when oracle/_ref exists, against it on random slabs; the
tensor splitter follows src/compile.cpp:449-479 (slab geometry) and
:268-275 (raw fallback)."""
import ctypes

import numpy as np
import pytest

from helpers import load_golden, words_for
from oracle.oracle import Oracle


@pytest.fixture(scope="module")
def xg():
    import build as b
    b.build()
    import xksv_gpu
    xksv_gpu.load()
    return xksv_gpu


def test_host_pack_matches_golden(xg):
    for g in load_golden():
        assert xg.host_pack(g["raw"], g["rows"], g["cols"], xg.CODEC_TILE16) == g["serial"], g["name"]
        if g["parallel"] is not None:
            assert xg.host_pack(g["raw"], g["rows"], g["cols"], xg.CODEC_PARALLEL32) == g["parallel"], g["name"]


@pytest.mark.parametrize("kind", ["normal002", "student3", "normal1e4", "uniform", "three_exp", "single"])
def test_host_pack_matches_oracle(xg, kind):
    o = Oracle()
    rng = np.random.default_rng(len(kind) * 7)
    for rows, cols in [(1, 1), (2, 3), (16, 48), (16, 1000), (19, 77)]:
        raw = words_for(kind, rows * cols, rng).astype("<u2").tobytes()
        assert xg.host_pack(raw, rows, cols, xg.CODEC_TILE16) == o.pack(raw, rows, cols)
        if rows <= 16:
            assert xg.host_pack(raw, rows, cols, xg.CODEC_PARALLEL32) == o.pack_parallel(raw, rows, cols)


def test_host_pack_rejects_like_reference(xg):
    raw = np.arange(64, dtype="<u2").tobytes()
    with pytest.raises(ValueError):
        xg.host_pack(raw, 0, 64, xg.CODEC_TILE16)
    with pytest.raises(ValueError):
        xg.host_pack(raw, 17, 4, xg.CODEC_PARALLEL32)  # parallel slabs have <= 16 rows


@pytest.mark.parametrize("codec", [1, 2])
def test_pack_tensor_geometry_and_fallback(xg, codec):
    o = Oracle()
    rng = np.random.default_rng(codec)
    rows, cols = 70, 5632
    w = words_for("normal002", rows * cols, rng).reshape(rows, cols)
    w[32:48] = words_for("uniform", 16 * cols, rng).reshape(16, cols)  # stored raw
    buf = np.ascontiguousarray(w.astype("<u2"))
    payload, slabs = xg.host_pack_tensor(buf.ctypes.data, buf.nbytes, rows, cols, codec, threads=3,
                                         dst_base=1000)
    assert [s["rows"] for s in slabs] == [16, 16, 16, 16, 6]
    assert [s["codec"] for s in slabs][2] == 0
    pay = payload.tobytes()
    for s in slabs:
        blob = pay[s["src_offset"]:s["src_offset"] + s["src_size"]]
        r0 = (s["dst_offset"] - 1000) // (cols * 2)
        raw = buf[r0:r0 + s["rows"]].tobytes()
        if s["codec"] == 0:
            assert blob == raw
        elif codec == 1:
            assert blob == o.pack(raw, s["rows"], cols)
        else:
            assert blob == o.pack_parallel(raw, s["rows"], cols)
