"""CPU: the oracle (oracle/xksv_oracle.c) is pinned to the reference codec
through golden vectors produced by the reference library itself
(tests/golden/make_golden.py), and, when oracle/_ref was compiled here, to
the reference on fresh random slabs."""
import numpy as np
import pytest

from helpers import load_golden, load_negative, words_for
from oracle.oracle import CodecError, Oracle, Reference, reference_available


@pytest.fixture(scope="module")
def oracle():
    return Oracle()


def test_golden_decode(oracle):
    n = 0
    for g in load_golden():
        assert oracle.unpack(g["serial"], g["rows"], g["cols"]) == g["raw"], g["name"]
        if g["parallel"] is not None:
            assert oracle.unpack_parallel(g["parallel"]) == g["raw"], g["name"]
        n += 1
    assert n >= 40


def test_golden_encode_byte_identical(oracle):
    for g in load_golden():
        assert oracle.pack(g["raw"], g["rows"], g["cols"]) == g["serial"], g["name"]
        if g["parallel"] is not None:
            assert oracle.pack_parallel(g["raw"], g["rows"], g["cols"]) == g["parallel"], g["name"]


def test_golden_negative_cases_rejected(oracle):
    neg = load_negative()
    assert len(neg) >= 5
    for k, blob in neg.items():
        with pytest.raises(CodecError):
            if k.startswith("serial"):
                oracle.unpack(blob, 16, 64)
            else:
                oracle.unpack_parallel(blob)


def test_argument_validation_matches_reference_rules(oracle):
    raw = np.arange(64, dtype="<u2").tobytes()
    with pytest.raises(CodecError):
        oracle.pack(raw, 0, 64)            # rows == 0 (c_api.cpp:20)
    with pytest.raises(CodecError):
        oracle.pack(raw[:-1], 1, 64)       # odd byte count
    with pytest.raises(CodecError):
        oracle.pack_parallel(raw, 17, 4)   # parallel rows > 16 (c_api.cpp:46)
    blob = oracle.pack(raw, 4, 16)
    with pytest.raises(CodecError):
        oracle.unpack(blob, 8, 16)         # count != rows*cols (c_api.cpp:33)
    with pytest.raises(CodecError):
        oracle.unpack(blob[:271], 4, 16)   # shorter than the header


@pytest.mark.skipif(not reference_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("kind", ["normal002", "student3", "normal1e4", "uniform", "three_exp", "single"])
def test_oracle_matches_reference_random(oracle, kind):
    ref = Reference()
    rng = np.random.default_rng(hash(kind) % 2**32)
    for rows, cols in [(1, 1), (3, 17), (16, 48), (16, 333), (21, 40)]:
        raw = words_for(kind, rows * cols, rng).astype("<u2").tobytes()
        s = ref.pack(raw, rows, cols)
        assert oracle.pack(raw, rows, cols) == s
        assert oracle.unpack(s, rows, cols) == raw
        if rows <= 16:
            p = ref.pack_parallel(raw, rows, cols)
            assert oracle.pack_parallel(raw, rows, cols) == p
            assert oracle.unpack_parallel(p) == raw
