"""GPU parity: every decode through the C ABI is bit-exact against the
oracle / the reference's golden vectors; fused GEMV/GEMM match an FP32
matmul of the decoded weights within the stated tolerances.

Shapes and tolerances follow the reference's tests/test_cuda.py (decode
:14-22, GEMV :26-33 atol=rtol=1e-5, GEMM :37-42, parallel decode :50-60,
truncated slab :62-65, parallel GEMV :68-73 atol=rtol=1e-3) and
tests/test_core.cpp:12-18 (all 65536 patterns, single symbol, truncation,
tile edges)."""
import ctypes
import hashlib
import struct

import numpy as np
import pytest

from helpers import (bf16_bits, bf16_to_f32, encode_with_lengths, load_golden, load_negative,
                     parallel_from_segments, parallel_segments, rel_l2, tile16, words_for)
from oracle.oracle import CodecError, Oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    import xksv_gpu
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return xksv_gpu.load()


@pytest.fixture(scope="module")
def oracle():
    return Oracle()


def gpu_decode(lib, blob, rows, cols, parallel=False, offset=0):
    buf = ctypes.create_string_buffer(blob, len(blob))
    out = torch.full((rows * cols * 2 + offset + 16,), 0xAB, dtype=torch.uint8, device="cuda")
    ptr = out.data_ptr() + offset
    rc = (lib.xksv_cuda_decode_parallel(buf, len(blob), ptr) if parallel
          else lib.xksv_cuda_decode(buf, len(blob), rows, cols, ptr))
    data = out.cpu().numpy().tobytes()
    # bytes outside the slab's output must be untouched
    assert data[:offset] == b"\xab" * offset
    assert data[offset + rows * cols * 2:] == b"\xab" * 16
    return rc, data[offset:offset + rows * cols * 2]


def test_golden_serial_and_parallel(lib):
    for g in load_golden():
        rc, got = gpu_decode(lib, g["serial"], g["rows"], g["cols"])
        assert rc == 0 and got == g["raw"], g["name"]
        assert hashlib.sha256(got).digest() == g["sha256"]
        if g["parallel"] is not None:
            rc, got = gpu_decode(lib, g["parallel"], g["rows"], g["cols"], parallel=True)
            assert rc == 0 and got == g["raw"], g["name"] + " (parallel)"


def test_golden_negatives_rejected(lib):
    for k, blob in load_negative().items():
        rc, _ = gpu_decode(lib, blob, 16, 64, parallel=k.startswith("parallel"))
        assert rc == 1, k


@pytest.mark.parametrize("rows,cols", [(1, 1), (1, 256), (7, 19), (16, 32), (17, 33), (31, 103),
                                       (16, 4096), (16, 4097), (33, 35), (16, 14336)])
@pytest.mark.parametrize("kind", ["three_exp", "uniform", "normal002", "student3", "normal1e4", "single"])
def test_random_slabs(lib, oracle, rows, cols, kind):
    rng = np.random.default_rng(rows * 7919 + cols * 31 + len(kind))
    raw = words_for(kind, rows * cols, rng).astype("<u2").tobytes()
    blob = oracle.pack(raw, rows, cols)
    rc, got = gpu_decode(lib, blob, rows, cols)
    assert rc == 0 and got == raw
    if rows <= 16:
        pblob = oracle.pack_parallel(raw, rows, cols)
        rc, got = gpu_decode(lib, pblob, rows, cols, parallel=True)
        assert rc == 0 and got == raw


@pytest.mark.parametrize("offset", [2, 6, 10])
def test_unaligned_output(lib, oracle, offset):
    rng = np.random.default_rng(offset)
    raw = words_for("normal002", 16 * 512, rng).astype("<u2").tobytes()
    for par in (False, True):
        blob = oracle.pack_parallel(raw, 16, 512) if par else oracle.pack(raw, 16, 512)
        rc, got = gpu_decode(lib, blob, 16, 512, parallel=par, offset=offset)
        assert rc == 0 and got == raw


def test_corrupted_streams_match_oracle_verdict(lib, oracle):
    """Random bit flips in the exponent stream / length table: the GPU
    accepts exactly the blobs the CPU codec accepts, with the same output."""
    rng = np.random.default_rng(99)
    raw = words_for("normal002", 16 * 256, rng).astype("<u2").tobytes()
    base_s = bytearray(oracle.pack(raw, 16, 256))
    base_p = bytearray(oracle.pack_parallel(raw, 16, 256))
    accepted = rejected = 0
    for trial in range(120):
        par = trial % 2 == 1
        b = bytearray(base_p if par else base_s)
        if par:
            seg_off, seg_len = parallel_segments(bytes(b))[trial % 32]
            lo, hi = (seg_off + 16, seg_off + 272) if trial % 3 == 0 else (seg_off + 272, seg_off + seg_len)
        else:
            lo, hi = (16, 272) if trial % 3 == 0 else (272 + 4096, len(b))
        for _ in range(1 + trial % 3):
            i = int(rng.integers(lo, hi))
            b[i] ^= 1 << int(rng.integers(0, 8))
        blob = bytes(b)
        try:
            want = oracle.unpack_parallel(blob) if par else oracle.unpack(blob, 16, 256)
        except CodecError:
            want = None
        rc, got = gpu_decode(lib, blob, 16, 256, parallel=par)
        if want is None:
            assert rc == 1, trial
            rejected += 1
        else:
            assert rc == 0 and got == want, trial
            accepted += 1
    assert rejected > 10


def test_truncated_parallel_slab(lib, oracle):
    # tests/test_cuda.py:62-65
    raw = (np.arange(16 * 4097) % 65536).astype("<u2").tobytes()
    blob = oracle.pack_parallel(raw, 16, 4097)
    rc, _ = gpu_decode(lib, blob[:-1], 16, 4097, parallel=True)
    assert rc == 1
    with pytest.raises(CodecError):
        oracle.unpack_parallel(blob[:-1])


def _long_code_lengths(maxlen, nsym, rng):
    """A complete canonical length table with lengths up to maxlen."""
    lens = [0] * 256
    syms = rng.choice(256, size=nsym, replace=False)
    # lengths 1, 2, ..., k then fill the last level to complete Kraft
    ls = list(range(1, maxlen)) + [maxlen, maxlen]
    ls = ls[:nsym] if nsym <= len(ls) else ls
    for s, l in zip(syms, ls):
        lens[int(s)] = l
    return lens, [int(s) for s in syms[:len(ls)]]


@pytest.mark.parametrize("maxlen", [12, 20, 24, 31, 33, 40, 60])
def test_long_codes(lib, oracle, maxlen):
    """Code lengths beyond every table level (the format allows up to 255),
    each used at least once."""
    rng = np.random.default_rng(maxlen)
    lens, syms = _long_code_lengths(maxlen, maxlen + 1, rng)
    rows, cols = 16, 64
    n = rows * cols
    # frequent short codes, but every symbol appears
    pick = [syms[min(int(k), len(syms) - 1)] for k in rng.geometric(0.5, n) - 1]
    pick[:len(syms)] = syms
    words = [((s << 7) | int(rng.integers(0, 128)) | (int(rng.integers(0, 2)) << 15)) for s in pick]
    tiled = tile16(words, rows, cols)
    blob = encode_with_lengths(tiled, lens)
    raw = np.asarray(words, dtype="<u2").tobytes()
    assert oracle.unpack(blob, rows, cols) == raw
    rc, got = gpu_decode(lib, blob, rows, cols)
    assert rc == 0 and got == raw
    # the same codebook in every substream of a parallel slab
    segs = []
    for i in range(32):
        s, e = n * i // 32, n * (i + 1) // 32
        segs.append(encode_with_lengths(tiled[s:e], lens))
    pblob = parallel_from_segments(rows, cols, segs)
    assert oracle.unpack_parallel(pblob) == raw
    rc, got = gpu_decode(lib, pblob, rows, cols, parallel=True)
    assert rc == 0 and got == raw


def test_incomplete_codebook_invalid_code(lib, oracle):
    """Kraft sum < 1: a code outside the codebook must be rejected."""
    lens = [0] * 256
    lens[100], lens[101] = 1, 2   # codes 0, 10 ; prefix 11 is unassigned
    words = [(100 << 7)] * 15 + [(101 << 7)]
    tiled = tile16(words, 1, 16)
    blob = bytearray(encode_with_lengths(tiled, lens))
    assert oracle.unpack(bytes(blob), 1, 16) == np.asarray(words, "<u2").tobytes()
    rc, got = gpu_decode(lib, bytes(blob), 1, 16)
    assert rc == 0
    blob[272 + 16] |= 0xC0  # first code becomes 11...
    with pytest.raises(CodecError):
        oracle.unpack(bytes(blob), 1, 16)
    rc, _ = gpu_decode(lib, bytes(blob), 1, 16)
    assert rc == 1


# ------------------------------------------------------------ GEMV / GEMM --
def _weights(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(rows, cols, generator=g).to(torch.bfloat16)


@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 19), (16, 32), (17, 33), (16, 4096), (33, 2048)])
def test_gemv_serial(lib, oracle, rows, cols):
    w = _weights(rows, cols, rows * cols)
    blob = oracle.pack(w.view(torch.uint8).numpy().tobytes(), rows, cols)
    buf = ctypes.create_string_buffer(blob, len(blob))
    x = torch.randn(cols, device="cuda")
    out = torch.full((rows,), float("nan"), device="cuda")
    assert lib.xksv_cuda_gemv(buf, len(blob), rows, cols, x.data_ptr(), out.data_ptr()) == 0
    ref = w.float().cuda() @ x
    if cols <= 64:
        assert torch.allclose(out, ref, atol=1e-5, rtol=1e-5)
    assert rel_l2(out.cpu(), ref.cpu()) < 1e-5


@pytest.mark.parametrize("rows,cols,batch", [(3, 7, 2), (17, 33, 4), (16, 4096, 3), (16, 1024, 11), (32, 256, 16)])
def test_gemm_serial(lib, oracle, rows, cols, batch):
    w = _weights(rows, cols, rows + cols + batch)
    blob = oracle.pack(w.view(torch.uint8).numpy().tobytes(), rows, cols)
    buf = ctypes.create_string_buffer(blob, len(blob))
    x = torch.randn(cols, batch, device="cuda")
    out = torch.full((rows, batch), float("nan"), device="cuda")
    assert lib.xksv_cuda_gemm(buf, len(blob), rows, cols, batch, x.data_ptr(), out.data_ptr()) == 0
    ref = w.float().cuda() @ x
    if cols <= 64:
        assert torch.allclose(out, ref, atol=1e-5, rtol=1e-5)
    assert rel_l2(out.cpu(), ref.cpu()) < 1e-5


@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 19), (16, 256), (16, 4096), (16, 5632)])
def test_gemv_parallel(lib, oracle, rows, cols):
    w = _weights(rows, cols, 5 * rows + cols)
    blob = oracle.pack_parallel(w.view(torch.uint8).numpy().tobytes(), rows, cols)
    buf = ctypes.create_string_buffer(blob, len(blob))
    x = torch.randn(cols, device="cuda")
    out = torch.full((rows,), float("nan"), device="cuda")
    assert lib.xksv_cuda_gemv_parallel(buf, len(blob), x.data_ptr(), out.data_ptr()) == 0
    ref = w.float().cuda() @ x
    assert torch.allclose(out, ref, atol=1e-3, rtol=1e-3)
    assert rel_l2(out.cpu(), ref.cpu()) < 1e-5


def test_gemv_rejects_bad_slab(lib, oracle):
    w = _weights(16, 64, 3)
    blob = oracle.pack(w.view(torch.uint8).numpy().tobytes(), 16, 64)
    x = torch.randn(64, device="cuda")
    out = torch.empty(16, device="cuda")
    bad = blob[:-1]
    buf = ctypes.create_string_buffer(bad, len(bad))
    assert lib.xksv_cuda_gemv(buf, len(bad), 16, 64, x.data_ptr(), out.data_ptr()) == 1
