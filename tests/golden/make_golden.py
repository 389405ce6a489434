"""Generates tests/golden/golden.npz from the reference CPU codec itself.

Run here, where the reference sources exist and oracle/Makefile compiles them
into oracle/_ref/libxksv_native.so:

    make -C oracle && python tests/golden/make_golden.py

Every case stores the raw BF16 slab (little-endian u16, row-major), the
reference's own ``xksv_pack`` output (src/c_api.cpp:18-28) and, for slabs of at
most 16 rows, its ``xksv_pack_parallel`` output (src/c_api.cpp:44-65), plus the
SHA-256 of the raw bytes (the per-block hash the archive index stores,
src/compile.cpp:251, 468).  Shapes follow the reference tests: tests/test_cuda.py
:14-22 and :50-60 and :68-73, tests/test_core.cpp:12-18; plus one slab of each
BASELINE value distribution.  Inputs are seeded numpy draws (not the reference
tests' own RNG streams), so the fixtures are reproducible from this script.

Negative cases hold reference-rejected blobs (``unpack`` returns non-zero).
"""
import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle.oracle import CodecError, Reference  # noqa: E402


# Cases whose raw words are a formula of the index are stored without their raw
# bytes; tests rebuild them with ``formula_words`` and check the stored SHA-256.
FORMULA_PREFIXES = ("iota_", "all_patterns_")


def formula_words(name, rows, cols):
    return (np.arange(rows * cols) % 65536).astype(np.uint16)


def bf16_bits(x):
    """float32 -> BF16 bit patterns with round-to-nearest-even (NaN-free input)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def make_cases():
    rng = np.random.default_rng(20260101)
    cases = []

    def add(name, rows, cols, words):
        cases.append((name, rows, cols, np.asarray(words, dtype=np.uint16).reshape(rows, cols)))

    # tests/test_cuda.py:14-22 shapes x {3-exponent words, uniform 16-bit}
    for rows, cols in [(1, 1), (1, 256), (7, 19), (16, 32), (17, 33), (31, 103)]:
        n = rows * cols
        add(f"three_exp_{rows}x{cols}", rows, cols,
            ((127 + (np.arange(n) % 3)) << 7) | rng.integers(0, 128, n))
        add(f"uniform_{rows}x{cols}", rows, cols, rng.integers(0, 65536, n))
    # tests/test_cuda.py:50-60 parallel shapes with words i % 65536
    for rows, cols in [(1, 1), (1, 256), (7, 19), (16, 32), (16, 4096), (16, 4097)]:
        add(f"iota_{rows}x{cols}", rows, cols, np.arange(rows * cols) % 65536)
    # tests/test_core.cpp:12-16: every BF16 pattern (NaN/Inf/subnormal/+-0), a
    # shuffled prefix, and a single-symbol block of 0x8000
    add("all_patterns_256x256", 256, 256, np.arange(65536))
    add("shuffled_16x255", 16, 255, rng.permutation(65536)[: 16 * 255])
    add("single_symbol_8x125", 8, 125, np.full(1000, 0x8000))
    # tests/test_core.cpp:18 tile edges (rows 1/7/32/33 x cols 1/9/32/35)
    for rows in (1, 7, 32, 33):
        for cols in (1, 9, 32, 35):
            add(f"edge_{rows}x{cols}", rows, cols, np.arange(rows * cols) * 37 % 65536)
    # BASELINE value distributions, one slab each
    add("normal002_16x4096", 16, 4096, bf16_bits(rng.standard_normal(16 * 4096) * 0.02))
    add("student3_16x2048", 16, 2048, bf16_bits(rng.standard_t(3, 16 * 2048) * 0.02))
    add("normal1e4_16x2048", 16, 2048, bf16_bits(rng.standard_normal(16 * 2048) * 1e-4))
    add("uniform_16x1024", 16, 1024, rng.integers(0, 65536, 16 * 1024))
    return cases


def main():
    ref = Reference()
    out = {}
    names = []
    for name, rows, cols, words in make_cases():
        raw = words.astype("<u2").tobytes()
        serial = ref.pack(raw, rows, cols)
        assert ref.unpack(serial, rows, cols) == raw
        if not name.startswith(FORMULA_PREFIXES):
            out[f"{name}/raw"] = np.frombuffer(raw, np.uint8)
        out[f"{name}/serial"] = np.frombuffer(serial, np.uint8)
        out[f"{name}/shape"] = np.array([rows, cols], np.uint64)
        out[f"{name}/sha256"] = np.frombuffer(hashlib.sha256(raw).digest(), np.uint8)
        if rows <= 16:
            par = ref.pack_parallel(raw, rows, cols)
            assert ref.unpack_parallel(par) == raw
            out[f"{name}/parallel"] = np.frombuffer(par, np.uint8)
        names.append(name)
    # negative cases: blobs the reference rejects
    raw = (np.arange(16 * 64) * 7 % 65536).astype("<u2").tobytes()
    serial = bytearray(ref.pack(raw, 16, 64))
    neg = {}
    t = bytearray(serial)  # one bit short, bytes unchanged -> trailing data
    t[8:16] = (int.from_bytes(serial[8:16], "little") - 1).to_bytes(8, "little")
    neg["serial_bitcount_minus1"] = t
    neg["serial_truncated_byte"] = serial[:-1]
    t = bytearray(serial)  # oversubscribed codebook: give every symbol length 1
    for i in range(256):
        if t[16 + i]:
            t[16 + i] = 1
    neg["serial_oversubscribed"] = t
    par = bytearray(ref.pack_parallel(raw, 16, 64))
    neg["parallel_truncated"] = par[:-1]
    t = bytearray(par)
    t[0] = ord("Y")
    neg["parallel_bad_magic"] = t
    for k, blob in neg.items():
        try:
            if k.startswith("serial"):
                ref.unpack(bytes(blob), 16, 64)
            else:
                ref.unpack_parallel(bytes(blob))
            raise SystemExit(f"reference accepted negative case {k}")
        except CodecError:
            pass
        out[f"neg/{k}"] = np.frombuffer(bytes(blob), np.uint8)
    out["names"] = np.array(names)
    path = Path(__file__).with_name("golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size} bytes, {len(names)} cases)")


if __name__ == "__main__":
    main()
