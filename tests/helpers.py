"""Shared test helpers: golden fixtures, seeded slab generators, reference
checkers.  The oracle (oracle/) is the checker only; products under test are
called through the C ABI."""
import hashlib
import struct
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden" / "golden.npz"
FORMULA_PREFIXES = ("iota_", "all_patterns_")
# xksv_plan_gemm runs batches from this size on the tensor cores (X rounded
# to BF16) when the plan allows it (xksv_plan_scratch_bytes > 0)
TC_MIN_BATCH = 4


def bf16_bits(x):
    """float32 -> BF16 bit patterns, round-to-nearest-even (finite input)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(words):
    return (np.asarray(words, dtype=np.uint32) << 16).view(np.float32)


def load_golden():
    """Yields dicts: name, rows, cols, raw, serial, parallel (or None), sha256."""
    z = np.load(GOLDEN)
    for name in z["names"]:
        name = str(name)
        rows, cols = (int(v) for v in z[f"{name}/shape"])
        if name.startswith(FORMULA_PREFIXES):
            raw = (np.arange(rows * cols) % 65536).astype("<u2").tobytes()
        else:
            raw = z[f"{name}/raw"].tobytes()
        sha = z[f"{name}/sha256"].tobytes()
        assert hashlib.sha256(raw).digest() == sha, name
        par = z[f"{name}/parallel"].tobytes() if f"{name}/parallel" in z.files else None
        yield dict(name=name, rows=rows, cols=cols, raw=raw, serial=z[f"{name}/serial"].tobytes(),
                   parallel=par, sha256=sha)


def load_negative():
    z = np.load(GOLDEN)
    return {k.split("/", 1)[1]: z[k].tobytes() for k in z.files if k.startswith("neg/")}


def words_for(kind, n, rng):
    if kind == "normal002":
        return bf16_bits(rng.standard_normal(n) * 0.02)
    if kind == "student3":
        return bf16_bits(rng.standard_t(3, n) * 0.02)
    if kind == "normal1e4":
        return bf16_bits(rng.standard_normal(n) * 1e-4)
    if kind == "uniform":
        return rng.integers(0, 65536, n).astype(np.uint16)
    if kind == "three_exp":
        return (((127 + (np.arange(n) % 3)) << 7) | rng.integers(0, 128, n)).astype(np.uint16)
    if kind == "single":
        return np.full(n, 0x3F80, np.uint16)
    raise ValueError(kind)


def parallel_segments(blob):
    """(offset, length) of each substream of an XKSP2 slab."""
    chunks = struct.unpack_from("<Q", blob, 24)[0]
    pos = 32 + 8 * chunks
    out = []
    for i in range(chunks):
        ln = struct.unpack_from("<Q", blob, 32 + 8 * i)[0]
        out.append((pos, ln))
        pos += ln
    return out


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ---- hand-built blocks (codebooks the reference encoder would not emit) ----
def canonical_codes(lengths):
    """Canonical code strings for a 256-entry length table, built the way
    src/codec.cpp:11-29 assigns them; None if oversubscribed."""
    order = sorted((l, s) for s, l in enumerate(lengths) if l)
    codes = {}
    code = ""
    for l, s in order:
        if not code:
            code = "0" * l
        else:
            i = len(code) - 1
            lst = list(code)
            while i >= 0 and lst[i] == "1":
                lst[i] = "0"
                i -= 1
            if i < 0:
                return None
            lst[i] = "1"
            code = "".join(lst) + "0" * (l - len(code))
        codes[s] = code
    return codes


def encode_with_lengths(tiled_words, lengths):
    """Serial block (c_api.cpp:24-25 layout) of already-tiled words with a
    caller-chosen length table."""
    codes = canonical_codes(lengths)
    bits = "".join(codes[(w >> 7) & 255] for w in tiled_words)
    sm = bytes((((w >> 8) & 0x80) | (w & 0x7F)) for w in tiled_words)
    nbits = len(bits)
    padded = bits + "0" * (-nbits % 8)
    ex = bytes(int(padded[i:i + 8], 2) for i in range(0, len(padded), 8))
    return (struct.pack("<QQ", len(tiled_words), nbits) + bytes(lengths) + sm + ex)


def tile16(words, rows, cols):
    """Row-major -> 16x16 tile order (src/layout.cpp:32-50)."""
    w = np.asarray(words).reshape(rows, cols)
    out = []
    for r in range(0, rows, 16):
        for c in range(0, cols, 16):
            out.extend(w[r:r + 16, c:c + 16].reshape(-1).tolist())
    return out


def parallel_from_segments(rows, cols, segments):
    head = b"XKSP2\0\0\0" + struct.pack("<QQQ", rows, cols, len(segments))
    head += b"".join(struct.pack("<Q", len(s)) for s in segments)
    return head + b"".join(segments)
