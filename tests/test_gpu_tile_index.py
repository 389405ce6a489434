"""GPU: the plan tile index (xksv_plan_index) and the tile-parallel fused
GEMV/GEMM it enables for 16-row serial-codec slabs.  The reference computes
out[r*batch + k] = sum_c bf16(W[r, c]) * x[c*batch + k] (cuda/decode.cu:28-45);
results are checked against an FP32 matmul of the oracle-decoded weights, and
slabs the index does not cover (other shapes, other codecs) must still go
through their own kernels in the same call."""
import numpy as np
import pytest

from helpers import TC_MIN_BATCH, bf16_to_f32, rel_l2, words_for
from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def xg():
    import xksv_gpu
    assert torch.cuda.is_available()
    xksv_gpu.load()
    return xksv_gpu


def weights_archive(oracle, mats, kind, rng, codec_for=lambda mi, r0: 1, lead=3):
    """Row-sharded 16-row slabs of each [R, C] matrix at odd payload offsets."""
    payload = bytearray(b"\x00" * lead)
    entries, ws = [], []
    xoff = yrow = 0
    for mi, (R, C) in enumerate(mats):
        w = words_for(kind, R * C, rng).reshape(R, C)
        ws.append(w)
        for r0 in range(0, R, 16):
            rows = min(16, R - r0)
            raw = w[r0:r0 + rows].astype("<u2").tobytes()
            codec = codec_for(mi, r0)
            blob = (oracle.pack(raw, rows, C) if codec == 1 else
                    oracle.pack_parallel(raw, rows, C) if codec == 2 else raw)
            entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=rows, cols=C,
                                dst_offset=yrow + r0, x_offset=xoff, codec=codec))
            payload += blob
            payload += b"\x00" * (len(entries) % 3)
        xoff += C
        yrow += R
    return bytes(payload), entries, ws, xoff, yrow


def check(ws, mats, x, y, tol, plan=None):
    """Against FP32 X below TC_MIN_BATCH (CUDA-core kernels); from there a
    plan with a tensor-core path runs it with X rounded to BF16."""
    xo = yo = 0
    if plan is not None and x.shape[1] >= TC_MIN_BATCH and plan.scratch_bytes():
        x = x.to(torch.bfloat16).float()
    for (R, C), w in zip(mats, ws):
        ref = torch.from_numpy(bf16_to_f32(w)).cuda() @ x[xo:xo + C]
        assert rel_l2(y[yo:yo + R].cpu(), ref.cpu()) < tol, (R, C)
        xo += C
        yo += R


@pytest.mark.parametrize("kind", ["normal002", "student3", "normal1e4"])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 6])
def test_indexed_gemm_matches_fp32(xg, kind, batch):
    oracle = Oracle()
    rng = np.random.default_rng(batch * 7 + len(kind))
    # 16 tiles, 256 tiles (one item), 257 tiles (two items), 896 tiles (4 items)
    mats = [(32, 256), (16, 4096), (32, 4112), (16, 14336)]
    payload, entries, ws, xn, yn = weights_archive(oracle, mats, kind, rng)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(xn, batch, device="cuda")
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0
    for rep in range(2):  # the split-slab counters must be back at zero
        y = torch.full((yn, batch), float("nan"), device="cuda")
        plan.gemm(d_payload, x, y, batch)
        assert plan.status() == 0
        check(ws, mats, x, y, 1e-5, plan)
    if batch < TC_MIN_BATCH:
        assert plan.launches() == 1
    plan.close()


def test_indexed_gemm_is_deterministic(xg):
    oracle = Oracle()
    rng = np.random.default_rng(11)
    mats = [(16, 14336), (48, 4096)]
    payload, entries, ws, xn, yn = weights_archive(oracle, mats, "normal002", rng)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(xn, 1, device="cuda")
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0
    outs = []
    for _ in range(3):
        y = torch.empty(yn, 1, device="cuda")
        plan.gemm(d_payload, x, y, 1)
        assert plan.status() == 0
        outs.append(y.cpu())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    plan.close()


def test_index_multi_round_dense_tiles(xg):
    """Exponents uniform over 128 values: ~7 bits per code, so a CTA's 256
    tiles need several shared-memory rounds of bits."""
    oracle = Oracle()
    rng = np.random.default_rng(12)
    mats = [(16, 4096), (32, 8192)]
    payload = bytearray(b"\x00")
    entries, ws = [], []
    xoff = yrow = 0
    for R, C in mats:
        sign = rng.integers(0, 2, R * C, dtype=np.uint16) << 15
        exp = rng.integers(64, 192, R * C, dtype=np.uint16) << 7
        mant = rng.integers(0, 128, R * C, dtype=np.uint16)
        w = (sign | exp | mant).reshape(R, C)
        ws.append(w)
        for r0 in range(0, R, 16):
            blob = oracle.pack(w[r0:r0 + 16].astype("<u2").tobytes(), 16, C)
            entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=16, cols=C,
                                dst_offset=yrow + r0, x_offset=xoff, codec=1))
            payload += blob
        xoff += C
        yrow += R
    d_payload = torch.frombuffer(payload, dtype=torch.uint8).cuda()
    x = torch.randn(xoff, 1, device="cuda")
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0
    y = torch.empty(yrow, 1, device="cuda")
    plan.gemm(d_payload, x, y, 1)
    assert plan.status() == 0
    check(ws, mats, x, y, 1e-5)
    plan.close()


def test_index_mixed_plan_and_fallbacks(xg):
    """Indexable slabs next to 7-row tails, cols % 16 != 0 and other codecs;
    a different payload pointer falls back to the unindexed kernels."""
    oracle = Oracle()
    rng = np.random.default_rng(13)
    mats = [(39, 2048), (16, 2050), (32, 512), (48, 1024)]
    cyc = lambda mi, r0: [1, 1, 2, 0][(mi + r0 // 16) % 4]
    payload, entries, ws, xn, yn = weights_archive(oracle, mats, "normal002", rng, cyc)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(xn, 2, device="cuda")
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0
    y = torch.full((yn, 2), float("nan"), device="cuda")
    plan.gemm(d_payload, x, y, 2)
    assert plan.status() == 0
    check(ws, mats, x, y, 1e-5)
    copy = d_payload.clone()
    y2 = torch.full((yn, 2), float("nan"), device="cuda")
    plan.gemm(copy, x, y2, 2)
    assert plan.status() == 0
    check(ws, mats, x, y2, 1e-5)
    plan.close()


def test_index_rejects_corrupt_slab(xg):
    oracle = Oracle()
    rng = np.random.default_rng(14)
    mats = [(64, 1024)]
    payload, entries, ws, xn, yn = weights_archive(oracle, mats, "normal002", rng)
    bad = bytearray(payload)
    e = entries[2]
    o = e["src_offset"]
    bad[o + 16:o + 20] = b"\x01\x01\x01\x01"  # four 1-bit codes: oversubscribed
    with pytest.raises(Exception):
        oracle.unpack(bytes(bad[o:o + e["src_size"]]), 16, 1024)
    d_bad = torch.frombuffer(bad, dtype=torch.uint8).cuda()
    plan = xg.Plan(entries)
    assert plan.index(d_bad) == 1
    assert plan.status() == 0  # the index call reports and clears its own error
    d_good = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    assert plan.index(d_good) == 0
    x = torch.randn(xn, 1, device="cuda")
    y = torch.empty(yn, 1, device="cuda")
    plan.gemm(d_good, x, y, 1)
    assert plan.status() == 0
    check(ws, mats, x, y, 1e-5)
    plan.close()


@pytest.mark.parametrize("kind", ["normal002", "student3", "dense7"])
def test_indexed_decode_bit_exact(xg, kind):
    """xksv_plan_decode after xksv_plan_index decodes the 16-row serial slabs
    one thread per tile; every slab's bytes equal the source, at 16-byte and at
    2-byte aligned outputs, next to slabs the index does not cover."""
    oracle = Oracle()
    rng = np.random.default_rng(31 + len(kind))
    shapes = [(16, 4096), (16, 4112), (7, 512), (16, 2050), (16, 256), (16, 8192)]
    payload = bytearray(b"\x00" * 3)
    entries, raws, out = [], [], 0
    for i, (r, c) in enumerate(shapes):
        if kind == "dense7":  # ~7-bit codes: several shared-memory rounds per CTA
            w = ((rng.integers(0, 2, r * c, dtype=np.uint16) << 15) |
                 (rng.integers(64, 192, r * c, dtype=np.uint16) << 7) |
                 rng.integers(0, 128, r * c, dtype=np.uint16))
        else:
            w = words_for(kind, r * c, rng)
        raw = w.astype("<u2").tobytes()
        blob = oracle.pack(raw, r, c) if i % 3 != 2 else oracle.pack_parallel(raw, r, c)
        entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=r, cols=c,
                            dst_offset=out, codec=1 if i % 3 != 2 else 2))
        payload += blob
        raws.append(raw)
        out += len(raw) + (2 if i % 2 else 16)
    d_payload = torch.frombuffer(payload, dtype=torch.uint8).cuda()
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0
    for rep in range(2):
        d_out = torch.full((out + 16,), 0xAB, dtype=torch.uint8, device="cuda")
        plan.decode(d_payload, d_out)
        assert plan.status() == 0
        got = d_out.cpu().numpy().tobytes()
        for e, raw in zip(entries, raws):
            assert got[e["dst_offset"]:e["dst_offset"] + len(raw)] == raw, e
    plan.close()


def test_indexed_one_and_two_threads_per_tile(xg):
    """At batch 1 (and for decode) a launch whose items fill under one wave of
    256-thread CTAs decodes each tile with two threads (rows 0-7 and 8-15, the
    second from the index's row-8 offset); a larger launch uses one.  A plan of
    700 slabs (700 items: one thread per tile) and one of its first 200 (two
    per tile): GEMV against FP32, decode bit-exact, on both."""
    rng = np.random.default_rng(41)
    R, C = 700 * 16, 256
    w = words_for("student3", R * C, rng).reshape(R, C)
    payload = bytearray(b"\x00" * 7)
    entries = []
    for r0 in range(0, R, 16):
        blob = xg.host_pack(w[r0:r0 + 16].astype("<u2").tobytes(), 16, C, 1)
        entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=16, cols=C,
                            dst_offset=r0, x_offset=0, codec=1))
        payload += blob + b"\x00" * (r0 % 3)
    d_payload = torch.frombuffer(payload, dtype=torch.uint8).cuda()
    x = torch.randn(C, 1, device="cuda")
    W = torch.from_numpy(bf16_to_f32(w)).cuda()
    for n in (700, 200):
        plan = xg.Plan(entries[:n])
        assert plan.index(d_payload) == 0
        for _ in range(2):
            y = torch.full((16 * n, 1), float("nan"), device="cuda")
            plan.gemm(d_payload, x, y, 1)
            assert plan.status() == 0 and plan.launches() == 1
            assert rel_l2(y.cpu(), (W[:16 * n] @ x).cpu()) < 1e-5
        dec = [dict(e, dst_offset=2 * C * e["dst_offset"]) for e in entries[:n]]
        dplan = xg.Plan(dec)
        assert dplan.index(d_payload) == 0
        d_out = torch.full((32 * C * n,), 0xAB, dtype=torch.uint8, device="cuda")
        dplan.decode(d_payload, d_out)
        assert dplan.status() == 0
        assert d_out.cpu().numpy().tobytes() == w[:16 * n].astype("<u2").tobytes()
        dplan.close()
        plan.close()
