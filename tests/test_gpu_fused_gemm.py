"""GPU: the fused decode -> tensor-core GEMM of indexed 16-row serial-codec
slabs (xksv_plan_gemm on an indexed plan, 4 <= batch <= 128): one kernel
decodes every tile row into the MMA operand stages, no decoded weight is
written to memory.  The tensor cores take X rounded to BF16, so results are
compared with an FP32 matmul of the source weights against BF16-rounded X
(relative L2 < 1e-5) and against the FP32 X the reference multiplies (< 1e-2,
the task's bound), and with the decode-to-scratch route of the same plan."""
import numpy as np
import pytest

from helpers import bf16_to_f32, rel_l2, words_for

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def xg():
    import xksv_gpu
    assert torch.cuda.is_available()
    xksv_gpu.load()
    return xksv_gpu


def archive(xg, mats, seed, dist="normal002", lead=3):
    """Serial-codec slabs of 16 rows for each (rows, cols, x_offset) weight;
    Y rows follow one another.  Returns payload, entries, weights, X rows, Y rows."""
    rng = np.random.default_rng(seed)
    payload = bytearray(b"\x00" * lead)
    entries, ws = [], []
    yrow = 0
    xn = 0
    for R, C, xoff in mats:
        w = words_for(dist, R * C, rng).reshape(R, C)
        ws.append((w, xoff, yrow))
        for r0 in range(0, R, 16):
            blob = xg.host_pack(w[r0:r0 + 16].astype("<u2").tobytes(), 16, C, 1)
            entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=16, cols=C,
                                dst_offset=yrow + r0, x_offset=xoff, codec=1))
            payload += blob
        yrow += R
        xn = max(xn, xoff + C)
    return bytes(payload), entries, ws, xn, yrow


def check(ws, x, y, tight=1e-5):
    xb = x.to(torch.bfloat16).float()
    for w, xoff, y0 in ws:
        R, C = w.shape
        W = torch.from_numpy(bf16_to_f32(w)).cuda()
        got = y[y0:y0 + R].cpu()
        assert rel_l2(got, (W @ xb[xoff:xoff + C]).cpu()) < tight, (R, C)
        assert rel_l2(got, (W @ x[xoff:xoff + C]).cpu()) < 1e-2, (R, C)


# groups of 32 slabs and partial groups, two weights sharing X columns, one
# at an X offset, and a 40-slab weight (one full group + 8 lanes)
MATS = [(512, 1024, 0), (48, 1024, 0), (640, 2048, 1024), (16, 4096, 0)]


@pytest.mark.parametrize("batch", [4, 16, 17, 32, 48, 64, 100, 128])
def test_fused_gemm_matches_fp32(xg, batch):
    payload, entries, ws, xn, yn = archive(xg, MATS, seed=batch)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(xn, batch, device="cuda")
    plan = xg.Plan(entries)
    assert not plan.fused_ready(d_payload)
    assert plan.index(d_payload) == 0
    assert plan.fused_ready(d_payload)
    for _ in range(2):
        y = torch.full((yn, batch), float("nan"), device="cuda")
        plan.gemm(d_payload, x, y, batch)
        assert plan.launches() == 2  # the prep kernel (X^T, zeroed rows) and the fused kernel
        assert plan.status() == 0
        check(ws, x, y)
    plan.close()


@pytest.mark.parametrize("batch", [16, 64])
def test_fused_gemm_agrees_with_scratch_route(xg, batch):
    payload, entries, ws, xn, yn = archive(xg, MATS, seed=100 + batch, dist="student3")
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(xn, batch, device="cuda")
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0
    y_fused = torch.full((yn, batch), float("nan"), device="cuda")
    plan.gemm(d_payload, x, y_fused, batch)
    assert plan.status() == 0
    plan.set_gemm_route(xg.GEMM_SCRATCH)
    y_scr = torch.full((yn, batch), float("nan"), device="cuda")
    plan.gemm(d_payload, x, y_scr, batch)
    assert plan.launches() != 2
    assert plan.status() == 0
    assert rel_l2(y_fused.cpu(), y_scr.cpu()) < 1e-6
    check(ws, x, y_fused)
    plan.close()


def test_fused_gemm_long_slabs(xg):
    """Llama-3-70B down_proj-wide slabs (16 x 28672) and heavy-tailed weights:
    long codebooks and a tile range split over many CTAs."""
    payload, entries, ws, xn, yn = archive(xg, [(64, 28672, 0)], seed=7, dist="student3")
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(xn, 16, device="cuda")
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0 and plan.fused_ready(d_payload)
    y = torch.full((yn, 16), float("nan"), device="cuda")
    plan.gemm(d_payload, x, y, 16)
    assert plan.status() == 0
    check(ws, x, y)
    plan.close()


def test_fused_gemm_reports_bad_stream(xg):
    """A bit stream changed after the index was built (same payload pointer;
    the index and the lane tables describe the old contents): a one-symbol
    codebook (code 0) meets 1 bits, which no code starts with; the fused kernel
    reports the stream error."""
    payload, entries, ws, xn, yn = archive(xg, [(64, 1024, 0)], seed=9, dist="single")
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0 and plan.fused_ready(d_payload)
    x = torch.randn(xn, 16, device="cuda")
    y = torch.empty(yn, 16, device="cuda")
    plan.gemm(d_payload, x, y, 16)
    assert plan.status() == 0
    e = entries[1]
    bits = e["src_offset"] + 272 + e["rows"] * e["cols"]  # header + lengths, sign/mantissa bytes, then bits
    d_payload[bits:bits + 8] = 0xFF
    plan.gemm(d_payload, x, y, 16)
    assert plan.status() == 1
    plan.close()


def test_fused_route_not_taken_outside_its_range(xg):
    """Batch 3 stays on the CUDA-core GEMV, batch 129 on the scratch route; a
    plan with a parallel-codec slab has no fused route."""
    payload, entries, ws, xn, yn = archive(xg, [(64, 1024, 0)], seed=11)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0 and plan.fused_ready(d_payload)
    for batch in (3, 129):
        x = torch.randn(xn, batch, device="cuda")
        y = torch.full((yn, batch), float("nan"), device="cuda")
        plan.gemm(d_payload, x, y, batch)
        assert plan.status() == 0 and plan.launches() != 2
        check(ws, x, y, tight=1e-5 if batch > 3 else 1e-2)
    plan.close()
    rng = np.random.default_rng(12)
    w = words_for("normal002", 16 * 1024, rng).reshape(16, 1024)
    blob = xg.host_pack(w.astype("<u2").tobytes(), 16, 1024, 2)
    e2 = dict(src_offset=len(payload), src_size=len(blob), rows=16, cols=1024, dst_offset=yn, x_offset=0, codec=2)
    d2 = torch.frombuffer(bytearray(payload + blob), dtype=torch.uint8).cuda()
    plan = xg.Plan(entries + [e2])
    assert plan.index(d2) == 0 and not plan.fused_ready(d2)
    plan.close()


@pytest.mark.parametrize("dist, fused", [("single", True), ("three_exp", True), ("normal1e4", True),
                                         ("uniform", False)])
def test_fused_gemm_codebook_shapes(xg, dist, fused):
    """One-symbol and three-symbol codebooks take the fused route; uniform
    16-bit patterns (about 256 codes of 8 bits) do not fit its lane tables and
    stay on the scratch route."""
    payload, entries, ws, xn, yn = archive(xg, [(96, 512, 0)], seed=13, dist=dist)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    plan = xg.Plan(entries)
    assert plan.index(d_payload) == 0
    assert plan.fused_ready(d_payload) == fused
    x = torch.randn(xn, 16, device="cuda")
    y = torch.full((yn, 16), float("nan"), device="cuda")
    plan.gemm(d_payload, x, y, 16)
    assert plan.status() == 0
    assert (plan.launches() == 2) == fused
    if dist != "uniform":  # uniform patterns hold NaN / Inf / 1e38 weights: overflow order decides
        check(ws, x, y)
    plan.close()
