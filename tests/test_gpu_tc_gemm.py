"""GPU: the batch >= 16 fused GEMM through the tensor cores (decode into
BF16 row groups, then tcgen05.mma kind::f16 with FP32 accumulation in TMEM).
X is rounded to BF16 for the tensor cores, so results are compared with an
FP32 matmul of the decoded weights twice: against BF16-rounded X (tight,
1e-5) and against the FP32 X the reference multiplies (the 1e-2 relative L2
bound of the task)."""
import numpy as np
import pytest

from helpers import bf16_to_f32, rel_l2, words_for
from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def xg():
    import xksv_gpu
    assert torch.cuda.is_available()
    xksv_gpu.load()
    return xksv_gpu


def archive(oracle, mats, rng, codecs=(1, 2, 0), lead=5, row_step=16):
    payload = bytearray(b"\x00" * lead)
    entries, ws = [], []
    xoff = yrow = 0
    for mi, (R, C) in enumerate(mats):
        w = words_for("normal002", R * C, rng).reshape(R, C)
        ws.append(w)
        for k, r0 in enumerate(range(0, R, row_step)):
            rows = min(row_step, R - r0)
            raw = w[r0:r0 + rows].astype("<u2").tobytes()
            codec = codecs[(k + mi) % len(codecs)]
            if codec == 2 and rows > 16:
                codec = 1
            blob = (oracle.pack(raw, rows, C) if codec == 1 else
                    oracle.pack_parallel(raw, rows, C) if codec == 2 else raw)
            entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=rows, cols=C,
                                dst_offset=yrow + r0, x_offset=xoff, codec=codec))
            payload += blob
        xoff += C
        yrow += R
    return bytes(payload), entries, ws, xoff, yrow


def check(ws, x, y):
    xo = yo = 0
    xb = x.to(torch.bfloat16).float()
    for w in ws:
        R, C = w.shape
        W = torch.from_numpy(bf16_to_f32(w)).cuda()
        got = y[yo:yo + R].cpu()
        assert rel_l2(got, (W @ xb[xo:xo + C]).cpu()) < 1e-5, (R, C)
        assert rel_l2(got, (W @ x[xo:xo + C]).cpu()) < 1e-2, (R, C)
        xo += C
        yo += R


@pytest.mark.parametrize("batch", [16, 17, 32, 64, 100, 256, 300])
def test_tc_gemm_mixed_codecs(xg, batch):
    oracle = Oracle()
    rng = np.random.default_rng(batch)
    mats = [(256, 512), (48, 2048), (16, 5632), (39, 1024)]  # 7-row tail slab in the last
    payload, entries, ws, xn, yn = archive(oracle, mats, rng)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(xn, batch, device="cuda")
    plan = xg.Plan(entries)
    for _ in range(2):
        y = torch.full((yn, batch), float("nan"), device="cuda")
        plan.gemm(d_payload, x, y, batch)
        assert plan.status() == 0
        check(ws, x, y)
    plan.close()


def test_tc_gemm_llama_shapes(xg):
    """Row-sharded 16-row slabs of 4096-wide and 14336-wide weights (serial
    codec, the compiler's Llama-3-8B slabs) at batch 16."""
    oracle = Oracle()
    rng = np.random.default_rng(3)
    mats = [(256, 4096), (64, 14336)]
    payload, entries, ws, xn, yn = archive(oracle, mats, rng, codecs=(1,))
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(xn, 16, device="cuda")
    y = torch.empty(yn, 16, device="cuda")
    plan = xg.Plan(entries)
    plan.gemm(d_payload, x, y, 16)
    assert plan.status() == 0
    check(ws, x, y)
    plan.close()


def test_tc_gemm_reports_corrupt_slab(xg):
    oracle = Oracle()
    rng = np.random.default_rng(9)
    payload, entries, ws, xn, yn = archive(oracle, [(64, 1024)], rng, codecs=(1,))
    bad = bytearray(payload)
    o = entries[1]["src_offset"]
    bad[o + 16:o + 20] = b"\x01\x01\x01\x01"  # oversubscribed code lengths
    d_bad = torch.frombuffer(bad, dtype=torch.uint8).cuda()
    x = torch.randn(xn, 16, device="cuda")
    y = torch.empty(yn, 16, device="cuda")
    plan = xg.Plan(entries)
    plan.gemm(d_bad, x, y, 16)
    assert plan.status() == 1
    plan.close()


@pytest.mark.parametrize("batch", [8, 16])
def test_tc_gemm_shared_scratch_and_x_base(xg, batch):
    """Two plans over disjoint parts of one X (the second's lowest x_offset is
    not 0, so its X^T covers only its own columns) share one caller-owned
    scratch; results match an FP32 matmul.  A too-small scratch is refused."""
    oracle = Oracle()
    rng = np.random.default_rng(40 + batch)
    mats = [(64, 512), (48, 1024), (32, 2048)]
    payload, entries, ws, xn, yn = archive(oracle, mats, rng, codecs=(1, 2, 0))
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(xn, batch, device="cuda")
    first = [e for e in entries if e["x_offset"] == 0]
    rest = [e for e in entries if e["x_offset"] > 0]
    p1, p2 = xg.Plan(first), xg.Plan(rest)
    need = max(p1.scratch_bytes(), p2.scratch_bytes())
    assert need > 0
    with pytest.raises(ValueError):
        p2.set_scratch(torch.empty(16, dtype=torch.uint8, device="cuda").data_ptr(), 16)
    scratch = torch.empty(need, dtype=torch.uint8, device="cuda")
    for p in (p1, p2):
        p.set_scratch(scratch.data_ptr(), need)
    for _ in range(2):
        y = torch.full((yn, batch), float("nan"), device="cuda")
        p1.gemm(d_payload, x, y, batch)
        p2.gemm(d_payload, x, y, batch)
        assert p1.status() == 0 and p2.status() == 0
        check(ws, x, y)
    p1.close()
    p2.close()
