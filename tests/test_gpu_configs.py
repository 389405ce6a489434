"""GPU: the BASELINE configurations' shapes and value distributions at test
sizes, through the compiler's slab geometry (xksv_host_pack_tensor):
config 4 (Llama-3-70B slabs 16x8192 and 16x28672, N(0, 0.015)): decode,
indexed GEMV and the batch-8/16 tensor-core GEMM; config 5 (Student-t(3)*0.02,
N(0, 1e-4) and uniform 16-bit patterns that become raw slabs): decode of a
mixed archive in both codecs, checked bit for bit and by device SHA-256."""
import hashlib

import numpy as np
import pytest

from helpers import TC_MIN_BATCH, bf16_bits, bf16_to_f32, rel_l2, words_for

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def xg():
    import xksv_gpu
    assert torch.cuda.is_available()
    xksv_gpu.load()
    return xksv_gpu


def compile_tensors(xg, mats, codec):
    """mats: list of uint16 [R, C] arrays -> payload, decode entries, GEMV entries."""
    parts, dec, gemv = [], [], []
    src = dst = row = xoff = 0
    for w in mats:
        R, C = w.shape
        pay, slabs = xg.host_pack_tensor(w.ctypes.data, w.nbytes, R, C, codec, dst_base=dst)
        for s in slabs:
            s["src_offset"] += src
            dec.append(dict(s))
            g = dict(s)
            g["dst_offset"] = row + (s["dst_offset"] - dst) // (2 * C)
            g["x_offset"] = xoff
            gemv.append(g)
        parts.append(pay)
        src += pay.nbytes
        dst += w.nbytes
        row += R
        xoff += C
    return np.concatenate(parts), dec, gemv, dst, row, xoff


@pytest.mark.parametrize("codec", [1, 2])
def test_config4_slabs(xg, codec):
    rng = np.random.default_rng(3)
    mats = [bf16_bits(rng.standard_normal((64, 8192)) * 0.015).astype("<u2"),
            bf16_bits(rng.standard_normal((32, 28672)) * 0.015).astype("<u2")]
    payload, dec, gemv, nbytes, nrows, ncols = compile_tensors(xg, mats, codec)
    assert all(s["codec"] == codec for s in dec)  # N(0, 0.015) always compresses
    d_payload = torch.from_numpy(payload).cuda()
    out = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    plan = xg.Plan(dec)
    plan.decode(d_payload, out)
    assert plan.status() == 0
    assert out.cpu().numpy().tobytes() == b"".join(m.tobytes() for m in mats)
    plan.close()
    gp = xg.Plan(gemv)
    if codec == 1:
        assert gp.index(d_payload) == 0
    W = [torch.from_numpy(bf16_to_f32(m)).cuda() for m in mats]
    for batch in (1, 4, 8, 16):
        x = torch.randn(ncols, batch, device="cuda")
        y = torch.full((nrows, batch), float("nan"), device="cuda")
        gp.gemm(d_payload, x, y, batch)
        assert gp.status() == 0
        xr = x.to(torch.bfloat16).float() if batch >= TC_MIN_BATCH and gp.scratch_bytes() else x
        ro = co = 0
        for w in W:
            ref = w @ xr[co:co + w.shape[1]]
            assert rel_l2(y[ro:ro + w.shape[0]].cpu(), ref.cpu()) < 1e-5, (batch, w.shape)
            ro += w.shape[0]
            co += w.shape[1]
    gp.close()


@pytest.mark.parametrize("codec", [1, 2])
def test_config5_mix(xg, codec):
    rng = np.random.default_rng(4)
    mats = [words_for(k, 96 * 2048, rng).astype("<u2").reshape(96, 2048)
            for k in ("student3", "student3", "normal1e4", "uniform")]
    payload, dec, _, nbytes, _, _ = compile_tensors(xg, mats, codec)
    kinds = [s["codec"] for s in dec]
    assert 0 in kinds and codec in kinds  # raw fallback for the uniform tensor only
    d_payload = torch.from_numpy(payload).cuda()
    out = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    plan = xg.Plan(dec)
    plan.decode(d_payload, out)
    dig = torch.empty(32 * len(dec), dtype=torch.uint8, device="cuda")
    plan.sha256(out, dig)
    assert plan.status() == 0
    src = b"".join(m.tobytes() for m in mats)
    assert out.cpu().numpy().tobytes() == src
    got = dig.cpu().numpy().tobytes()
    for i, s in enumerate(dec):
        n = s["src_size"] if s["codec"] == 0 else s["rows"] * s["cols"] * 2
        assert got[32 * i:32 * i + 32] == hashlib.sha256(src[s["dst_offset"]:s["dst_offset"] + n]).digest()
    plan.close()
