"""GPU: the batched device-resident plan API (include/xksv_cuda.h part 2) over
a payload of many blocks at arbitrary byte offsets, mixed codecs (serial,
parallel, raw) -- the layout of an .xksv archive's block region
(src/compile.cpp:459-470)."""
import hashlib

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


def build_archive(oracle, shapes, kinds, rng, codec_cycle=(1, 2, 0)):
    """Returns payload bytes, slab entries, expected raw output, per-slab sha."""
    payload = bytearray(b"\x00" * 3)  # blocks start at odd offsets
    out_off = 0
    entries, raws = [], []
    for i, ((rows, cols), kind) in enumerate(zip(shapes, kinds)):
        raw = words_for(kind, rows * cols, rng).astype("<u2").tobytes()
        codec = codec_cycle[i % len(codec_cycle)]
        if codec == 2 and rows > 16:
            codec = 1
        blob = (oracle.pack(raw, rows, cols) if codec == 1 else
                oracle.pack_parallel(raw, rows, cols) if codec == 2 else raw)
        entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=rows, cols=cols,
                            dst_offset=out_off, codec=codec))
        payload += blob
        payload += b"\x00" * (i % 5)
        raws.append(raw)
        out_off += len(raw)
    return bytes(payload), entries, raws


def test_plan_decode_mixed(xg):
    oracle = Oracle()
    rng = np.random.default_rng(5)
    shapes = [(16, 2048), (16, 5632), (1, 2048), (16, 4096), (7, 19), (16, 32), (16, 4097), (33, 35)] * 6
    kinds = ["normal002", "student3", "single", "normal1e4", "uniform", "three_exp"] * 8
    payload, entries, raws = build_archive(oracle, shapes, kinds, rng)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    total = sum(len(r) for r in raws)
    d_out = torch.full((total + 64,), 0xCD, dtype=torch.uint8, device="cuda")
    plan = xg.Plan(entries)
    plan.decode(d_payload, d_out)
    assert plan.status() == 0
    got = d_out.cpu().numpy().tobytes()
    for e, raw in zip(entries, raws):
        seg = got[e["dst_offset"]:e["dst_offset"] + len(raw)]
        assert hashlib.sha256(seg).digest() == hashlib.sha256(raw).digest(), e
    assert got[total:] == b"\xcd" * 64
    assert plan.launches() == 3
    plan.close()


def test_plan_reports_corrupt_slab(xg):
    oracle = Oracle()
    rng = np.random.default_rng(6)
    payload, entries, raws = build_archive(oracle, [(16, 512)] * 8, ["normal002"] * 8, rng,
                                           codec_cycle=(1, 2))
    bad = bytearray(payload)
    e = entries[3]
    bad[e["src_offset"] + 8] ^= 0x01  # bit_count of a parallel slab's header field / serial count
    d_payload = torch.frombuffer(bad, dtype=torch.uint8).cuda()
    d_out = torch.zeros(sum(len(r) for r in raws), dtype=torch.uint8, device="cuda")
    plan = xg.Plan(entries)
    plan.decode(d_payload, d_out)
    assert plan.status() == 1
    # the status word is cleared after being read
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    plan.decode(d_payload, d_out)
    assert plan.status() == 0


@pytest.mark.parametrize("batch", [1, 2, 5, 8, 16])
def test_plan_gemm_multi_tensor(xg, batch):
    """One plan covering two weight matrices with different x offsets."""
    oracle = Oracle()
    rng = np.random.default_rng(batch)
    mats = [(64, 2048), (48, 5632)]
    payload = bytearray(b"\x00" * 5)
    entries, ws = [], []
    xoff = 0
    yrow = 0
    for mi, (R, C) in enumerate(mats):
        w = words_for("normal002", R * C, rng).reshape(R, C)
        ws.append(w)
        for r0 in range(0, R, 16):
            raw = w[r0:r0 + 16].astype("<u2").tobytes()
            codec = [1, 2, 0][(r0 // 16 + mi) % 3]
            blob = oracle.pack(raw, 16, C) if codec == 1 else oracle.pack_parallel(raw, 16, C) if codec == 2 else raw
            entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=16, cols=C,
                                dst_offset=yrow + r0, x_offset=xoff, codec=codec))
            payload += blob
        xoff += C
        yrow += R
    x = torch.randn(xoff, batch, device="cuda")
    y = torch.full((yrow, batch), float("nan"), device="cuda")
    d_payload = torch.frombuffer(payload, dtype=torch.uint8).cuda()
    plan = xg.Plan(entries)
    plan.gemm(d_payload, x, y, batch)
    assert plan.status() == 0
    xo = yo = 0
    # from TC_MIN_BATCH the plan runs on the tensor cores with X rounded to BF16
    xr = x.to(torch.bfloat16).float() if batch >= TC_MIN_BATCH and plan.scratch_bytes() else x
    for (R, C), w in zip(mats, ws):
        ref = torch.from_numpy(bf16_to_f32(w)).cuda() @ xr[xo:xo + C]
        got = y[yo:yo + R]
        assert rel_l2(got.cpu(), ref.cpu()) < 1e-5
        xo += C
        yo += R
    plan.close()


def test_misaligned_outputs_are_refused(xg):
    """BF16 outputs need 2-byte and FP32 buffers 4-byte alignment: the calls
    return 1 without launching anything (a misaligned store would fault)."""
    import ctypes
    oracle = Oracle()
    rng = np.random.default_rng(21)
    raw = words_for("normal002", 16 * 256, rng).astype("<u2").tobytes()
    blob = oracle.pack(raw, 16, 256)
    lib = xg.load()
    d_out = torch.zeros(16 * 256 * 2 + 16, dtype=torch.uint8, device="cuda")
    host = ctypes.create_string_buffer(blob, len(blob))
    assert lib.xksv_cuda_decode(host, len(blob), 16, 256, d_out.data_ptr() + 1) == 1
    x = torch.zeros(256 + 4, device="cuda")
    y = torch.zeros(16 + 4, device="cuda")
    assert lib.xksv_cuda_gemv(host, len(blob), 16, 256, x.data_ptr() + 2, y.data_ptr()) == 1
    d_payload = torch.frombuffer(bytearray(blob), dtype=torch.uint8).cuda()
    odd = xg.Plan([dict(src_offset=0, src_size=len(blob), rows=16, cols=256, dst_offset=3, codec=1)])
    with pytest.raises(RuntimeError):
        odd.decode(d_payload, d_out)
    odd.close()
    ok = xg.Plan([dict(src_offset=0, src_size=len(blob), rows=16, cols=256, dst_offset=0, codec=1)])
    with pytest.raises(RuntimeError):
        ok.decode(d_payload, d_out.data_ptr() + 1, out_bytes=d_out.numel() - 1)
    ok.decode(d_payload, d_out)
    assert ok.status() == 0
    assert d_out[:len(raw)].cpu().numpy().tobytes() == raw
    ok.close()


@pytest.mark.parametrize("order", ["archive", "shuffled"])
def test_plan_decode_host_matches_device_decode(xg, order):
    """xksv_plan_decode_host: pinned host payload copied in pieces while the
    landed slabs decode (archive order), or one copy then the decode
    (shuffled table): both bit-exact; a payload_size short of the last slab
    is refused."""
    oracle = Oracle()
    rng = np.random.default_rng(9)
    shapes = [(16, 2048), (16, 5632), (1, 2048), (16, 4096), (7, 19), (16, 32), (16, 4097), (33, 35)] * 8
    kinds = ["normal002", "student3", "single", "normal1e4", "uniform", "three_exp"] * 11
    payload, entries, raws = build_archive(oracle, shapes, kinds, rng)
    if order == "shuffled":
        idx = rng.permutation(len(entries))
        entries, raws = [entries[i] for i in idx], [raws[i] for i in idx]
    h_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).pin_memory()
    d_payload = torch.empty(len(payload), dtype=torch.uint8, device="cuda")
    total = sum(len(r) for r in raws)
    d_out = torch.full((total + 64,), 0xCD, dtype=torch.uint8, device="cuda")
    plan = xg.Plan(entries)
    for _ in range(2):  # the second call reuses the plan's copy stream and events
        d_out.fill_(0xCD)
        plan.decode_host(h_payload.data_ptr(), len(payload), d_payload, d_out)
        assert plan.status() == 0
        got = d_out.cpu().numpy().tobytes()
        for e, raw in zip(entries, raws):
            assert got[e["dst_offset"]:e["dst_offset"] + len(raw)] == raw
    assert plan.launches() >= (4 if order == "archive" else 1)
    short = max(e["src_offset"] + e["src_size"] for e in entries) - 1
    assert xg.load().xksv_plan_decode_host(plan.handle, h_payload.data_ptr(), short, d_payload.data_ptr(),
                                           d_out.data_ptr(), d_out.numel(), None) == 1
    plan.close()
