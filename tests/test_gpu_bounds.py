"""GPU: every plan call, the tensor-parallel calls and the no-allocation decode
refuse a slab that lies outside the buffers they are given -- return 1 (or
raise in the binding) before launching anything, so the output keeps its
sentinel bytes and the plan's status word stays clear -- and the fused
tensor-parallel GEMV's bounded flag wait ends with an error status when a
peer's flag never advances."""
import ctypes
import subprocess
import sys
import textwrap
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parents[1]


def _archive(lib, seed=21):
    """A mixed archive: 3 serial + 3 parallel 16x256 slabs and one raw slab,
    at odd byte offsets; entries decode back to back (dst = byte offsets)."""
    import xksv_gpu
    from helpers import words_for
    rng = np.random.default_rng(seed)
    payload = bytearray(b"\x00" * 5)
    entries, raws, dst = [], [], 0
    for k in range(7):
        w = words_for("normal002", 16 * 256, rng).astype("<u2")
        raw = w.tobytes()
        codec = (1, 1, 1, 2, 2, 2, 0)[k]
        blob = raw if codec == 0 else xksv_gpu.host_pack(raw, 16, 256, codec, lib)
        entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=16, cols=256,
                            dst_offset=dst, x_offset=0, codec=codec))
        payload += blob + b"\x01" * 3
        raws.append(raw)
        dst += len(raw)
    need_pay = max(e["src_offset"] + e["src_size"] for e in entries)
    return bytes(payload[:need_pay]), entries, raws, dst


def _gemm_entries(entries):
    """The same slabs as one GEMV over X [256]: slab k computes rows 16k.."""
    return [dict(e, dst_offset=16 * k) for k, e in enumerate(entries)]


def test_plan_calls_refuse_buffers_smaller_than_the_table():
    import xksv_gpu
    lib = xksv_gpu.load()
    payload, entries, raws, out_bytes = _archive(lib)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    out = torch.full((out_bytes,), 0xCD, dtype=torch.uint8, device="cuda")
    plan = xksv_gpu.Plan(entries)
    stream = torch.cuda.current_stream().cuda_stream
    # one byte short of the payload or of the output: refused, nothing written
    with pytest.raises(RuntimeError):
        plan.decode(d_payload, out, stream, payload_bytes=len(payload) - 1)
    with pytest.raises(RuntimeError):
        plan.decode(d_payload, out, stream, out_bytes=out_bytes - 1)
    h_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).pin_memory()
    with pytest.raises(RuntimeError):
        plan.decode_host(h_payload.data_ptr(), len(payload), d_payload, out, stream, out_bytes=out_bytes - 1)
    assert lib.xksv_plan_decode_host(plan.handle, h_payload.data_ptr(), len(payload) - 1, d_payload.data_ptr(),
                                     out.data_ptr(), out_bytes, None) == 1
    dig = torch.zeros(32 * len(entries), dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError):
        plan.sha256(out, dig, stream, out_bytes=out_bytes - 1)
    torch.cuda.synchronize()
    assert bool((out == 0xCD).all())
    assert plan.status(stream) == 0
    # the exact sizes decode every slab
    plan.decode(d_payload, out, stream)
    assert plan.status(stream) == 0
    assert out.cpu().numpy().tobytes() == b"".join(raws)
    plan.close()

    # GEMV: payload, X rows and Y rows each one short are refused
    gplan = xksv_gpu.Plan(_gemm_entries(entries))
    x = torch.randn(256, device="cuda")
    y = torch.full((16 * len(entries),), float("nan"), device="cuda")
    assert gplan.index(d_payload, stream, payload_bytes=len(payload) - 1) == 1
    for kw in (dict(payload_bytes=len(payload) - 1), dict(x_rows=255), dict(y_rows=16 * len(entries) - 1)):
        with pytest.raises(RuntimeError):
            gplan.gemm(d_payload, x, y, 1, stream, **kw)
    torch.cuda.synchronize()
    assert bool(torch.isnan(y).all())
    assert gplan.status(stream) == 0
    gplan.gemm(d_payload, x, y, 1, stream)
    assert gplan.status(stream) == 0
    ws = [np.frombuffer(r, dtype="<u2").reshape(16, 256) for r in raws]
    from helpers import bf16_to_f32
    ref = np.concatenate([bf16_to_f32(w) @ x.cpu().numpy() for w in ws])
    got = y.cpu().numpy()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5
    gplan.close()


def test_plan_create_refuses_extents_past_64_bits():
    import xksv_gpu
    big = (1 << 64) - 8
    for e in (dict(src_offset=big, src_size=16, rows=16, cols=256, dst_offset=0, codec=1),
              dict(src_offset=0, src_size=4096, rows=16, cols=256, dst_offset=big, codec=1),
              dict(src_offset=0, src_size=4096, rows=1 << 40, cols=1 << 40, dst_offset=0, codec=1)):
        with pytest.raises(ValueError):
            xksv_gpu.Plan([e])


def test_noalloc_refuses_out_of_range_and_overflowing_tables():
    import xksv_gpu
    lib = xksv_gpu.load()
    payload, entries, raws, out_bytes = _archive(lib, seed=22)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    out = torch.full((out_bytes,), 0xCD, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def call(tab, pay=len(payload), n_out=out_bytes):
        table, n = xksv_gpu.slab_table(tab)
        return lib.xksv_cuda_decode_noalloc(table, n, d_payload.data_ptr(), pay, out.data_ptr(), n_out, stream)

    assert call(entries, pay=len(payload) - 1) == 1
    assert call(entries, n_out=out_bytes - 1) == 1
    wrap = dict(entries[0], src_offset=(1 << 64) - 8, src_size=16)
    assert call([wrap] + entries[1:]) == 1
    past = dict(entries[3], dst_offset=(1 << 64) - 2)
    assert call(entries[:3] + [past] + entries[4:]) == 1
    torch.cuda.synchronize()
    assert bool((out == 0xCD).all())
    assert call(entries) == 0
    assert out.cpu().numpy().tobytes() == b"".join(raws)


def _fused_plan(lib):
    """Three 16-row serial slabs over X [512] (48 rows) with a tile index."""
    import xksv_gpu
    from helpers import words_for
    rng = np.random.default_rng(31)
    payload, entries, ws = bytearray(b"\x00" * 3), [], []
    for k in range(3):
        w = words_for("normal002", 16 * 512, rng).astype("<u2").reshape(16, 512)
        blob = xksv_gpu.host_pack(w.tobytes(), 16, 512, 1, lib)
        entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=16, cols=512,
                            dst_offset=16 * k, x_offset=0, codec=1))
        payload += blob
        ws.append(w)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    plan = xksv_gpu.Plan(entries, lib)
    assert plan.index(d_payload) == 0
    return plan, d_payload, ws


def _fused_ctx(lib, world, rank, rows):
    ctx = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    assert lib.xksv_tp_fused_create(world, rank, rows, 1, ctypes.byref(ctx), h) == 0
    return ctx, h.raw


def test_tp_fused_refuses_a_plan_past_its_rows():
    """A plan writing rows at or past rows_shard would store into the next
    rank's block or past the gathered buffer onto the flags: refused."""
    import xksv_gpu
    from helpers import bf16_to_f32
    lib = xksv_gpu.load()
    plan, d_payload, ws = _fused_plan(lib)
    ctx, h = _fused_ctx(lib, 1, 0, 64)
    assert lib.xksv_tp_fused_open(ctx, ctypes.create_string_buffer(h, 64)) == 0
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.randn(512, device="cuda")
    y = torch.full((64,), float("nan"), device="cuda")
    g = ctypes.c_void_p()
    args = lambda rows: (ctx, plan.handle, d_payload.data_ptr(), d_payload.numel(), x.data_ptr(), 512, rows, 1,
                         y.data_ptr(), ctypes.byref(g), stream)
    assert lib.xksv_tp_fused_gemm(*args(47)) == 1
    assert lib.xksv_tp_fused_gemm(ctx, plan.handle, d_payload.data_ptr(), d_payload.numel(), x.data_ptr(), 511,
                                  48, 1, y.data_ptr(), ctypes.byref(g), stream) == 1
    torch.cuda.synchronize()
    assert bool(torch.isnan(y).all())
    assert lib.xksv_tp_fused_gemm(*args(48)) == 0
    assert plan.status(stream) == 0
    ref = np.concatenate([bf16_to_f32(w) @ x.cpu().numpy() for w in ws])
    got = y[:48].cpu().numpy()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5
    lib.xksv_tp_fused_destroy(ctx)
    plan.close()


_IDLE_PEER = textwrap.dedent("""
    import ctypes, sys
    sys.path.insert(0, {pkg!r})
    import xksv_gpu
    lib = xksv_gpu.load()
    ctx = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    assert lib.xksv_tp_fused_create(2, 1, 64, 1, ctypes.byref(ctx), h) == 0
    sys.stdout.write(h.raw.hex() + "\\n")
    sys.stdout.flush()
    sys.stdin.readline()          # the test is done with this rank's buffers
    lib.xksv_tp_fused_destroy(ctx)
""")


def test_tp_fused_wait_times_out_when_a_peer_never_arrives():
    """Rank 1 lives in a child process that creates its context, hands over
    its IPC handle and then launches nothing, so its flag never reaches the
    call: rank 0's bounded wait (about a second) gives up, sets the error bit
    in the plan's status word, and the GPU stays usable."""
    import xksv_gpu
    lib = xksv_gpu.load()
    child = subprocess.Popen([sys.executable, "-c", _IDLE_PEER.format(pkg=str(ROOT / "xks-vectorforge_b200"))],
                             stdin=subprocess.PIPE, stdout=subprocess.PIPE, text=True)
    try:
        h1 = bytes.fromhex(child.stdout.readline().strip())
        assert len(h1) == 64
        plan, d_payload, ws = _fused_plan(lib)
        ctx, h0 = _fused_ctx(lib, 2, 0, 64)
        assert lib.xksv_tp_fused_open(ctx, ctypes.create_string_buffer(h0 + h1, 128)) == 0
        stream = torch.cuda.current_stream().cuda_stream
        x = torch.randn(512, device="cuda")
        g = ctypes.c_void_p()
        t0 = time.perf_counter()
        assert lib.xksv_tp_fused_gemm(ctx, plan.handle, d_payload.data_ptr(), d_payload.numel(), x.data_ptr(),
                                      512, 64, 1, None, ctypes.byref(g), stream) == 0
        assert plan.status(stream) == 1  # the wait ran out
        dt = time.perf_counter() - t0
        assert 0.2 < dt < 10.0, dt
        # the context and the device are still usable: a plain decode works
        payload, entries, raws, out_bytes = _archive(lib, seed=23)
        dp = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
        out = torch.empty(out_bytes, dtype=torch.uint8, device="cuda")
        p2 = xksv_gpu.Plan(entries)
        p2.decode(dp, out, stream)
        assert p2.status(stream) == 0
        assert out.cpu().numpy().tobytes() == b"".join(raws)
        p2.close()
        torch.cuda.synchronize()
        lib.xksv_tp_fused_destroy(ctx)  # closes the mapping of rank 1's buffers first
        plan.close()
    finally:
        child.stdin.write("\n")
        child.stdin.flush()
        child.wait(timeout=60)
