"""GPU: xksv_cuda_decode_noalloc, the entry point for callers that cannot let
a library allocate device memory (a server that reserved the whole GPU for
its own allocator, or code that cannot take cudaMalloc's device-wide
synchronisation).  It must decode exactly what the plan API decodes, on two
calls in a row (the calls share one scratch array that keeps the previous
call's contents), byte for byte equal to the slabs' source words (what the
oracle's unpack returns for these slabs) and to the plan API's decode, and
refuse tables larger than its scratch array.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test."""
import numpy as np
import pytest

from helpers import words_for
from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _archive(seed):
    oracle = Oracle()
    rng = np.random.default_rng(seed)
    shapes = [(16, 2048), (16, 512), (1, 2048), (7, 19), (16, 4097), (33, 35)] * 5
    kinds = ["normal002", "student3", "single", "uniform", "normal1e4", "three_exp"] * 5
    payload = bytearray(b"\x00" * 7)
    entries, out, source = [], 0, bytearray()
    for i, ((rows, cols), kind) in enumerate(zip(shapes, kinds)):
        raw = words_for(kind, rows * cols, rng).astype("<u2").tobytes()
        codec = [1, 2, 0][i % 3]
        if codec == 2 and rows > 16:
            codec = 1
        blob = oracle.pack(raw, rows, cols) if codec == 1 else oracle.pack_parallel(raw, rows, cols) if codec == 2 else raw
        entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=rows, cols=cols,
                            dst_offset=out, codec=codec))
        payload += blob + b"\x00" * (i % 3)
        out += len(raw)
        source += raw
    return bytes(payload), entries, out, bytes(source)


def test_noalloc_matches_plan_decode_twice():
    import xksv_gpu
    assert torch.cuda.is_available()
    lib = xksv_gpu.load()
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (11, 12):  # two calls in a row, different slabs each time
        payload, entries, out_bytes, source = _archive(seed)
        d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
        want = torch.full((out_bytes,), 0x5A, dtype=torch.uint8, device="cuda")
        plan = xksv_gpu.Plan(entries)
        plan.decode(d_payload, want, stream)
        assert plan.status(stream) == 0
        plan.close()
        got = torch.full((out_bytes,), 0xA5, dtype=torch.uint8, device="cuda")
        table, n = xksv_gpu.slab_table(entries)
        assert lib.xksv_cuda_decode_noalloc(table, n, d_payload.data_ptr(), d_payload.numel(), got.data_ptr(),
                                            got.numel(), stream) == 0
        assert torch.equal(got, want)
        assert got.cpu().numpy().tobytes() == source


def test_noalloc_reports_bad_slab_and_limit():
    import xksv_gpu
    lib = xksv_gpu.load()
    stream = torch.cuda.current_stream().cuda_stream
    payload, entries, out_bytes, _ = _archive(13)
    bad = bytearray(payload)
    bad[entries[0]["src_offset"] + 8] ^= 1  # first slab (serial): bit count off by one
    d_payload = torch.frombuffer(bad, dtype=torch.uint8).cuda()
    out = torch.empty(out_bytes, dtype=torch.uint8, device="cuda")
    table, n = xksv_gpu.slab_table(entries)
    assert lib.xksv_cuda_decode_noalloc(table, n, d_payload.data_ptr(), d_payload.numel(), out.data_ptr(),
                                        out.numel(), stream) == 1
    # the status word is cleared by the next call
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    assert lib.xksv_cuda_decode_noalloc(table, n, d_payload.data_ptr(), d_payload.numel(), out.data_ptr(),
                                        out.numel(), stream) == 0
    big, nbig = xksv_gpu.slab_table([entries[0]] * (xksv_gpu.NOALLOC_MAX_SLABS + 1))
    assert lib.xksv_cuda_decode_noalloc(big, nbig, d_payload.data_ptr(), d_payload.numel(), out.data_ptr(),
                                        out.numel(), stream) == 2
