"""Rank bodies for the tensor-parallel tests (started with the `spawn` method).

Each rank shards the same seeded row-sharded weights (16-row slabs of several
matrices in one plan) with xksv_gpu.shard_entries, computes its shard of
Y = W X, all-gathers the shards and maps them back to full rows with
xksv_gpu.gathered_to_full; rank 0 writes the max relative error to a file.
"""
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "xks-vectorforge_b200"))
sys.path.insert(0, str(ROOT / "tests"))

MATS = [(48, 512), (96, 256), (16, 1024)]  # (rows, cols); 3, 6 and 1 slabs


def make_archive(pack):
    """Payload bytes, GEMV entries (dst_offset = first row in the full Y,
    x_offset = first column in X, plus their tensor's first row and row
    count), weights per matrix, X length and Y length."""
    import numpy as np
    from helpers import words_for
    rng = np.random.default_rng(77)
    payload = bytearray(b"\x00" * 7)
    entries, ws = [], []
    xoff = yrow = 0
    for R, C in MATS:
        w = words_for("normal002", R * C, rng).reshape(R, C)
        ws.append(w)
        for r0 in range(0, R, 16):
            raw = w[r0:r0 + 16].astype("<u2").tobytes()
            blob = pack(raw, 16, C)
            entries.append(dict(src_offset=len(payload), src_size=len(blob), rows=16, cols=C,
                                dst_offset=yrow + r0, x_offset=xoff, codec=1,
                                tensor_row0=yrow, tensor_rows=R))
            payload += blob
        xoff += C
        yrow += R
    return bytes(payload), entries, ws, xoff, yrow


def rows_of(e):
    return e["tensor_row0"], e["tensor_rows"]


def init_group(rank, world, port, backend):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    return dist


def cpu_shard_check(rank, world, port, out):
    """gloo on CPU: sharding and all-gather layout with a numpy matmul per shard."""
    import numpy as np
    import torch
    import xksv_gpu
    from helpers import bf16_to_f32
    from oracle.oracle import Oracle
    dist = init_group(rank, world, port, "gloo")
    oracle = Oracle()
    payload, entries, ws, xn, yn = make_archive(oracle.pack)
    x = np.random.default_rng(5).standard_normal(xn).astype(np.float32)
    local, rows_shard, runs = xksv_gpu.shard_entries(entries, world, rank, rows_of)
    # every rank pads its shard to the largest shard so all-gather sizes agree
    sizes = [None] * world
    dist.all_gather_object(sizes, rows_shard)
    pad = max(sizes)
    y = np.zeros(pad, np.float32)
    for e in local:
        blob = payload[e["src_offset"]:e["src_offset"] + e["src_size"]]
        raw = oracle.unpack(blob, e["rows"], e["cols"])
        W = bf16_to_f32(np.frombuffer(raw, "<u2").reshape(e["rows"], e["cols"]))
        y[e["dst_offset"]:e["dst_offset"] + 16] = W @ x[e["x_offset"]:e["x_offset"] + e["cols"]]
    parts = [torch.zeros(pad) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(y))
    gathered = torch.cat(parts).numpy()
    all_runs = [None] * world
    dist.all_gather_object(all_runs, runs)
    idx = xksv_gpu.gathered_to_full(gathered, world, all_runs, pad)
    full = gathered[idx]
    ref = np.concatenate([bf16_to_f32(w) @ x[o:o + w.shape[1]]
                          for w, o in zip(ws, np.cumsum([0] + [w.shape[1] for w in ws])[:-1])])
    err = float(np.abs(full - ref).max() / np.abs(ref).max())
    if rank == 0:
        Path(out).write_text(json.dumps(dict(err=err, rows=int(len(full)), shards=sizes)))
    dist.barrier()
    dist.destroy_process_group()


def gpu_tp_check(rank, world, port, out):
    """One GPU per rank: xksv_tp_gemm (plan GEMV on the rank's slabs + NCCL
    all-gather) against an FP32 matmul of the decoded weights."""
    import numpy as np
    import torch
    import xksv_gpu
    from helpers import bf16_to_f32
    torch.cuda.set_device(rank)
    dist = init_group(rank, world, port, "gloo")
    lib = xksv_gpu.load()
    payload, entries, ws, xn, yn = make_archive(
        lambda raw, r, c: xksv_gpu.host_pack(raw, r, c, 1, lib))
    local, rows_shard, runs = xksv_gpu.shard_entries(entries, world, rank, rows_of)
    sizes = [None] * world
    dist.all_gather_object(sizes, rows_shard)
    pad = max(sizes)
    comm = xksv_gpu.TPComm(rank, world, lib)
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    batch = 3
    x = torch.from_numpy(np.random.default_rng(5).standard_normal((xn, batch)).astype(np.float32)).cuda()
    plan = xksv_gpu.Plan(local, lib)
    assert plan.index(d_payload) == 0
    y_shard = torch.zeros(pad, batch, device="cuda")
    y_full = torch.full((world * pad, batch), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    comm.gemm(plan, d_payload, x, y_shard, pad, y_full,
              batch, stream)
    assert plan.status(stream) == 0
    torch.cuda.synchronize()
    all_runs = [None] * world
    dist.all_gather_object(all_runs, runs)
    idx = torch.from_numpy(xksv_gpu.gathered_to_full(None, world, all_runs, pad)).cuda()
    full = y_full[idx].cpu().numpy()
    xs = x.cpu().numpy()
    ref = np.concatenate([bf16_to_f32(w) @ xs[o:o + w.shape[1]]
                          for w, o in zip(ws, np.cumsum([0] + [w.shape[1] for w in ws])[:-1])])
    err = float(np.linalg.norm(full - ref) / np.linalg.norm(ref))
    plan.close()
    comm.close()
    if rank == 0:
        Path(out).write_text(json.dumps(dict(err=err, rows=int(len(full)), shards=sizes)))
    dist.barrier()
    dist.destroy_process_group()


def gpu_tp_fused_check(rank, world, port, out):
    """One GPU per rank: xksv_tp_fused_gemm (indexed GEMV whose epilogue
    stores each row into every rank's gathered buffer over NVLink, then a
    bounded flag wait), three successive calls with different X and batch,
    each against an FP32 matmul of the weights."""
    import numpy as np
    import torch
    import xksv_gpu
    from helpers import bf16_to_f32
    torch.cuda.set_device(rank)
    dist = init_group(rank, world, port, "gloo")
    lib = xksv_gpu.load()
    payload, entries, ws, xn, yn = make_archive(
        lambda raw, r, c: xksv_gpu.host_pack(raw, r, c, 1, lib))
    local, rows_shard, runs = xksv_gpu.shard_entries(entries, world, rank, rows_of)
    sizes = [None] * world
    dist.all_gather_object(sizes, rows_shard)
    pad = max(sizes)
    all_runs = [None] * world
    dist.all_gather_object(all_runs, runs)
    idx = torch.from_numpy(xksv_gpu.gathered_to_full(None, world, all_runs, pad)).cuda()
    d_payload = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    plan = xksv_gpu.Plan(local, lib)
    assert plan.index(d_payload) == 0
    fused = xksv_gpu.TPFused(rank, world, pad, 4, lib)
    stream = torch.cuda.current_stream().cuda_stream
    errs = []
    for call, batch in enumerate((1, 3, 4, 2)):
        xs = np.random.default_rng(call).standard_normal((xn, batch)).astype(np.float32)
        x = torch.from_numpy(xs).cuda()
        y_full = torch.full((world * pad, batch), float("nan"), device="cuda")
        fused.gemm(plan, d_payload, x, pad, batch, stream, y_full)
        assert plan.status(stream) == 0
        full = y_full[idx].cpu().numpy()
        ref = np.concatenate([bf16_to_f32(w) @ xs[o:o + w.shape[1]]
                              for w, o in zip(ws, np.cumsum([0] + [w.shape[1] for w in ws])[:-1])])
        errs.append(float(np.linalg.norm(full - ref) / np.linalg.norm(ref)))
    torch.cuda.synchronize()
    dist.barrier()  # no rank frees its IPC-shared buffers while another may still use them
    plan.close()
    fused.close()
    if rank == 0:
        Path(out).write_text(json.dumps(dict(err=max(errs), rows=int(len(idx)), shards=sizes)))
    dist.barrier()
    dist.destroy_process_group()
