"""Tensor-parallel host logic (no GPU): row sharding in whole 16-row slabs and
the all-gather layout, run as world_size-2 gloo ranks on the CPU with a numpy
matmul standing in for each rank's fused GEMV."""
import json
import socket

import pytest

import xksv_gpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("rows,world", [(16, 1), (48, 2), (96, 4), (16, 2), (1792, 8), (28672, 8),
                                        (33, 2), (0, 3)])
def test_shard_rows_partition(rows, world):
    parts = [xksv_gpu.shard_rows(rows, world, g) for g in range(world)]
    assert parts[0][0] == 0 and parts[-1][1] == rows
    for (a0, a1), (b0, b1) in zip(parts, parts[1:]):
        assert a1 == b0
    for r0, r1 in parts:
        assert r0 % 16 == 0 and r1 >= r0
        assert r1 == rows or r1 % 16 == 0
    slabs = [(r1 - r0 + 15) // 16 for r0, r1 in parts]
    assert max(slabs) - min(slabs) <= 1


def test_shard_entries_rebases_rows():
    entries = []
    for t0, R in ((0, 48), (48, 32)):
        for r0 in range(0, R, 16):
            entries.append(dict(dst_offset=t0 + r0, tensor_row0=t0, tensor_rows=R))
    rows_of = lambda e: (e["tensor_row0"], e["tensor_rows"])
    seen = []
    for g in range(2):
        local, n, runs = xksv_gpu.shard_entries(entries, 2, g, rows_of)
        assert n == sum(r[2] for r in runs)
        assert sorted(e["dst_offset"] for e in local) == list(range(0, n, 16))
        for full0, local0, k in runs:
            seen += list(range(full0, full0 + k))
    assert sorted(seen) == list(range(80))


def test_tp_two_gloo_ranks(tmp_path):
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp
    import tp_worker
    out = tmp_path / "res.json"
    mp.start_processes(tp_worker.cpu_shard_check, args=(2, free_port(), str(out)), nprocs=2,
                       start_method="spawn", join=True)
    res = json.loads(out.read_text())
    assert res["rows"] == sum(r for r, _ in tp_worker.MATS)
    assert res["err"] < 1e-5
