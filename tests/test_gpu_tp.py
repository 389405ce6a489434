"""GPU, 2+ devices: xksv_tp_gemm (each rank's fused plan GEMM on its row
shard, then one NCCL all-gather) against an FP32 matmul of the weights.
Skipped on single-GPU machines."""
import json
import socket

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_tp_gemm_two_gpus(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import tp_worker
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "res.json"
    mp.start_processes(tp_worker.gpu_tp_check, args=(2, port, str(out)), nprocs=2,
                       start_method="spawn", join=True)
    res = json.loads(out.read_text())
    assert res["rows"] == sum(r for r, _ in tp_worker.MATS)
    assert res["err"] < 1e-5


def test_tp_fused_gemm_two_gpus(tmp_path):
    """The fused variant: peer stores from the GEMV epilogue + bounded flag
    wait, four calls alternating the gathered buffers."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import tp_worker
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "res.json"
    mp.start_processes(tp_worker.gpu_tp_fused_check, args=(2, port, str(out)), nprocs=2,
                       start_method="spawn", join=True)
    res = json.loads(out.read_text())
    assert res["rows"] == sum(r for r, _ in tp_worker.MATS)
    assert res["err"] < 1e-5
