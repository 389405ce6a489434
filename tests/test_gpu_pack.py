"""GPU encoder (xksv_cuda_pack_tensor): byte-identical payload and slab table
to the host encoder xksv_host_pack_tensor (itself pinned to the reference's
xksv_pack / xksv_pack_parallel by test_pack.py), for both codecs, partial
slabs, 1 MiB single-row slabs, raw fallback, single-symbol blocks; and a
round trip through the plan decode."""
import numpy as np
import pytest

from helpers import words_for

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def xg():
    import xksv_gpu
    assert torch.cuda.is_available()
    xksv_gpu.load()
    return xksv_gpu


CASES = [((16, 4096), "normal002"), ((40, 1000), "student3"), ((7, 19), "normal1e4"),
         ((1, 2048), "single"), ((300, 2048), "normal002"), ((2, 524288), "normal002"),
         ((33, 512), "uniform"), ((64, 256), "three_exp"), ((1, 1), "normal002"), ((17, 4112), "student3")]


@pytest.mark.parametrize("codec", [1, 2])
@pytest.mark.parametrize("shape,kind", CASES)
def test_gpu_encoder_matches_host(xg, codec, shape, kind):
    rows, cols = shape
    rng = np.random.default_rng(rows * 7 + cols)
    w = words_for(kind, rows * cols, rng).astype("<u2").reshape(rows, cols)
    host_pay, host_slabs = xg.host_pack_tensor(w.ctypes.data, w.nbytes, rows, cols, codec, dst_base=64)
    d = torch.from_numpy(w.view(np.int16).copy()).cuda()
    dptr, n, slabs = xg.cuda_pack_tensor(d.data_ptr(), rows, cols, codec, dst_base=64)
    try:
        assert slabs == host_slabs
        assert n == len(host_pay)
        # the device payload, copied out with a one-raw-slab plan (a byte copy)
        buf = torch.empty(n, dtype=torch.uint8, device="cuda")
        cp = xg.Plan([dict(src_offset=0, src_size=n, rows=1, cols=1, dst_offset=0, codec=0)])
        cp.decode(dptr, buf, payload_bytes=n)
        assert cp.status() == 0
        cp.close()
        got = buf.cpu().numpy()
        assert np.array_equal(got, host_pay)
        # round trip: decode the GPU payload with a plan
        out = torch.empty(rows * cols * 2 + 64, dtype=torch.uint8, device="cuda")
        pl = xg.Plan(slabs)
        pl.decode(dptr, out, payload_bytes=n)
        assert pl.status() == 0
        assert out[64:].cpu().numpy().tobytes() == w.tobytes()
        pl.close()
    finally:
        xg.free_device(dptr)
