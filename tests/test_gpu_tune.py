"""Autotuner on the GPU: device-timed measurements of both codecs, and an
autotuned compile whose archive decodes bit-exact and records the profile."""
import json
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import xksv_compile as xc  # noqa: E402
import xksv_gpu  # noqa: E402
import xksv_runtime as rt  # noqa: E402
import xksv_tune  # noqa: E402
from golden.make_archives import checkpoint_tensors, write_safetensors  # noqa: E402
from helpers import bf16_bits  # noqa: E402


def test_select_measures_both_codecs():
    rng = np.random.default_rng(11)
    raw = bf16_bits(rng.standard_normal(16 * 4096) * 0.02).astype("<u2").tobytes()
    ser = xksv_gpu.host_pack(raw, 16, 4096, xksv_gpu.CODEC_TILE16)
    par = xksv_gpu.host_pack(raw, 16, 4096, xksv_gpu.CODEC_PARALLEL32)
    tuner = xksv_tune.GpuTuner(copies=64)
    codec, data = tuner.select(ser, par, raw, 16, 4096)
    (key, choice), = tuner.profile["choices"].items()
    assert key == f"16:4096:{len(ser) * 16 // len(raw)}"
    assert 0 < choice["serial_seconds"] < 1e-3 and 0 < choice["parallel_seconds"] < 1e-3
    assert codec == ("bf16-huffman-parallel32" if choice["prefer_parallel"] else "bf16-huffman-tile16")
    assert data == (par if choice["prefer_parallel"] else ser)
    # a resumed profile is reused without measuring again
    again = xksv_tune.GpuTuner(tuner.profile, copies=64)
    again.measure = None
    assert again.select(ser, par, raw, 16, 4096) == (codec, data)


def tune_tensors():
    """The misc fixture tensors plus a 32 x 8192 weight, wide enough that the
    parallel encoding is within 15 % of the serial one (a timed decision)."""
    rng = np.random.default_rng(12)
    wide = bf16_bits(rng.standard_normal(32 * 8192) * 0.02).astype("<u2").tobytes()
    return checkpoint_tensors("misc") + [("wide.weight", "BF16", [32, 8192], wide)]


@pytest.mark.parametrize("encoder", ["gpu", "host"])
def test_autotune_compile_decodes_bit_exact(tmp_path, encoder):
    src = tmp_path / "misc"
    src.mkdir()
    write_safetensors(src / "model.safetensors", tune_tensors())
    out = xc.compile_checkpoint(src, tmp_path / "a.xksv", "autotune", encoder=encoder, device="cuda:0")
    a = rt.ResidentArchive(out, "cuda:0")
    a.verify()
    assert a.index["codec_preference"] == "autotune" and a.index["tuning"]["choices"]
    dec = a.decode_all()
    for name, _, _, raw in tune_tensors():
        got = dec[name].contiguous().view(torch.uint8).reshape(-1).cpu().numpy().tobytes() if raw else b""
        assert got == raw, name
    codecs = {b["codec"] for t in a.tensors.values() for b in t["blocks"]}
    assert "raw" in codecs and codecs & {"bf16-huffman-tile16", "bf16-huffman-parallel32"}
