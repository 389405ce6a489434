"""Autotuner decision rules (no GPU): the size rules of python/tune.py:22-24,
the grouping key and the cached profile, with the timing replaced by a stub."""
import pytest

import xksv_tune


def test_size_rules():
    raw = bytes(100)
    assert xksv_tune.size_rule(bytes(100), bytes(120), raw) == ("raw", raw)
    assert xksv_tune.size_rule(bytes(100), bytes(90), raw)[0] == "bf16-huffman-parallel32"
    assert xksv_tune.size_rule(bytes(80), bytes(100), raw)[0] == "bf16-huffman-tile16"
    # parallel more than 15 % larger than serial: serial without timing
    assert xksv_tune.size_rule(bytes(60), bytes(70), raw)[0] == "bf16-huffman-tile16"
    assert xksv_tune.size_rule(bytes(60), bytes(69), raw) is None


class StubTuner(xksv_tune.GpuTuner):
    """GpuTuner without a GPU: measure() returns scripted times."""

    def __init__(self, times, profile=None):
        self.profile = profile or {"device": {"name": "stub", "compute_capability": [10, 0]},
                                   "method": "stub", "choices": {}}
        self.times, self.calls = list(times), 0

    def measure(self, blob, rows, cols, codec):
        self.calls += 1
        return self.times.pop(0)


def test_measured_choice_is_cached_per_group():
    t = StubTuner([2.0, 1.0])  # serial 2 s, parallel 1 s
    raw, ser, par = bytes(1000), bytes(700), bytes(760)
    assert t.select(ser, par, raw, 16, 4096) == ("bf16-huffman-parallel32", par)
    # same rows, cols and serial size in sixteenths of raw: no new measurement
    assert t.select(bytes(710), bytes(770), raw, 16, 4096)[0] == "bf16-huffman-parallel32"
    assert t.calls == 2
    assert t.profile["choices"] == {"16:4096:11": {"serial_seconds": 2.0, "parallel_seconds": 1.0,
                                                   "prefer_parallel": True}}
    t.times = [1.0, 3.0]
    assert t.select(bytes(600), bytes(650), raw, 16, 4096)[0] == "bf16-huffman-tile16"
    assert "16:4096:9" in t.profile["choices"] and t.calls == 4


def test_tuner_needs_a_gpu_or_matching_profile():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        with pytest.raises(ValueError, match="resume GPU differs"):
            xksv_tune.GpuTuner({"device": {"name": "other", "compute_capability": [1, 0]}})
    else:
        with pytest.raises(ValueError, match="requires CUDA"):
            xksv_tune.GpuTuner()
