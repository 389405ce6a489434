"""Codec autotuner on this library's kernels (python/tune.py:8-42, GpuTuner).

For each BF16 block the compiler encodes both codecs and asks ``select``
which to store.  The rules are the reference's: raw when neither encoding is
smaller than the raw bytes; the other codec when one of them is not; serial
when the parallel encoding is more than 15 % larger; otherwise a measured
decode-time comparison, cached per (rows, cols, serial size in sixteenths of
raw) so similar slabs share one measurement, in a profile stored in the
archive index (and accepted back on resume only on the same GPU model).

What is timed differs from the reference on purpose: the reference times one
blocking ABI call per slab (host buffer, copy, launch, synchronise), which on
this library measures the call overhead rather than the codec.  Here a slab is
replicated `copies` times in HBM and decoded by one plan launch, device-timed
with CUDA events: the per-slab cost the resident runtime pays.
"""
import statistics

import xksv_gpu

MAX_PARALLEL_OVERHEAD = 115  # percent of the serial size (python/tune.py:23)


class GpuTuner:
    def __init__(self, profile=None, device=None, copies=256, repeats=3):
        import torch
        if not torch.cuda.is_available():
            raise ValueError("autotuning requires CUDA-enabled PyTorch and an available GPU")
        self.torch = torch
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        props = torch.cuda.get_device_properties(self.device)
        identity = {"name": props.name, "compute_capability": [props.major, props.minor]}
        if profile is not None and profile.get("device") != identity:
            raise ValueError("resume GPU differs from the autotuning GPU")
        self.copies, self.repeats = copies, repeats
        self.profile = profile if profile is not None else {
            "device": identity,
            "method": (f"median of {repeats} device-timed plan decodes of {copies} copies of the slab "
                       "after warmup, seconds per slab; parallel limited to 15% larger than serial"),
            "choices": {}}
        self.lib = xksv_gpu.load()

    def select(self, serial, parallel, raw, rows, cols):
        """(codec name, bytes to store) for one block."""
        rule = size_rule(serial, parallel, raw)
        if rule is not None:
            return rule
        key = f"{rows}:{cols}:{len(serial) * 16 // len(raw)}"
        choice = self.profile["choices"].get(key)
        if choice is None:
            ts = self.measure(serial, rows, cols, xksv_gpu.CODEC_TILE16)
            tp = self.measure(parallel, rows, cols, xksv_gpu.CODEC_PARALLEL32)
            choice = {"serial_seconds": ts, "parallel_seconds": tp, "prefer_parallel": tp < ts}
            self.profile["choices"][key] = choice
        return ("bf16-huffman-parallel32", parallel) if choice["prefer_parallel"] else ("bf16-huffman-tile16", serial)

    def measure(self, blob, rows, cols, codec):
        """Device seconds per slab of decoding `copies` copies of `blob`."""
        torch = self.torch
        blob = bytes(memoryview(blob))
        n, size = self.copies, len(blob)
        stride = -(-size // 16) * 16
        host = bytearray(stride * n)
        for i in range(n):
            host[i * stride:i * stride + size] = blob
        with torch.cuda.device(self.device):
            payload = torch.frombuffer(host, dtype=torch.uint8).to(self.device)
            out = torch.empty(n * rows * cols * 2, dtype=torch.uint8, device=self.device)
            entries = [dict(src_offset=i * stride, src_size=size, rows=rows, cols=cols,
                            dst_offset=i * rows * cols * 2, codec=codec) for i in range(n)]
            plan = xksv_gpu.Plan(entries, lib=self.lib)
            stream = torch.cuda.current_stream(self.device)
            try:
                plan.decode(payload, out, stream.cuda_stream)
                if plan.status(stream.cuda_stream):
                    raise ValueError("GPU autotuning decode failed")
                samples = []
                for _ in range(self.repeats):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record(stream)
                    plan.decode(payload, out, stream.cuda_stream)
                    b.record(stream)
                    b.synchronize()
                    samples.append(a.elapsed_time(b) / 1e3 / n)
                if plan.status(stream.cuda_stream):
                    raise ValueError("GPU autotuning decode failed")
            finally:
                plan.close()
        return statistics.median(samples)


def size_rule(serial, parallel, raw):
    """The size-only decisions of python/tune.py:22-24, or None when the two
    codecs need a timing comparison."""
    if len(serial) >= len(raw) and len(parallel) >= len(raw):
        return "raw", raw
    if len(serial) >= len(raw):
        return "bf16-huffman-parallel32", parallel
    if len(parallel) >= len(raw) or len(parallel) * 100 > len(serial) * MAX_PARALLEL_OVERHEAD:
        return "bf16-huffman-tile16", serial
    return None
