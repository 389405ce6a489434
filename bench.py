#!/usr/bin/env python3
"""Benchmark of the .xksv slab-decode hot path on B200.

Workload: a Llama-1.1B-shaped checkpoint (hidden
2048, 22 layers, 32 q / 4 kv heads of dim 64, FFN 5632, vocab 32000, untied
lm_head; linear weights and embeddings BF16 N(0, 0.02), norms 1.0, seeded),
compiled with the `dfloat11-parallel` codec into the compiler's slabs (16-row,
1 MiB slabs; raw when encoding does not shrink a slab), and decoded whole to
BF16 on each GPU.  A step is one decode of the whole checkpoint from
HBM-resident compressed slabs (value); `e2e` repeats it through the public C
ABI with the compressed payload in pinned host memory, host->device copy
inside the timed region.  Secondary (`fused_gemv`): batch-1 fused decode+GEMV
over every linear of a Llama-3-8B-shaped model.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "xks-vectorforge_b200"))

METRIC = "decode GB/s (BF16 out) vs HBM roofline; fused-GEMV tok/s Llama-8B b=1"
HBM_FALLBACK_GBS = 6650.0
# bytes of one 16-row serial slab's GEMV tables kept by xksv_plan_index
# (sizeof(GemvTabs) in the library: 2048 16-bit entries + long-code data)
GEMV_TABLE_BYTES = 5920


def llama_tensors(hidden, layers, q_heads, kv_heads, head_dim, ffn, vocab, tied=False):
    """(name, rows, cols, kind) in checkpoint order; 1-D norms are 1 x hidden
    slabs, as the compiler lays out 1-D BF16 tensors of <= 4096 elements."""
    out = [("model.embed_tokens.weight", vocab, hidden, "w")]
    for i in range(layers):
        p = f"model.layers.{i}."
        out += [(p + "self_attn.q_proj.weight", q_heads * head_dim, hidden, "w"),
                (p + "self_attn.k_proj.weight", kv_heads * head_dim, hidden, "w"),
                (p + "self_attn.v_proj.weight", kv_heads * head_dim, hidden, "w"),
                (p + "self_attn.o_proj.weight", hidden, q_heads * head_dim, "w"),
                (p + "mlp.gate_proj.weight", ffn, hidden, "w"),
                (p + "mlp.up_proj.weight", ffn, hidden, "w"),
                (p + "mlp.down_proj.weight", hidden, ffn, "w"),
                (p + "input_layernorm.weight", 1, hidden, "norm"),
                (p + "post_attention_layernorm.weight", 1, hidden, "norm")]
    out.append(("model.norm.weight", 1, hidden, "norm"))
    if not tied:
        out.append(("lm_head.weight", vocab, hidden, "w"))
    return out


CONFIG2 = dict(hidden=2048, layers=22, q_heads=32, kv_heads=4, head_dim=64, ffn=5632, vocab=32000)
CONFIG3 = dict(hidden=4096, layers=32, q_heads=32, kv_heads=8, head_dim=128, ffn=14336, vocab=128256)


def host_threads(world):
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(1, n // max(1, world))


def build_archive(tensors, codec, sigma, seed, device, threads, only_kinds=("w", "norm"),
                  row_range=None):
    """Generates the seeded BF16 tensors on the GPU, compiles them on the host
    with the library's encoder, returns (payload uint8 numpy, slabs, out_bytes,
    per-tensor info).  `row_range(rows) -> (r0, r1)` keeps only those rows of
    every tensor (a tensor-parallel shard; the full tensors are generated so
    every rank sees the same weights)."""
    import numpy as np
    import torch
    import xksv_gpu

    gen = torch.Generator(device=device).manual_seed(seed)
    parts, slabs, info = [], [], []
    src = dst = 0
    for name, rows, cols, kind in tensors:
        if kind not in only_kinds:
            continue
        if kind == "norm":
            t = torch.ones(rows, cols, dtype=torch.bfloat16, device=device)
        else:
            t = (torch.randn(rows, cols, generator=gen, device=device) * sigma).to(torch.bfloat16)
        if row_range is not None:
            r0, r1 = row_range(rows)
            t = t[r0:r1].contiguous()
            rows = r1 - r0
        h = t.view(torch.int16).cpu().numpy()
        pay, sl = xksv_gpu.host_pack_tensor(h.ctypes.data, h.nbytes, rows, cols, codec,
                                            threads=threads, dst_base=dst)
        for s in sl:
            s["src_offset"] += src
        info.append(dict(name=name, rows=rows, cols=cols, dst=dst, first=len(slabs), n=len(sl)))
        slabs += sl
        parts.append(pay)
        src += pay.nbytes
        dst += h.nbytes
    return np.concatenate(parts), slabs, dst, info


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
        except Exception:
            pass
    return HBM_FALLBACK_GBS, "fallback (no MEASURED_PEAKS.json)"


class ClockSampler:
    """nvidia-smi clock / throttle sampling under load.  The sampler is started
    before the warm-up and waits for its first sample; the summary covers the
    samples taken from mark() (the start of the warm-up steps) to the end of
    the timed steps, at 10 ms intervals: the timed region alone is a few tens
    of milliseconds, shorter than nvidia-smi's start-up."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.mark_at = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "10", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            t0 = time.time()
            while not self.lines and self.proc.poll() is None and time.time() - t0 < 5.0:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        return self

    def mark(self):
        self.mark_at = len(self.lines)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            t0 = time.time()  # at least two samples from the loaded window
            while len(self.lines) < self.mark_at + 2 and self.proc.poll() is None and time.time() - t0 < 1.0:
                time.sleep(0.005)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = self.lines[self.mark_at:] or self.lines
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=mx or None,
                    reasons=sorted(reasons), samples=len(sm), window="warm-up and timed steps, 10 ms interval")


def time_steps(fn, steps, stream):
    import torch
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    stop.record(stream)
    stop.synchronize()
    return start.elapsed_time(stop) / 1e3


def workload_config(world):
    """The `config` of the headline line, from the workload's definition alone,
    so the reference arm (which never builds the GPU archive) prints the same
    dict as this arm."""
    tensors = llama_tensors(**CONFIG2)
    return dict(workload="configs[1]: Llama-1.1B-shaped checkpoint (h2048, 22L, 32/4 heads, FFN 5632, "
                         "vocab 32000, untied), dfloat11-parallel, whole-checkpoint decode per GPU",
                codec="bf16-huffman-parallel32", weights="BF16 N(0, 0.02) seed 1, norms 1.0",
                tensors=len(tensors), out_bytes=sum(r * c * 2 for _, r, c, _ in tensors),
                l2="inputs (compressed + decoded, ~3.9 GB) larger than L2 (126 MB); no flush",
                parallelism=f"slab partition, {world} independent GPU(s), no collective")


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _bf16_rne(x):
    """float32 numpy array -> BF16 bit patterns (round to nearest even)."""
    import numpy as np
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype("<u2")


CPU_SAMPLE_FRACTION = 0.1


def cpu_sample(threads, fraction=CPU_SAMPLE_FRACTION, sigma=0.02, seed=1):
    """A stratified sample of the configs[1] checkpoint for the CPU legs: the
    first `fraction` of every tensor's 16-row slabs (every norm whole), drawn
    with numpy (seeded per tensor) and encoded by the reference's own encoder
    (oracle/_ref xksv_pack_parallel; a slab that does not shrink is stored raw,
    src/compile.cpp:264-273, slab rows as src/compile.cpp:471-479).  Returns
    (reference library or None, kind, [dict(blob, raw, rows, cols, codec)]).
    Loads no library of this repository's product."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    from oracle.oracle import Oracle, Reference
    try:
        lib, kind = Reference(), "reference"
    except OSError:
        lib, kind = Oracle(), "port"
    jobs = []
    for i, (name, rows, cols, kind_t) in enumerate(llama_tensors(**CONFIG2)):
        nslab = -(-rows // 16)
        take = nslab if kind_t == "norm" else max(1, int(nslab * fraction))
        r = min(rows, take * 16)
        if kind_t == "norm":
            w = np.full((r, cols), 0x3F80, dtype="<u2")
        else:
            rng = np.random.default_rng([seed, i])
            w = _bf16_rne(rng.standard_normal((r, cols), dtype=np.float32) * sigma)
        for r0 in range(0, r, 16):
            jobs.append((w[r0:r0 + 16].tobytes(), min(16, r - r0), cols))

    def enc(job):
        raw, rows, cols = job
        blob = lib.pack_parallel(raw, rows, cols)
        if len(blob) < len(raw):
            return dict(blob=blob, raw=raw, rows=rows, cols=cols, codec=2)
        return dict(blob=raw, raw=raw, rows=rows, cols=cols, codec=0)

    with ThreadPoolExecutor(max_workers=threads) as ex:
        slabs = list(ex.map(enc, jobs))
    return lib, kind, slabs


def cpu_decode_rate(lib, slabs, threads, seconds, check=False):
    """Reference CPU decode (xksv_unpack_parallel; raw slabs are copies) of the
    sample on `threads` host threads, repeated for at least `seconds` (one
    pass at least).  With `check`, an untimed pass first compares every
    decoded slab with its source bytes.  Returns (GB/s of BF16 out, passes,
    seconds, bytes_match)."""
    import ctypes
    from concurrent.futures import ThreadPoolExecutor
    coded = [s for s in slabs if s["codec"] == 2]
    bufs = [ctypes.create_string_buffer(s["blob"], len(s["blob"])) for s in coded]
    unpack = getattr(lib.lib, lib.prefix + "unpack_parallel")
    free = getattr(lib.lib, lib.prefix + "free")

    def one(k, check=False):
        out, size = ctypes.c_void_p(), ctypes.c_size_t()
        if unpack(bufs[k], len(coded[k]["blob"]), ctypes.byref(out), ctypes.byref(size)):
            raise RuntimeError("reference CPU decode failed")
        ok = True
        if check:
            ok = ctypes.string_at(out, size.value) == coded[k]["raw"]
        free(out)
        return size.value, ok

    match = True
    done, passes = 0, 0
    with ThreadPoolExecutor(max_workers=threads) as ex:
        if check:
            match = all(r[1] for r in ex.map(lambda k: one(k, True), range(len(coded))))
        t0 = time.perf_counter()
        while passes == 0 or time.perf_counter() - t0 < seconds:
            done += sum(r[0] for r in ex.map(one, range(len(coded))))
            passes += 1
    dt = time.perf_counter() - t0
    return done / dt / 1e9, passes, dt, bool(match)


def cpu_baseline(seconds):
    """The reference's CPU decode of the workload, on the GPU box's host: one
    thread (how the reference itself decodes: per block in sequence,
    src/verify.cpp:251-255, python/xksv.py:370) and every host thread (one slab
    per task).  `value` is the all-thread figure."""
    threads = host_threads(1)
    lib, kind, slabs = cpu_sample(threads)
    out = sum(len(s["raw"]) for s in slabs if s["codec"] == 2)
    v1, p1, t1, ok1 = cpu_decode_rate(lib, slabs, 1, seconds / 2, check=True)
    vn, pn, tn, okn = cpu_decode_rate(lib, slabs, threads, seconds / 2)
    return dict(value=round(vn, 3), unit="GB/s", cores=threads, kind=kind,
                single_thread=dict(value=round(v1, 3), unit="GB/s", cores=1),
                cpu_model=cpu_model(), bytes_match=ok1 and okn,
                sample=(f"{len([s for s in slabs if s['codec'] == 2])} coded slabs ({out / 1e9:.3f} GB BF16 out: "
                        f"the first {int(CPU_SAMPLE_FRACTION * 100)} % of every tensor's slabs, numpy-drawn, encoded "
                        f"by the reference encoder), decoded {p1} x on 1 thread in {t1:.1f} s and {pn} x on "
                        f"{threads} threads in {tn:.1f} s; every slab byte-checked in an untimed pass"))


def run_reference(args, rank, world):
    """The reference arm: the reference's own CPU decode (oracle/_ref, built
    from its sources) of the headline workload on this box's host threads.
    It loads no library of this repository's product (no GPU path)."""
    if rank != 0:
        return
    threads = host_threads(1)
    lib, kind, slabs = cpu_sample(threads)
    vals = []
    _, _, _, match = cpu_decode_rate(lib, slabs, threads, 0.0, check=True)  # warm-up, byte-checked
    for _ in range(max(0, args.warmup_cpu)):
        cpu_decode_rate(lib, slabs, threads, 0.0)
    t_all = 0.0
    for _ in range(args.steps):
        v, _, dt, _ = cpu_decode_rate(lib, slabs, threads, 0.0)
        vals.append(v)
        t_all += dt
    value = statistics.median(vals)
    coded = [s for s in slabs if s["codec"] == 2]
    out = sum(len(s["raw"]) for s in coded)
    sample = (f"{len(coded)} coded slabs ({out / 1e9:.3f} GB BF16 out: the first {int(CPU_SAMPLE_FRACTION * 100)} % "
              f"of every tensor's slabs, numpy-drawn, encoded by the reference encoder); one decode pass of the "
              f"sample per step, {args.steps} steps in {t_all:.1f} s; median step")
    line = dict(metric=METRIC, value=round(value, 3), unit="GB/s", impl="reference", n_gpus=world,
                steps=args.steps, warmup=args.warmup, ms_per_step=round(t_all / max(1, args.steps) * 1e3, 3),
                higher_is_better=True, scaling="weak", vs_baseline=None, dtype="bf16",
                data="synthetic: seeded BF16 N(0,0.02) Llama-1.1B-shaped weights, norms 1.0 (no checkpoint download)",
                config=workload_config(world),
                cpu_baseline=dict(value=round(value, 3), unit="GB/s", cores=threads, kind=kind, sample=sample,
                                  cpu_model=cpu_model(), bytes_match=bool(match)),
                e2e=dict(value=round(value, 3), unit="GB/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


def fused_gemv(args, dev, stream, threads):
    """Batch-1 fused decode+GEMV over every linear of a Llama-3-8B-shaped
    model (lm_head excluded, as the reference runtime does, runtime.py:258);
    one plan per layer group so each layer's four dependent GEMV launches
    (qkv, o, gate+up, down) run in order, all captured in one CUDA graph."""
    import numpy as np
    import torch
    import xksv_gpu

    cfg = CONFIG3
    tensors = [t for t in llama_tensors(**cfg) if t[3] == "w" and ("layers." in t[0])]
    payload, slabs, _, info = build_archive(tensors, 1, 0.02, 2, dev, threads)
    d_payload = torch.from_numpy(payload).to(dev)
    comp_bytes = payload.nbytes
    # x segments: one FP32 vector per linear input; y rows per linear
    groups = []  # per layer: [qkv], [o], [gate, up], [down]
    xs, ys = 0, 0
    plans = []
    name_to = {i["name"]: i for i in info}
    for L in range(cfg["layers"]):
        p = f"model.layers.{L}."
        for members in ([p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight"],
                        [p + "self_attn.o_proj.weight"],
                        [p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"],
                        [p + "mlp.down_proj.weight"]):
            cols = name_to[members[0]]["cols"]
            entries = []
            for m in members:
                t = name_to[m]
                for s in slabs[t["first"]:t["first"] + t["n"]]:
                    e = dict(s)
                    e["dst_offset"] = ys + (s["dst_offset"] - t["dst"]) // (2 * t["cols"])
                    e["x_offset"] = xs
                    entries.append(e)
                ys += t["rows"]
            xs += cols
            plans.append(xksv_gpu.Plan(entries))
    x = torch.randn(xs, generator=torch.Generator(device=dev).manual_seed(3), device=dev).to(torch.bfloat16).float()
    y = torch.empty(ys, device=dev)
    h = stream.cuda_stream
    # one-time tile index of the resident weights (xksv_plan_index)
    t_idx = time.perf_counter()
    for pl in plans:
        if pl.index(d_payload, h):
            raise RuntimeError("xksv_plan_index failed")
    index_s = time.perf_counter() - t_idx

    def forward():
        for pl in plans:
            pl.gemm(d_payload, x, y, 1, h)

    with torch.cuda.stream(stream):
        for _ in range(3):
            forward()
    stream.synchronize()
    bad = sum(pl.status(h) for pl in plans)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        forward()
    launches = sum(pl.launches() for pl in plans)
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
        torch.cuda.nvtx.range_push("timed")
        t = time_steps(graph.replay, args.gemv_steps, stream)
        torch.cuda.nvtx.range_pop()
    ms = t / args.gemv_steps * 1e3
    bad += sum(pl.status(h) for pl in plans)
    # correctness spot check of one layer's down_proj against an FP32 matmul of
    # the decoded weights (decode plan of the same slabs)
    t0 = name_to["model.layers.0.mlp.down_proj.weight"]
    dplan = xksv_gpu.Plan(slabs[t0["first"]:t0["first"] + t0["n"]])
    wdec = torch.empty(t0["rows"] * t0["cols"] * 2 + t0["dst"], dtype=torch.uint8, device=dev)
    dplan.decode(d_payload, wdec, h)
    bad += dplan.status(h)
    W = wdec[t0["dst"]:].view(torch.bfloat16).view(t0["rows"], t0["cols"]).float()
    # down_proj is the 4th group of layer 0: its x and y offsets
    xo = cfg["hidden"] + cfg["q_heads"] * cfg["head_dim"] + cfg["hidden"]
    yo = (cfg["q_heads"] + 2 * cfg["kv_heads"]) * cfg["head_dim"] + cfg["hidden"] + 2 * cfg["ffn"]
    ref = W @ x[xo:xo + t0["cols"]]
    got = y[yo:yo + t0["rows"]]
    rel = float((got - ref).norm() / ref.norm())
    del graph
    # batch 16 on the tensor cores: the fused decode -> tcgen05 kernel against
    # the decode-to-scratch route (one scratch shared by every plan)
    nb = 16
    xb = torch.randn(xs, nb, generator=torch.Generator(device=dev).manual_seed(4), device=dev)
    yb = torch.empty(ys, nb, device=dev)
    need = max(pl.scratch_bytes() for pl in plans)
    scratch = torch.empty(need, dtype=torch.uint8, device=dev)
    for pl in plans:
        pl.set_scratch(scratch.data_ptr(), need)
    b16 = dict(batch=nb, fused_ready_plans=sum(pl.fused_ready(d_payload) for pl in plans), plans=len(plans))
    for route, code in (("fused", xksv_gpu.GEMM_FUSED), ("scratch", xksv_gpu.GEMM_SCRATCH)):
        for pl in plans:
            pl.set_gemm_route(code)

        def forward_b():
            for pl in plans:
                pl.gemm(d_payload, xb, yb, nb, h)
        with torch.cuda.stream(stream):
            for _ in range(2):
                forward_b()
        stream.synchronize()
        bad += sum(pl.status(h) for pl in plans)
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=stream):
            forward_b()
        nl = sum(pl.launches() for pl in plans)
        with torch.cuda.stream(stream):
            g2.replay()
            t2 = time_steps(g2.replay, args.gemv_steps, stream)
        ms2 = t2 / args.gemv_steps * 1e3
        bad += sum(pl.status(h) for pl in plans)
        refb = W @ xb[xo:xo + t0["cols"]].to(torch.bfloat16).float()
        relb = float((yb[yo:yo + t0["rows"]] - refb).norm() / refb.norm())
        b16[route] = dict(tok_s=round(nb * 1e3 / ms2, 1), ms_per_forward=round(ms2, 3), launches=nl,
                          hbm_gbs=round(comp_bytes / (ms2 / 1e3) / 1e9, 1), rel_l2_layer0_down=relb)
        del g2
    for pl in plans:
        pl.set_gemm_route(xksv_gpu.GEMM_AUTO)
        pl.close()
    dplan.close()
    del scratch
    return dict(metric="fused-GEMV tok/s Llama-8B b=1", value=round(1e3 / ms, 2), unit="tok/s",
                ms_per_token=round(ms, 4), codec="dfloat11", compressed_bytes=comp_bytes,
                hbm_gbs=round(comp_bytes / (ms / 1e3) / 1e9, 1), launches_per_token=launches,
                index_build_s=round(index_s, 3),
                index_bytes=8 * sum(t["n"] * (t["cols"] // 16 + 1) for t in info),
                table_bytes=GEMV_TABLE_BYTES * sum(t["n"] for t in info),
                rel_l2_layer0_down=rel, status_errors=bad, batch16=b16,
                note="per token: 128 dependent plan launches (qkv, o, gate+up, down per layer) in one CUDA graph; "
                     "lm_head excluded as in runtime.py:258; batch16: the same plans at batch 16 on the tensor cores "
                     "(fused decode->tcgen05 kernel vs decode to a BF16 scratch + tcgen05 GEMM), X rounded to BF16")


def run_case(args):
    """Small fixed decode workload for profiling and kernel timing:
    `--case CODEC:ROWSxCOLS:SLABS` decodes SLABS slabs (64 distinct seeded
    N(0, 0.02) slabs, repeated) in one plan launch per step, HBM-resident;
    CODEC is `serial` (bf16-huffman-tile16) or `parallel` (XKSP2).  Prints
    one JSON line with the per-launch time."""
    import numpy as np
    import torch
    import xksv_gpu

    codec_name, shape, nslabs = args.case.split(":")
    gemv = codec_name.startswith("gemv-")
    indexed = codec_name == "iserial"  # serial codec, decoded through the plan's tile index
    codec = {"serial": 1, "parallel": 2, "iserial": 1}[codec_name[5:] if gemv else codec_name]
    rows, cols = map(int, shape.split("x"))
    nslabs = int(nslabs)
    dev = "cuda:0"
    torch.cuda.set_device(0)
    lib = xksv_gpu.load()
    gen = torch.Generator(device=dev).manual_seed(5)
    uniq = []
    for _ in range(min(64, nslabs)):
        w = (torch.randn(rows, cols, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        tile = w.view(torch.int16).cpu().numpy().tobytes()
        uniq.append(xksv_gpu.host_pack(tile, rows, cols, codec, lib))
    payload, entries, out = bytearray(), [], 0
    for i in range(nslabs):
        b = uniq[i % len(uniq)]
        # GEMV: slab i computes rows 16i.. of Y from all of X
        entries.append(dict(src_offset=len(payload), src_size=len(b), rows=rows, cols=cols,
                            dst_offset=i * rows if gemv else out, codec=codec))
        payload += b
        out += rows * cols * 2
    d_payload = torch.frombuffer(payload, dtype=torch.uint8).to(dev)
    plan = xksv_gpu.Plan(entries)
    stream = torch.cuda.Stream(device=dev)
    h = stream.cuda_stream
    if gemv:
        nb = args.batch
        x = torch.randn(cols, nb, device=dev)
        y = torch.empty(nslabs * rows, nb, device=dev)
        if plan.index(d_payload, h):
            raise RuntimeError("xksv_plan_index failed")
        plan.set_gemm_route({"auto": xksv_gpu.GEMM_AUTO, "scratch": xksv_gpu.GEMM_SCRATCH,
                             "fused": xksv_gpu.GEMM_FUSED}[args.route])
        fn = lambda: plan.gemm(d_payload, x, y, nb, h)
    else:
        d_out = torch.empty(out, dtype=torch.uint8, device=dev)
        if indexed and plan.index(d_payload, h):
            raise RuntimeError("xksv_plan_index failed")
        fn = lambda: plan.decode(d_payload, d_out, h)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            fn()
        assert plan.status(h) == 0, "slab error"
        torch.cuda.nvtx.range_push("timed")
        t = time_steps(fn, args.steps, stream)
        torch.cuda.nvtx.range_pop()
    assert plan.status(h) == 0
    launches = plan.launches()
    plan.close()
    ms = t / args.steps * 1e3
    line = dict(case=args.case, slabs=nslabs, compressed_bytes=len(payload), out_bytes=out,
                ms_per_launch=round(ms, 5))
    if gemv:
        # read per call: each tile's first-code offset (and row-8 offset when a
        # tile takes two threads) and each slab's tables from the index pass
        idx = nslabs * ((cols // 16 + 1) * 8 + GEMV_TABLE_BYTES)
        line.update(batch=args.batch, launches=launches, route=args.route,
                    tflops=round(2 * (out / 2) * args.batch / ms / 1e9, 2),
                    gweights_per_s=round(out / 2 / ms / 1e6, 1),
                    traffic_gbs=round((len(payload) + idx) / ms / 1e6, 1), index_bytes=idx)
    else:
        line.update(out_gbs=round(out / ms / 1e6, 1), traffic_gbs=round((out + len(payload)) / ms / 1e6, 1))
    print(json.dumps(line), flush=True)


CONFIG4 = dict(hidden=8192, layers=80, q_heads=64, kv_heads=8, head_dim=128, ffn=28672, vocab=128256)


class _DeviceBytes:
    """Zero-copy torch view of library-allocated device bytes."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def device_archive(specs, codec, dev, stream, bound):
    """Encodes tensors on the GPU (xksv_cuda_pack_tensor) into one device
    payload.  specs: (name, rows, cols, make) with make() -> BF16 [rows, cols]
    on `dev`.  The payload buffer is allocated once at `bound` x the raw bytes
    (each tensor's slabs start 16-byte aligned).  Returns (payload, [dict(name,
    rows, cols, slabs)], compressed bytes, raw bytes)."""
    import torch
    import xksv_gpu
    raw = sum(r * c * 2 for _, r, c, _ in specs)
    buf = torch.empty(int(raw * bound) + (64 << 20), dtype=torch.uint8, device=dev)
    h = stream.cuda_stream
    pos, info = 0, []
    for name, rows, cols, make in specs:
        t = make()
        stream.wait_stream(torch.cuda.current_stream(dev))  # t is made on the current stream
        with torch.cuda.stream(stream):
            ptr, n, sl = xksv_gpu.cuda_pack_tensor(t.data_ptr(), rows, cols, codec, 0, h)
            try:
                if pos + n > buf.numel():
                    raise RuntimeError("compressed payload exceeds its preallocated bound")
                if n:
                    buf[pos:pos + n].copy_(torch.as_tensor(_DeviceBytes(ptr, n), device=dev))
            finally:
                xksv_gpu.free_device(ptr)
        for s in sl:
            s["src_offset"] += pos
        info.append(dict(name=name, rows=rows, cols=cols, slabs=sl))
        pos = (pos + n + 15) // 16 * 16
        del t
    stream.synchronize()
    return buf, info, pos, raw


def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _max_over_ranks(v, world, dev):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def config4_specs(world, rank, dev, sigma=0.015, seed=3):
    """The Llama-3-70B tensors in checkpoint order, this
    rank's rows (whole 16-row slabs; the 1-row norms on rank 0), generated on
    the GPU from one seeded stream (every rank draws the full tensors, so the
    shards partition one model)."""
    import torch
    import xksv_gpu
    gen = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for name, rows, cols, kind in llama_tensors(**CONFIG4):
        if kind == "norm":
            if rank == 0:
                out.append((name, rows, cols, lambda r=rows, c=cols: torch.ones(r, c, dtype=torch.bfloat16, device=dev)))
            continue
        r0, r1 = xksv_gpu.shard_rows(rows, world, rank)

        def make(rows=rows, cols=cols, r0=r0, r1=r1):
            full = (torch.randn(rows, cols, generator=gen, device=dev) * sigma).to(torch.bfloat16)
            return full[r0:r1].contiguous()
        out.append((name, r1 - r0, cols, make))
    return out


def _case_setup():
    """Device, NCCL group (N > 1) and stream of a `--case` run."""
    import torch
    import xksv_gpu
    world, rank, local = _dist_env()
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=torch.device(dev))
    xksv_gpu.load()
    return world, rank, dev, torch.cuda.Stream(device=dev)


def run_config4_decode(args):
    """`--case config4-decode`: prints config4_decode()'s line."""
    world, rank, dev, stream = _case_setup()
    line = config4_decode(args, dev, stream, world, rank)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def config4_decode(args, dev, stream, world, rank):
    """Whole-model decode of the Llama-3-70B-shaped model (BASELINE
    configs[3]), `dfloat11-parallel`, row-sharded over the ranks (strong
    scaling: the model is fixed).  The rank's compressed shard (~97 GB / N) is
    resident; a step decodes every slab once, in plans of ~6 GB of output
    each, into an output buffer the plans reuse (compressed + decoded = 238 GB
    does not fit one GPU).  Before timing, every decoded tensor is compared
    bit for bit with its source regenerated from the seed."""
    import torch
    import xksv_gpu
    h = stream.cuda_stream
    t0 = time.perf_counter()
    specs = config4_specs(world, rank, dev)
    payload, info, comp, raw = device_archive(specs, 2, dev, stream, 0.78)
    build_s = time.perf_counter() - t0
    # plans of whole layers holding ~6 GB of output each (4 layers on one GPU,
    # more when the rows are sharded; embed and lm_head join the first and
    # last): a launch of many waves keeps each plan's tail short; within a
    # plan the longest slabs start first
    groups, cur, cur_bytes = [], [], 0
    for t in info:
        cur.append(t)
        cur_bytes += t["rows"] * t["cols"] * 2
        if t["name"].endswith("post_attention_layernorm.weight") and cur_bytes >= (6 << 30):
            groups.append(cur)
            cur, cur_bytes = [], 0
    if cur:
        groups.append(cur)
    plans, spans, max_out = [], [], 0
    for g in groups:
        entries, base, span = [], 0, []
        for t in g:
            for s in t["slabs"]:
                e = dict(s)
                e["dst_offset"] = base + s["dst_offset"]
                entries.append(e)
            span.append((t["name"], base, t["rows"] * t["cols"] * 2))
            base += (t["rows"] * t["cols"] * 2 + 255) // 256 * 256
        entries.sort(key=lambda e: -e["src_size"])
        plans.append(xksv_gpu.Plan(entries))
        spans.append(span)
        max_out = max(max_out, base)
    out = torch.empty(max_out, dtype=torch.uint8, device=dev)

    def step():
        for pl in plans:
            pl.decode(payload, out, h)

    # bit-exact check of every tensor against its regenerated source
    check = config4_specs(world, rank, dev)
    k = 0
    mismatches = 0
    with torch.cuda.stream(stream):
        for pl, span in zip(plans, spans):
            pl.decode(payload, out, h)
            if pl.status(h):
                raise RuntimeError("decode reported a slab error")
            for name, off, n in span:
                _, rows, cols, make = check[k]
                assert name == check[k][0]
                src = make().view(torch.int16).reshape(-1)
                got = out[off:off + n].view(torch.int16)
                mismatches += int(not torch.equal(src, got))
                k += 1
    if mismatches:
        raise RuntimeError(f"{mismatches} tensors differ from their source")
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        stream.synchronize()
        if world > 1:
            torch.distributed.barrier()
        t = time_steps(step, args.steps, stream)
    t = _max_over_ranks(t, world, dev)
    bad = sum(pl.status(h) for pl in plans)
    ms = t / args.steps * 1e3
    peak, peak_src = measured_peak()
    line = dict(case="config4-decode", config="configs[3] Llama-3-70B shapes, N(0,0.015) seed 3, dfloat11-parallel, "
                "rows sharded in whole slabs", scaling="strong", n_gpus=world, steps=args.steps,
                ms_per_step=round(ms, 3),
                per_rank_out_bytes=raw, per_rank_compressed_bytes=comp,
                value=round(world * raw / (ms / 1e3) / 1e9, 1), unit="GB/s BF16 out (all ranks)",
                per_gpu_out_gbs=round(raw / (ms / 1e3) / 1e9, 1),
                roofline=dict(bound="hbm", achieved=round((raw + comp) / (ms / 1e3) / 1e9, 1), peak=peak,
                              frac=round((raw + comp) / (ms / 1e3) / 1e9 / peak, 4), peak_source=peak_src),
                launches_per_step=sum(pl.launches() for pl in plans), plans=len(plans),
                bit_exact_tensors=len(check), status_errors=bad, build_s=round(build_s, 1),
                note="output buffer reused per plan of ~6 GB output; inputs larger than L2")
    for pl in plans:
        pl.close()
    del payload, out
    torch.cuda.empty_cache()
    return line


def run_config4_gemv(args):
    """`--case config4-gemv`: fused decode-GEMV/GEMM over the linears of the
    Llama-3-70B-shaped model, `dfloat11` with the tile
    index, 1 GPU: the full forward of linears (320 dependent plan calls, one
    CUDA graph) at batch 1 and 4 on the CUDA cores and at batch 8 and 16 on
    the tensor cores, all plans sharing one decode scratch."""
    import torch
    import xksv_gpu
    torch.cuda.set_device(0)
    dev = "cuda:0"
    xksv_gpu.load()
    stream = torch.cuda.Stream(device=dev)
    h = stream.cuda_stream
    cfg = CONFIG4
    specs = [s for s in config4_specs(1, 0, dev) if "layers." in s[0] and not s[0].endswith("norm.weight")]
    t0 = time.perf_counter()
    payload, info, comp, raw = device_archive(specs, 1, dev, stream, 0.72)
    build_s = time.perf_counter() - t0
    by = {t["name"]: t for t in info}
    plans, xs, ys, groups = [], 0, 0, []
    for L in range(cfg["layers"]):
        p = f"model.layers.{L}."
        for members in ([p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight"],
                        [p + "self_attn.o_proj.weight"],
                        [p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"],
                        [p + "mlp.down_proj.weight"]):
            entries, y0 = [], ys
            for m in members:
                t = by[m]
                for s in t["slabs"]:
                    e = dict(s)
                    e["dst_offset"] = ys + s["dst_offset"] // (2 * t["cols"])
                    e["x_offset"] = xs
                    entries.append(e)
                ys += t["rows"]
            groups.append((members, xs, y0, ys - y0, by[members[0]]["cols"]))
            xs += by[members[0]]["cols"]
            plans.append(xksv_gpu.Plan(entries))
    t_idx = time.perf_counter()
    for pl in plans:
        if pl.index(payload, h):
            raise RuntimeError("xksv_plan_index failed")
    index_s = time.perf_counter() - t_idx
    # batch >= 4 runs on the tensor cores after decoding each plan's weights
    # into a BF16 scratch: one scratch, sized for the largest plan, is lent to
    # every plan (their calls are serialised on one stream)
    need = max(pl.scratch_bytes() for pl in plans)
    scratch = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
    for pl in plans:
        if pl.scratch_bytes():
            pl.set_scratch(scratch.data_ptr(), scratch.numel())
    res = {}
    g = torch.Generator(device=dev).manual_seed(5)
    peak = measured_peak()[0]
    for batch in (1, 4, 8, 16):
        x = torch.randn(xs, batch, generator=g, device=dev).to(torch.bfloat16).float()
        y = torch.empty(ys, batch, device=dev)

        def forward():
            for pl in plans:
                pl.gemm(payload, x, y, batch, h)
        with torch.cuda.stream(stream):
            forward()  # first call: the tensor-core path allocates its X^T buffers
        assert all(pl.status(h) == 0 for pl in plans)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            forward()
        steps = max(3, args.gemv_steps // 4)
        with torch.cuda.stream(stream):
            for _ in range(2):
                graph.replay()
            t = time_steps(graph.replay, steps, stream)
        assert all(pl.status(h) == 0 for pl in plans)
        ms = t / steps * 1e3
        # layer 0 down_proj against an FP32 matmul of its decoded weights
        members, x0, y0, nrows, cols = groups[3]
        td = by[members[0]]
        dplan = xksv_gpu.Plan(td["slabs"])
        w = torch.empty(td["rows"] * td["cols"] * 2, dtype=torch.uint8, device=dev)
        dplan.decode(payload, w, h)
        assert dplan.status(h) == 0
        dplan.close()
        W = w.view(torch.bfloat16).view(td["rows"], td["cols"]).float()
        ref = W @ (x[x0:x0 + cols] if batch < 4 else x[x0:x0 + cols].bfloat16().float())
        rel = float((y[y0:y0 + nrows] - ref).norm() / ref.norm())
        res[f"batch{batch}"] = dict(ms_per_forward=round(ms, 3), tok_per_s=round(batch * 1e3 / ms, 2),
                                    path="CUDA cores, FP32 x" if batch < 4 else "tcgen05, x in BF16",
                                    compressed_gbs=round(comp / (ms / 1e3) / 1e9, 1),
                                    frac_of_hbm=round(comp / (ms / 1e3) / 1e9 / peak, 4),
                                    tflops=round(2 * (raw // 2) * batch / (ms / 1e3) / 1e12, 2),
                                    rel_l2_layer0_down=rel)
        del graph
    line = dict(case="config4-gemv", config="configs[3] Llama-3-70B linears (80 layers), N(0,0.015) seed 3, "
                "dfloat11 + tile index, 1 GPU", compressed_bytes=comp, weights=raw // 2,
                index_build_s=round(index_s, 2), build_s=round(build_s, 1), plan_calls_per_forward=len(plans),
                shared_scratch_bytes=int(scratch.numel()),
                **res)
    print(json.dumps(line), flush=True)
    for pl in plans:
        pl.close()


def run_config5(args):
    """`--case config5`: prints config5()'s line."""
    world, rank, dev, stream = _case_setup()
    line = config5(args, dev, stream, world, rank)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def config5(args, dev, stream, world, rank):
    """The adversarial exponent mix of BASELINE configs[4]: 64 tensors of
    8192x8192 BF16 from seed 4 -- 32 Student-t(3) x 0.02, 16 N(0, 1e-4), 16
    uniform 16-bit patterns (raw-fallback slabs) -- encoded on the GPU in both
    codecs and decoded whole (one plan per codec), bit-exact against the
    source; tensors split over the ranks (tensor i on rank i % N: strong
    scaling)."""
    import torch
    import xksv_gpu
    h = stream.cuda_stream
    n = 8192
    torch.manual_seed(4)
    torch.cuda.manual_seed(4)
    srcs, names = [], []
    for i in range(64):
        if i < 32:  # Student-t(3): z / sqrt(chi2_3 / 3), chi2_3 = 2 * Gamma(1.5)
            z = torch.randn(n, n, device=dev)
            chi2 = 2.0 * torch._standard_gamma(torch.full((n, n), 1.5, device=dev))
            w = (z / torch.sqrt(chi2 / 3.0) * 0.02).to(torch.bfloat16)
            kind = "student3"
        elif i < 48:
            w = (torch.randn(n, n, device=dev) * 1e-4).to(torch.bfloat16)
            kind = "normal1e-4"
        else:
            w = torch.randint(-32768, 32768, (n, n), device=dev, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
            kind = "uniform16"
        if i % world == rank:
            srcs.append(w)
            names.append(f"t{i}.{kind}")
        else:
            del w
    raw_bytes = sum(s.numel() * 2 for s in srcs)
    results = {}
    for codec, cname in ((1, "bf16-huffman-tile16"), (2, "bf16-huffman-parallel32")):
        specs = [(nm, n, n, (lambda s=s: s)) for nm, s in zip(names, srcs)]
        payload, info, comp, raw = device_archive(specs, codec, dev, stream, 1.02)
        entries, base = [], 0
        for t in info:
            for s in t["slabs"]:
                e = dict(s)
                e["dst_offset"] = base + s["dst_offset"]
                entries.append(e)
            base += t["rows"] * t["cols"] * 2
        plan = xksv_gpu.Plan(entries)
        out = torch.empty(base, dtype=torch.uint8, device=dev)
        with torch.cuda.stream(stream):
            plan.decode(payload, out, h)
        if plan.status(h):
            raise RuntimeError("decode reported a slab error")
        exact = all(torch.equal(out[k * n * n * 2:(k + 1) * n * n * 2].view(torch.int16),
                                s.view(torch.int16).reshape(-1)) for k, s in enumerate(srcs))
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                plan.decode(payload, out, h)
            stream.synchronize()
            if world > 1:
                torch.distributed.barrier()
            t = time_steps(lambda: plan.decode(payload, out, h), args.steps, stream)
        t = _max_over_ranks(t, world, dev)
        ms = t / args.steps * 1e3
        kinds = {}
        for e in entries:
            kinds[e["codec"]] = kinds.get(e["codec"], 0) + 1
        peak = measured_peak()[0]
        results[cname] = dict(ms_per_step=round(ms, 3), value=round(world * raw / (ms / 1e3) / 1e9, 1),
                              per_gpu_out_gbs=round(raw / (ms / 1e3) / 1e9, 1), compressed_bytes=comp,
                              ratio=round(comp / raw, 4), slabs_by_codec=kinds,
                              roofline_frac=round((raw + comp) / (ms / 1e3) / 1e9 / peak, 4),
                              bit_exact=exact, status_errors=plan.status(h))
        plan.close()
        del payload, out
        torch.cuda.empty_cache()
    line = dict(case="config5", config="configs[4] 64 x 8192x8192 BF16, seed 4: 32 Student-t(3)*0.02, "
                "16 N(0,1e-4), 16 uniform 16-bit", scaling="strong", n_gpus=world, steps=args.steps,
                per_rank_out_bytes=raw_bytes, unit="GB/s BF16 out (all ranks)", **results)
    del srcs
    torch.cuda.empty_cache()
    return line


def run_runtime(args):
    """`--case runtime`: the archive path around the kernels on the config-2
    checkpoint.  Writes the seeded checkpoint as Safetensors to a temporary
    directory, compiles it with the GPU encoder and with the host encoder (all
    cores; byte-identical outputs checked), then loads the archive as the
    runtime does: upload of the block region to HBM, device verification
    (every block decoded, block digests on the device, tensor digests on host
    threads), and whole-checkpoint decode into tensors (one plan).  Wall
    times with the device synchronised; the file is in the page cache."""
    import filecmp
    import shutil
    import tempfile

    import numpy as np
    import torch
    import xksv_compile as xc
    import xksv_runtime as rt

    dev = "cuda:0"
    torch.cuda.set_device(0)
    tmp = Path(tempfile.mkdtemp(prefix="xksv-bench-"))
    try:
        gen = torch.Generator(device=dev).manual_seed(1)
        header, parts, pos = {}, [], 0
        for name, rows, cols, kind in llama_tensors(**CONFIG2):
            if kind == "norm":
                t, shape = torch.ones(cols, dtype=torch.bfloat16, device=dev), [cols]
            else:
                t = (torch.randn(rows, cols, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
                shape = [rows, cols]
            b = t.view(torch.int16).cpu().numpy()
            header[name] = dict(dtype="BF16", shape=shape, data_offsets=[pos, pos + b.nbytes])
            parts.append(b)
            pos += b.nbytes
        h = json.dumps(header, separators=(",", ":")).encode()
        h += b" " * (-len(h) % 8)
        src = tmp / "ckpt"
        src.mkdir()
        with open(src / "model.safetensors", "wb") as f:
            f.write(len(h).to_bytes(8, "little") + h)
            for b in parts:
                f.write(memoryview(b))
        del parts
        raw_bytes = pos

        def timed(fn):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            r = fn()
            torch.cuda.synchronize()
            return r, time.perf_counter() - t0

        arch = tmp / "gpu.xksv"
        _, t_gpu = timed(lambda: xc.compile_checkpoint(src, arch, "dfloat11-parallel", encoder="gpu",
                                                        device=dev, verify=False))
        _, t_host = timed(lambda: xc.compile_checkpoint(src, tmp / "host.xksv", "dfloat11-parallel",
                                                         encoder="host", verify=False))
        identical = filecmp.cmp(arch, tmp / "host.xksv", shallow=False)
        (tmp / "host.xksv").unlink()
        a, t_up = timed(lambda: rt.ResidentArchive(arch, dev))
        _, t_ver = timed(a.verify)
        a.decode_all()  # first call: allocator growth
        dec = []
        for _ in range(max(1, args.steps)):
            out, t = timed(a.decode_all)
            dec.append(t)
            del out
        t_dec = statistics.median(dec)
        # the reference's caller pattern (python/runtime.py:89-99) through this
        # library's legacy entry points: per block a file read, a ctypes
        # string buffer and one blocking decode call, on a sample of blocks
        import xksv_gpu
        lib = xksv_gpu.load()
        blocks = [(t, b) for t in a.tensors.values() for b in t["blocks"]]
        sample = blocks[:1000]
        scratch = torch.empty(1 << 21, dtype=torch.uint8, device=dev)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with open(arch, "rb") as f:
            for t, b in sample:
                f.seek(b["offset"])
                data = f.read(b["size"])
                if b["codec"] == "raw":
                    scratch[:len(data)].copy_(torch.frombuffer(bytearray(data), dtype=torch.uint8))
                    continue
                buf = ctypes.create_string_buffer(data)
                rc = (lib.xksv_cuda_decode_parallel(buf, len(data), scratch.data_ptr())
                      if b["codec"] == "bf16-huffman-parallel32" else
                      lib.xksv_cuda_decode(buf, len(data), b["rows"], b["cols"], scratch.data_ptr()))
                assert rc == 0
        torch.cuda.synchronize()
        t_legacy = (time.perf_counter() - t0) / len(sample) * len(blocks)
        arch_bytes = arch.stat().st_size
        line = dict(case="runtime", config="configs[1] Llama-1.1B shape, dfloat11-parallel",
                    checkpoint_bytes=raw_bytes, archive_bytes=arch_bytes, blocks=sum(
                        len(t["blocks"]) for t in a.tensors.values()),
                    compile_gpu_s=round(t_gpu, 3), compile_gpu_gbs=round(raw_bytes / t_gpu / 1e9, 2),
                    compile_host_s=round(t_host, 3), compile_host_threads=os.cpu_count(),
                    compile_outputs_identical=identical,
                    upload_s=round(t_up, 3), upload_gbs=round(arch_bytes / t_up / 1e9, 2),
                    verify_s=round(t_ver, 3), verify_gbs=round(raw_bytes / t_ver / 1e9, 2),
                    decode_all_ms=round(t_dec * 1e3, 2), decode_all_gbs=round(raw_bytes / t_dec / 1e9, 1),
                    load_s=round(t_up + t_ver + t_dec, 3),
                    per_block_abi_decode_s_est=round(t_legacy, 2),
                    per_block_abi_sample_blocks=len(sample))
        a.close()
        print(json.dumps(line), flush=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def tp_gemv(args, dev, stream, threads, rank, world):
    """Tensor-parallel batch-1 fused GEMV over every linear of the
    Llama-3-8B-shaped model: each rank encodes and holds only its row shard
    of every weight (whole 16-row slabs), and per layer runs four fused plan
    GEMVs (qkv, o, gate+up, down) each followed by one NCCL all-gather of the
    output shards (xksv_tp_gemm).  Timed on the device, max over ranks."""
    import torch
    import torch.distributed as dist
    import xksv_gpu

    cfg = CONFIG3
    tensors = [t for t in llama_tensors(**cfg) if t[3] == "w" and ("layers." in t[0])]
    payload, slabs, _, info = build_archive(
        tensors, 1, 0.02, 2, dev, threads, row_range=lambda rows: xksv_gpu.shard_rows(rows, world, rank))
    d_payload = torch.from_numpy(payload).to(dev)
    name_to = {i["name"]: i for i in info}
    comm = xksv_gpu.TPComm(rank, world)
    groups, xs = [], 0
    for L in range(cfg["layers"]):
        p = f"model.layers.{L}."
        for members in ([p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight"],
                        [p + "self_attn.o_proj.weight"],
                        [p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"],
                        [p + "mlp.down_proj.weight"]):
            cols = name_to[members[0]]["cols"]
            entries, yl = [], 0
            for m in members:
                t = name_to[m]
                for sl in slabs[t["first"]:t["first"] + t["n"]]:
                    e = dict(sl)
                    e["dst_offset"] = yl + (sl["dst_offset"] - t["dst"]) // (2 * t["cols"])
                    e["x_offset"] = xs
                    entries.append(e)
                yl += t["rows"]
            plan = xksv_gpu.Plan(entries)
            if plan.index(d_payload, stream.cuda_stream):
                raise RuntimeError("xksv_plan_index failed")
            groups.append(dict(plan=plan, rows=yl, y=torch.empty(yl, device=dev),
                               yfull=torch.empty(world * yl, device=dev)))
            xs += cols
    x = torch.randn(xs, generator=torch.Generator(device=dev).manual_seed(3), device=dev).to(torch.bfloat16).float()
    h = stream.cuda_stream

    def forward():
        for g in groups:
            comm.gemm(g["plan"], d_payload, x, g["y"].data_ptr(), g["rows"],
                      g["yfull"].data_ptr(), 1, h)

    with torch.cuda.stream(stream):
        for _ in range(3):
            forward()
    stream.synchronize()
    bad = sum(g["plan"].status(h) for g in groups)
    dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        t = time_steps(forward, args.gemv_steps, stream)
    bad += sum(g["plan"].status(h) for g in groups)
    tt = torch.tensor([t], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t = float(tt.item())
    # the all-gather placed every rank's shard at its rank's block
    g0 = groups[-1]
    own = bool(torch.equal(g0["yfull"][rank * g0["rows"]:(rank + 1) * g0["rows"]], g0["y"]))
    ms = t / args.gemv_steps * 1e3

    # the same plans without any gather: the all-gather's share of a token
    def forward_local():
        for g in groups:
            g["plan"].gemm(d_payload, x, g["y"], 1, h)

    with torch.cuda.stream(stream):
        for _ in range(3):
            forward_local()
    stream.synchronize()
    bad += sum(g["plan"].status(h) for g in groups)
    dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        tl = time_steps(forward_local, args.gemv_steps, stream)
    tt = torch.tensor([tl], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms_l = float(tt.item()) / args.gemv_steps * 1e3

    # fused all-gather: the GEMV epilogue stores rows into every rank's gathered
    # buffer over NVLink, then a bounded flag wait (xksv_tp_fused_gemm)
    fused = xksv_gpu.TPFused(rank, world, max(g["rows"] for g in groups), 1)

    def forward_fused():
        for g in groups:
            g["fused_y"] = fused.gemm(g["plan"], d_payload, x, g["rows"], 1, h)

    with torch.cuda.stream(stream):
        for _ in range(3):
            forward_fused()
    stream.synchronize()
    bad += sum(g["plan"].status(h) for g in groups)
    dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        tf = time_steps(forward_fused, args.gemv_steps, stream)
    bad += sum(g["plan"].status(h) for g in groups)
    tt = torch.tensor([tf], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms_f = float(tt.item()) / args.gemv_steps * 1e3
    # same gathered rows as the NCCL path (last group, this rank's block)
    chk = torch.empty(world * g0["rows"], device=dev)
    fused.gemm(g0["plan"], d_payload, x, g0["rows"], 1, h, chk)
    stream.synchronize()
    fused_match = bool(torch.allclose(chk, g0["yfull"], rtol=1e-5, atol=1e-6))
    torch.cuda.synchronize()
    dist.barrier()
    fused.close()
    for g in groups:
        g["plan"].close()
    comm.close()
    return dict(metric="TP fused-GEMV tok/s Llama-8B b=1", value=round(1e3 / ms_f, 2), unit="tok/s",
                ms_per_token=round(ms_f, 4), n_gpus=world, compressed_bytes_per_rank=int(payload.nbytes),
                launches_per_token=2 * len(groups), status_errors=int(bad), matches_nccl_path=fused_match,
                nccl_allgather=dict(value=round(1e3 / ms, 2), ms_per_token=round(ms, 4),
                                    own_shard_gathered=own, allgather_share=round(1 - ms_l / ms, 3)),
                local_gemv_ms_per_token=round(ms_l, 4), allgather_share=round(1 - ms_l / ms_f, 3),
                note="rows sharded per GPU in whole slabs; value: xksv_tp_fused_gemm (GEMV epilogue stores "
                     "rows into every rank's buffer over NVLink + flag wait); nccl_allgather: xksv_tp_gemm "
                     "(plan GEMV + ncclAllGather); local_gemv_ms_per_token: the same plans with no gather "
                     "(max over ranks); allgather_share = 1 - local / path")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU baseline leg: seconds of reference decode (half on 1 thread, half on all)")
    ap.add_argument("--warmup-cpu", type=int, default=0)
    ap.add_argument("--gemv-steps", type=int, default=20)
    ap.add_argument("--no-gemv", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the configs[3] and configs[4] keys")
    ap.add_argument("--batch", type=int, default=1, help="batch columns of X in gemv- cases")
    ap.add_argument("--route", default="auto", choices=("auto", "scratch", "fused"),
                    help="tensor-core GEMM route of gemv- cases at batch >= 4 (xksv_plan_set_gemm_route)")
    ap.add_argument("--case", default=None,
                    help="CODEC:ROWSxCOLS:SLABS small decode workload (profiling), e.g. parallel:16x2048:2048; "
                         "gemv-serial:16x4096:1024 runs the indexed batch-1 GEMV instead")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    # stdout carries the JSON line(s) alone: Python's prints keep the real
    # stdout, while file descriptor 1, where native libraries (NCCL's version
    # and debug lines among them) write, goes to stderr
    sys.stdout.flush()
    real_stdout = os.dup(1)
    os.dup2(2, 1)
    sys.stdout = os.fdopen(real_stdout, "w", buffering=1)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # NCCL's init lines (ranks, transports, NVLS) on record, on stderr; set
        # before torch loads NCCL, which reads it once
        os.environ.setdefault("NCCL_DEBUG", "INFO")
    named = {"runtime": run_runtime, "config4-decode": run_config4_decode,
             "config4-gemv": run_config4_gemv, "config5": run_config5}
    if args.case in named:
        named[args.case](args)
        return
    if args.case:
        run_case(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    import xksv_gpu

    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device(dev))
    xksv_gpu.load()
    threads = host_threads(world)
    tensors = llama_tensors(**CONFIG2)
    payload, slabs, out_bytes, _ = build_archive(tensors, 2, 0.02, 1, dev, threads)
    comp_bytes = payload.nbytes
    n_par = sum(1 for s in slabs if s["codec"] == 2)
    n_raw = sum(1 for s in slabs if s["codec"] == 0)
    par_comp = sum(s["src_size"] for s in slabs if s["codec"] == 2)
    par_out = sum(s["rows"] * s["cols"] * 2 for s in slabs if s["codec"] == 2)

    d_payload = torch.from_numpy(payload).to(dev)
    d_out = torch.empty(out_bytes, dtype=torch.uint8, device=dev)
    plan = xksv_gpu.Plan(slabs)
    par_plan = xksv_gpu.Plan([s for s in slabs if s["codec"] == 2])
    stream = torch.cuda.Stream(device=dev)
    h = stream.cuda_stream

    def step():
        plan.decode(d_payload, d_out, h)

    # correctness of the decoded checkpoint: every slab's bytes against the
    # BF16 source regenerated with the same seed
    with torch.cuda.stream(stream):
        step()
    assert plan.status(h) == 0, "decode reported a slab error"
    gen = torch.Generator(device=dev).manual_seed(1)
    checked = 0
    for name, rows, cols, kind in tensors:
        ref = (torch.ones(rows, cols, dtype=torch.bfloat16, device=dev) if kind == "norm" else
               (torch.randn(rows, cols, generator=gen, device=dev) * 0.02).to(torch.bfloat16))
        seg = d_out[checked:checked + rows * cols * 2]
        assert torch.equal(seg, ref.view(torch.uint8).reshape(-1)), f"decode mismatch in {name}"
        checked += rows * cols * 2
    assert checked == out_bytes

    with ClockSampler(local) as clk:
        clk.mark()
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")
        t = time_steps(step, args.steps, stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    assert plan.status(h) == 0
    launches = plan.launches() * args.steps
    if world > 1:
        tt = torch.tensor([t], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
        dist.barrier()
    value = world * out_bytes * args.steps / t / 1e9

    # dominant kernel alone (the parallel-codec decode), for the roofline
    with torch.cuda.stream(stream):
        for _ in range(3):
            par_plan.decode(d_payload, d_out, h)
    tk = time_steps(lambda: par_plan.decode(d_payload, d_out, h), args.steps, stream)
    assert par_plan.status(h) == 0
    kdur = tk / args.steps
    peak, peak_src = measured_peak()
    achieved = (par_comp + par_out) / kdur / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic_parallel_decode.json"
    if tf.exists():
        try:
            d = json.loads(tf.read_text())
            traffic = int(d["dram_bytes_per_byte_algorithmic"] * (par_comp + par_out))
        except Exception:
            traffic = None

    # integrity check on the device: SHA-256 of every decoded slab (the archive
    # index's per-block digests, src/verify.cpp:262), spot-checked on the host
    import hashlib
    d_dig = torch.zeros(32 * len(slabs), dtype=torch.uint8, device=dev)
    with torch.cuda.stream(stream):
        plan.decode(d_payload, d_out, h)
        plan.sha256(d_out, d_dig, h)
        ts = time_steps(lambda: plan.sha256(d_out, d_dig, h), 3, stream)
    assert plan.status(h) == 0
    dig = d_dig.cpu().numpy().tobytes()
    sha_ok = True
    for i in range(0, len(slabs), max(1, len(slabs) // 16)):
        s_ = slabs[i]
        n_ = s_["src_size"] if s_["codec"] == 0 else s_["rows"] * s_["cols"] * 2
        seg = d_out[s_["dst_offset"]:s_["dst_offset"] + n_].cpu().numpy().tobytes()
        sha_ok &= hashlib.sha256(seg).digest() == dig[32 * i:32 * i + 32]
    sha = dict(blocks=len(slabs), ms=round(ts / 3 * 1e3, 3), gbs=round(out_bytes * 3 / ts / 1e9, 1),
               host_spot_check=bool(sha_ok))

    # GPU encoder: the largest tensor of the checkpoint compiled on the device,
    # byte-compared with the host encoder's payload for the same tensor
    enc = None
    try:
        name, er, ec, _ = max(tensors, key=lambda t: t[1] * t[2])
        g2 = torch.Generator(device=dev).manual_seed(11)
        wt = (torch.randn(er, ec, generator=g2, device=dev) * 0.02).to(torch.bfloat16)
        with torch.cuda.stream(stream):
            dptr, nbytes_e, sl_e = xksv_gpu.cuda_pack_tensor(wt.data_ptr(), er, ec, 2, 0, h)
            xksv_gpu.free_device(dptr)
            t0 = time.perf_counter()
            dptr, nbytes_e, sl_e = xksv_gpu.cuda_pack_tensor(wt.data_ptr(), er, ec, 2, 0, h)
            te_enc = time.perf_counter() - t0
        hw = wt.view(torch.int16).cpu().numpy()
        hp, hs = xksv_gpu.host_pack_tensor(hw.ctypes.data, hw.nbytes, er, ec, 2, threads=threads)
        dpay = torch.empty(nbytes_e, dtype=torch.uint8, device=dev)
        cp = xksv_gpu.Plan([dict(src_offset=0, src_size=nbytes_e, rows=1, cols=1, dst_offset=0, codec=0)])
        cp.decode(dptr, dpay, h, payload_bytes=nbytes_e)
        same = cp.status(h) == 0 and sl_e == hs and bool(np.array_equal(dpay.cpu().numpy(), hp))
        cp.close()
        xksv_gpu.free_device(dptr)
        enc = dict(tensor=name, shape=[er, ec], codec="bf16-huffman-parallel32",
                   ms=round(te_enc * 1e3, 2), gbs=round(wt.numel() * 2 / te_enc / 1e9, 1),
                   identical_to_host_encoder=same,
                   note="wall time of one xksv_cuda_pack_tensor call (synchronous: kernels, host "
                        "offsets, allocation)")
        del wt
    except Exception as ex:  # reported, never silently replaced
        enc = dict(error=f"{type(ex).__name__}: {ex}")

    # end to end through the public API: pinned host payload -> device, decode,
    # status word back
    h_payload = torch.from_numpy(payload).pin_memory()

    def e2e_step():
        # xksv_plan_decode_host: the payload crosses PCIe in pieces while the
        # slabs of the pieces already landed decode
        plan.decode_host(h_payload.data_ptr(), payload.nbytes, d_payload, d_out, h)
        if plan.status(h):
            raise RuntimeError("decode error")

    with torch.cuda.stream(stream):
        for _ in range(2):
            e2e_step()
        te = time_steps(e2e_step, max(3, args.steps // 4), stream)
    e2e_steps = max(3, args.steps // 4)
    if world > 1:
        tt = torch.tensor([te], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        te = float(tt.item())
    e2e_val = world * out_bytes * e2e_steps / te / 1e9

    tp = None
    if not args.no_gemv and world > 1:
        del d_out
        torch.cuda.empty_cache()
        try:
            tp = tp_gemv(args, dev, stream, threads, rank, world)
        except Exception as ex:  # reported, never silently replaced
            tp = dict(error=f"{type(ex).__name__}: {ex}")
    gemv = None
    if not args.no_gemv and rank == 0 and world == 1:
        del d_out
        torch.cuda.empty_cache()
        try:
            gemv = fused_gemv(args, dev, stream, threads)
        except Exception as ex:  # reported, never silently replaced
            gemv = dict(error=f"{type(ex).__name__}: {ex}")

    # the other BASELINE configs measured in the same run (their own roofline
    # and bit-exact checks): configs[3] whole-model decode, configs[4] mix
    del d_payload, h_payload
    if "d_out" in locals():
        del d_out
    torch.cuda.empty_cache()
    c4 = c5 = None
    if not args.no_configs:
        try:
            c4 = config4_decode(args, dev, stream, world, rank)
        except Exception as ex:  # reported, never silently replaced
            c4 = dict(error=f"{type(ex).__name__}: {ex}")
        torch.cuda.empty_cache()
        try:
            c5 = config5(args, dev, stream, world, rank)
        except Exception as ex:  # reported, never silently replaced
            c5 = dict(error=f"{type(ex).__name__}: {ex}")
        torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline(args.cpu_seconds)

    clocks = clk.summary()
    if world > 1:
        allc = [None] * world
        dist.all_gather_object(allc, clocks)
        sm = [c["sm_mhz"] for c in allc if c["sm_mhz"]]
        clocks = dict(sm_mhz=statistics.median(sm) if sm else None,
                      sm_max_mhz=max((c["sm_max_mhz"] or 0) for c in allc) or None,
                      reasons=sorted(set(r for c in allc for r in c["reasons"])),
                      samples=sum(c["samples"] for c in allc))
    if rank == 0:
        line = dict(
            metric=METRIC, value=round(value, 2), unit="GB/s", n_gpus=world, per_gpu_gbs=round(value / world, 2),
            steps=args.steps, warmup=args.warmup, ms_per_step=round(t / args.steps * 1e3, 4), higher_is_better=True,
            scaling="weak", vs_baseline=None, dtype="bf16",
            data="synthetic: seeded BF16 N(0,0.02) Llama-1.1B-shaped weights, norms 1.0 (no checkpoint download)",
            config=workload_config(world),
            archive=dict(slabs=len(slabs), parallel_slabs=n_par, raw_slabs=n_raw, compressed_bytes=comp_bytes,
                         out_bytes=out_bytes, encoder="host (xksv_host_pack_tensor, byte-identical to the "
                                                      "reference encoder)"),
            roofline=dict(bound="hbm", achieved=round(achieved, 1), peak=peak, unit="GB/s",
                          frac=round(achieved / peak, 4), traffic=traffic,
                          kernel="parallel_slab_kernel<0> (decode)", peak_source=peak_src,
                          algorithmic_bytes_per_launch=par_comp + par_out,
                          launch_ms=round(kdur * 1e3, 4)),
            cpu_baseline=cpu,
            e2e=dict(value=round(e2e_val, 2), unit="GB/s", h2d_bytes_per_step=comp_bytes,
                     d2h_bytes_per_step=4, steps=e2e_steps,
                     path="pinned host payload -> xksv_plan_decode_host (8 copy pieces overlapped with "
                          "their slabs' decode) -> xksv_plan_status"),
            clocks=clocks, gpu_launches=launches, sha256_verify=sha, gpu_encoder=enc, fused_gemv=gemv,
            tp_fused_gemv=tp, config4_decode=c4, config5=c5)
        print(json.dumps(line), flush=True)
    plan.close()
    par_plan.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
