"""Archive compiler on this library's encoders: Safetensors checkpoint ->
.xksv archive, byte-identical to the reference's ``compile_model``
(python/xksv.py:197-300; fresh compiles, without its resume journal).

The reference encodes block by block on a CPU thread pool through
``xksv_pack`` / ``xksv_pack_parallel``.  Here each run of equal-width blocks
of a tensor is one call of ``xksv_cuda_pack_tensor`` (GPU: histograms,
Huffman lengths, canonical codes and bit packing in kernels) or of
``xksv_host_pack_tensor`` (all host cores), both byte-identical to the
reference's per-block encoder.  The block layout, the raw fallback, the
index fields and their order, the asset list and the JSON encoding follow
the reference, so the reference's own ``verify`` accepts the output and the
golden archives it compiled are reproduced byte for byte.
"""
import base64
import hashlib
import json
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

import xksv_gpu
from xksv_runtime import DTYPE_SIZES, HEADER, MAGIC, RAW_CHUNK, fail

MAX_HEADER = 100_000_000
# files copied into the archive as assets, in this order (python/xksv.py:248)
ASSET_NAMES = ("config.json", "generation_config.json", "tokenizer.json", "tokenizer_config.json",
               "vocab.json", "merges.txt", "special_tokens_map.json", "added_tokens.json",
               "chat_template.jinja", "tokenizer.model", "vocab.txt", "preprocessor_config.json",
               "processor_config.json", "video_preprocessor_config.json", "LICENSE", "NOTICE", "README.md")
CODEC_NAMES = {"dfloat11": "bf16-huffman-tile16", "dfloat11-parallel": "bf16-huffman-parallel32"}


class _StrictObjects:
    """object_pairs_hook / parse_constant of a JSON reader that refuses what
    Python's default reader lets through silently: a repeated key (the last
    one would win) and the NaN / Infinity literals.  The messages are the
    ones the reference compiler prints (python/xksv.py:30-40)."""

    @staticmethod
    def build(items):
        obj = dict(items)
        if len(obj) != len(items):
            seen = set()
            for key, _ in items:
                if key in seen:
                    fail(f"duplicate JSON key: {key}")
                seen.add(key)
        return obj

    @staticmethod
    def constant(_literal):
        fail("invalid JSON number")


def parse_json(data):
    """Strict JSON (bytes or str): repeated keys and NaN/Infinity rejected."""
    return json.loads(data, object_pairs_hook=_StrictObjects.build, parse_constant=_StrictObjects.constant)


# The index's role label of a tensor: the first rule whose substrings occur in
# the tensor name decides.  The labels and their precedence are part of the
# archive format (the reference's index lists them, python/xksv.py:43-57).
_ROLE_RULES = (
    (("embed_tokens", "word_embeddings"), "token_embedding"),
    (("lm_head", "output_projection"), "language_model_head"),
    (("visual", "vision"), "vision_component"),
    (("linear_attn",), "deltanet"),
    (("self_attn", ".attention."), "attention_parameter"),
    (("expert",), "moe_expert"),
    (("router",), "moe_router"),
    ((".mlp.", ".feed_forward."), "feed_forward_parameter"),
    (("norm",), "normalization_parameter"),
)
# linear-attention (DeltaNet) tensors are labelled by their part
_DELTANET_RULES = (
    (("conv",), "deltanet_convolution"),
    (("in_proj",), "deltanet_input_projection"),
    (("out_proj",), "deltanet_output_projection"),
)


def _first_rule(name, rules, default):
    return next((role for keys, role in rules if any(k in name for k in keys)), default)


def tensor_role(name):
    """The index's role label of a tensor name."""
    role = _first_rule(name, _ROLE_RULES, "other")
    return _first_rule(name, _DELTANET_RULES, "deltanet_state_parameter") if role == "deltanet" else role


def contiguous_strides(shape):
    out, stride = [], 1
    for dim in reversed(shape):
        out.append(stride)
        stride *= dim
    return list(reversed(out))


def _shard_files(path):
    """The checkpoint's shard files, and the shard index's tensor -> file map
    when a directory has a model.safetensors.index.json (else None)."""
    if not path.is_dir():
        return [path], None
    index_file = path / "model.safetensors.index.json"
    if not index_file.is_file():
        return sorted(path.glob("*.safetensors")), None
    weight_map = parse_json(index_file.read_bytes()).get("weight_map")
    plain_file = lambda v: isinstance(v, str) and Path(v).name == v and v.endswith(".safetensors")
    if not isinstance(weight_map, dict) or not all(plain_file(v) for v in weight_map.values()):
        fail("invalid shard index")
    return [path / name for name in sorted(set(weight_map.values()))], weight_map


def _shard_header(file):
    """(header bytes, data section bytes) of one Safetensors file: a u64
    little-endian header length, the JSON header, then the data."""
    if not file.is_file() or file.suffix != ".safetensors":
        fail(f"not a Safetensors file: {file}")
    total = file.stat().st_size
    with file.open("rb") as f:
        head = f.read(8)
        if len(head) < 8:
            fail(f"truncated header: {file}")
        (hlen,) = struct.unpack("<Q", head)
        if hlen > min(MAX_HEADER, total - 8):
            fail(f"invalid header length: {file}")
        return f.read(hlen), total - 8 - hlen


def _tensor_record(name, desc, data_bytes):
    """One header entry, validated: a known dtype, a shape of non-negative
    ints, [start, end) data offsets inside the data section whose length is
    exactly the shape's element count times the dtype's size."""
    if not isinstance(desc, dict):
        fail(f"invalid descriptor: {name}")
    dtype, shape, offsets = desc.get("dtype"), desc.get("shape"), desc.get("data_offsets")
    if dtype not in DTYPE_SIZES:
        fail(f"unsupported dtype {dtype} for {name}")
    if not isinstance(shape, list) or not all(type(d) is int and d >= 0 for d in shape):
        fail(f"invalid shape: {name}")
    if not (isinstance(offsets, list) and len(offsets) == 2 and all(type(o) is int for o in offsets)):
        fail(f"invalid offsets: {name}")
    start, end = offsets
    want = int(np.prod(shape, dtype=object)) * DTYPE_SIZES[dtype]
    if not 0 <= start <= end <= data_bytes or end - start != want:
        fail(f"invalid tensor extent: {name}")
    return dict(name=name, dtype=dtype, shape=shape, strides=contiguous_strides(shape),
                role=tensor_role(name), start=start, size=end - start)


def _check_tiling(file, tensors, data_bytes):
    """The non-empty tensors cover the data section back to back: no gap,
    no overlap, nothing after the last one."""
    expect = 0
    for t in sorted((t for t in tensors if t["size"]), key=lambda t: t["start"]):
        if t["start"] != expect:
            fail(f"overlapping or noncontiguous tensors in {file}")
        expect = t["start"] + t["size"]
    if expect != data_bytes:
        fail(f"unreferenced data in {file}")


def checkpoint(path):
    """Shards of a Safetensors checkpoint (a file, or a directory with an
    optional model.safetensors.index.json), every header entry validated and
    each shard's data section tiled exactly by its tensors; tensors listed in
    data order.  Error messages are the reference compiler's
    (python/xksv.py:83-135)."""
    files, weight_map = _shard_files(Path(path))
    if not files:
        fail("no Safetensors shards found")
    shards, seen = [], set()
    for file in files:
        header, data_bytes = _shard_header(file)
        entries = parse_json(header)
        if not isinstance(entries, dict):
            fail("invalid Safetensors header")
        tensors = []
        for name, desc in entries.items():
            if name == "__metadata__":
                continue
            if name in seen:
                fail(f"duplicate tensor: {name}")
            seen.add(name)
            tensors.append(_tensor_record(name, desc, data_bytes))
        _check_tiling(file, tensors, data_bytes)
        tensors.sort(key=lambda t: t["start"])
        shards.append(dict(name=file.name, path=str(file), header=base64.b64encode(header).decode("ascii"),
                           header_size=len(header), tensors=tensors))
    if weight_map is not None and weight_map != {t["name"]: s["name"] for s in shards for t in s["tensors"]}:
        fail("shard index does not match discovered tensor names and files")
    return shards


def block_layout(dtype, shape, size):
    """[(byte offset, bytes, rows, cols)] of a tensor's blocks: the
    compiler's split (python/xksv.py:262, 283-286; src/compile.cpp:449-479).
    rows == 0 marks a raw block of a non-BF16 tensor."""
    if dtype == "BF16":
        cols = shape[1] if len(shape) == 2 and shape[1] and shape[1] * 2 <= RAW_CHUNK else min(4096, size // 2)
    else:
        cols = 0
    out, pos, remaining = [], 0, size
    while remaining:
        rows = min(16, RAW_CHUNK // (cols * 2), remaining // (cols * 2)) if cols else 0
        if cols and not rows:
            cols = min(4096, remaining // 2)
            rows = 1
        length = rows * cols * 2 if cols else min(remaining, RAW_CHUNK)
        out.append((pos, length, rows, cols))
        pos += length
        remaining -= length
    return out


def coded_runs(layout):
    """Consecutive BF16 blocks of equal width as (first byte, rows, cols, n)."""
    runs = []
    for off, length, rows, cols in layout:
        if not rows:
            continue
        if runs and runs[-1][2] == cols and runs[-1][0] + runs[-1][1] * cols * 2 == off:
            r = runs[-1]
            runs[-1] = (r[0], r[1] + rows, cols, r[3] + 1)
        else:
            runs.append((off, rows, cols, 1))
    return runs


class _DevicePayload:
    """Zero-copy torch view of library-allocated device bytes."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class ArchiveWriter:
    """Writes an archive in the reference's layout: header, assets, blocks in
    tensor order, JSON index.  ``encoder`` is "gpu" (xksv_cuda_pack_tensor on
    `device`) or "host" (xksv_host_pack_tensor on all cores)."""

    def __init__(self, output, codec_preference="dfloat11", encoder="gpu", device="cuda:0", threads=0,
                 tuning=None):
        if codec_preference not in CODEC_NAMES and codec_preference != "autotune":
            fail(f"unsupported codec preference: {codec_preference}")
        if encoder not in ("gpu", "host"):
            fail(f"unknown encoder: {encoder}")
        self.output = Path(output).absolute()
        if self.output.exists():
            fail("output already exists")
        self.partial = self.output.with_name(self.output.name + ".partial")
        if self.partial.exists():
            fail("partial compilation exists; choose another output")
        # autotune: both codecs are encoded and the tuner picks per block
        # (python/xksv.py:206-208, 269, 274-275)
        self.tuner = None
        if codec_preference == "autotune":
            import xksv_tune
            self.tuner = xksv_tune.GpuTuner(tuning, device)
            self.codec_name, self.codec = None, None
        else:
            self.codec_name = CODEC_NAMES[codec_preference]
            self.codec = xksv_gpu.CODEC_BY_NAME[self.codec_name]
        self.encoder, self.device, self.threads = encoder, device, threads
        self.lib = xksv_gpu.load()
        self.pool = ThreadPoolExecutor(max_workers=max(2, min(32, os.cpu_count() or 2)))
        # tensors whose digest is still running keep their bytes alive: bound them
        self._pending, self._pending_bytes, self._max_pending_bytes = [], 0, 4 << 30
        fd = os.open(self.partial, os.O_CREAT | os.O_EXCL | os.O_RDWR, 0o600)
        self.f = os.fdopen(fd, "w+b")
        self.f.write(HEADER.pack(MAGIC, 0))
        self.index = dict(version=1, format="safetensors", codec_preference=codec_preference, shards=[],
                          assets=[])
        if self.tuner:
            self.index["tuning"] = self.tuner.profile

    def add_asset(self, name, data):
        self.index["assets"].append(dict(name=name, offset=self.f.tell(), size=len(data),
                                         sha256=hashlib.sha256(data).hexdigest()))
        self.f.write(data)

    def begin_shard(self, name, header_b64, source_sha256):
        """source_sha256: hex digest, or a Future of one (resolved at close)."""
        self.index["shards"].append(dict(name=name, header=header_b64, source_sha256=source_sha256, tensors=[]))

    def _encode(self, raw, off, rows, cols, codec):
        """(payload bytes, slab dicts) of rows x cols BF16 at raw[off:]."""
        nbytes = rows * cols * 2
        if self.encoder == "host":
            ptr = raw.ctypes.data + off
            payload, slabs = xksv_gpu.host_pack_tensor(ptr, nbytes, rows, cols, codec, self.threads,
                                                       0, lib=self.lib)
            return payload, slabs
        import torch
        d = torch.from_numpy(raw[off:off + nbytes]).to(self.device)
        with torch.cuda.device(d.device):
            stream = torch.cuda.current_stream().cuda_stream
            ptr, n, slabs = xksv_gpu.cuda_pack_tensor(d.data_ptr(), rows, cols, codec, 0, stream,
                                                      lib=self.lib)
            try:
                payload = torch.as_tensor(_DevicePayload(ptr, n), device=d.device).cpu().numpy() if n else \
                    np.zeros(0, np.uint8)
            finally:
                xksv_gpu.free_device(ptr, lib=self.lib)
        return payload, slabs

    def add_tensor(self, desc, raw, shard=-1):
        """desc: name, dtype, shape, strides, role, start, size (the checkpoint
        descriptor); raw: the tensor's bytes (bytes or a uint8 numpy array);
        shard: position of the shard entry that lists the tensor."""
        raw = np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw
        if raw.size != desc["size"]:
            fail(f"tensor bytes differ from descriptor: {desc['name']}")
        t = dict(desc)
        t["blocks"] = []
        layout = block_layout(desc["dtype"], desc["shape"], desc["size"])
        # digests on host threads while the blocks encode
        tensor_digest = self.pool.submit(lambda: hashlib.sha256(raw).hexdigest())
        block_digests = [self.pool.submit(lambda o=o, n=n: hashlib.sha256(raw[o:o + n]).hexdigest())
                         for o, n, _, _ in layout]
        codecs = ([xksv_gpu.CODEC_TILE16, xksv_gpu.CODEC_PARALLEL32] if self.tuner else [self.codec])
        encoded = {c: {} for c in codecs}
        for off, rows, cols, nblocks in coded_runs(layout):
            for c in codecs:
                payload, slabs = self._encode(raw, off, rows, cols, c)
                if len(slabs) != nblocks:
                    fail(f"encoder block split differs from the compiler's: {desc['name']}")
                for s in slabs:
                    encoded[c][off + s["dst_offset"]] = (s, payload)

        def blob(c, off, rows, cols, length):
            """The block's encoding under codec c, or None when the encoding
            is not smaller than the raw bytes (the encoder's raw fallback)."""
            s, payload = encoded[c].get(off, (None, None))
            if s is None or s["rows"] != rows or s["cols"] != cols:
                fail(f"encoder block split differs from the compiler's: {desc['name']}")
            if s["codec"] == xksv_gpu.CODEC_RAW:
                return None
            return payload[s["src_offset"]:s["src_offset"] + s["src_size"]]

        for i, (off, length, rows, cols) in enumerate(layout):
            data, codec = raw[off:off + length], "raw"
            if rows and self.tuner:
                ser = blob(xksv_gpu.CODEC_TILE16, off, rows, cols, length)
                par = blob(xksv_gpu.CODEC_PARALLEL32, off, rows, cols, length)
                codec, data = self.tuner.select(data if ser is None else ser, data if par is None else par,
                                                data, rows, cols)
            elif rows:
                enc = blob(self.codec, off, rows, cols, length)
                if enc is not None:
                    data, codec = enc, self.codec_name
            t["blocks"].append(dict(offset=self.f.tell(), size=int(data.size), raw_size=length, codec=codec,
                                    rows=rows if codec != "raw" else 0, cols=cols if codec != "raw" else 0,
                                    sha256=block_digests[i].result()))
            self.f.write(memoryview(data))
        # the tensor digest is one sequential pass: collect it later, keeping
        # a bounded number of tensors in flight
        self._pending.append((t, tensor_digest, raw.size))
        self._pending_bytes += raw.size
        while len(self._pending) > 1 and self._pending_bytes > self._max_pending_bytes:
            self._settle_one()
        self.index["shards"][shard]["tensors"].append(t)
        return t

    def _settle_one(self):
        t, fut, n = self._pending.pop(0)
        t["sha256"] = fut.result()
        self._pending_bytes -= n

    def close(self):
        """Writes the index and the header and moves the file into place."""
        while self._pending:
            self._settle_one()
        for sh in self.index["shards"]:
            if hasattr(sh["source_sha256"], "result"):
                sh["source_sha256"] = sh["source_sha256"].result()
        offset = self.f.tell()
        self.f.write(json.dumps(self.index, separators=(",", ":"), ensure_ascii=False).encode())
        self.f.seek(0)
        self.f.write(HEADER.pack(MAGIC, offset))
        self.f.flush()
        os.fsync(self.f.fileno())
        self.f.close()
        self.pool.shutdown()
        os.link(self.partial, self.output)
        os.unlink(self.partial)
        return self.output

    def abort(self):
        self.f.close()
        self.pool.shutdown()
        if self.partial.exists():
            self.partial.unlink()


def compile_checkpoint(source, output, codec_preference="dfloat11", encoder="gpu", device="cuda:0", verify=True,
                       tuning=None):
    """``compile_model(source, output, codec_preference=...)`` on this
    library's encoders; codec_preference "dfloat11", "dfloat11-parallel" or
    "autotune" (GpuTuner per block; `tuning` resumes a saved profile).  With
    `verify`, the archive is then loaded and checked on the device (every
    block decoded, every SHA-256 compared)."""
    shards = checkpoint(source)
    output = Path(output).absolute()
    for s in shards:
        if Path(s["path"]).resolve() == output.resolve():
            fail("output would overwrite source")
    w = ArchiveWriter(output, codec_preference, encoder, device, tuning=tuning)
    try:
        for s in shards:
            w.begin_shard(s["name"], s["header"], w.pool.submit(_sha_file, s["path"]))
        if Path(source).is_dir():
            for name in ASSET_NAMES:
                p = Path(source) / name
                if p.is_file():
                    if p.stat().st_size > 100_000_000:
                        fail(f"asset too large: {name}")
                    w.add_asset(name, p.read_bytes())
        # the next tensor is read while the current one encodes
        jobs = [(i, s, t) for i, s in enumerate(shards) for t in s["tensors"]]
        with ThreadPoolExecutor(max_workers=1) as reader:
            nxt = reader.submit(_read_tensor, *jobs[0][1:]) if jobs else None
            for k, (i, s, t) in enumerate(jobs):
                raw = nxt.result()
                nxt = reader.submit(_read_tensor, *jobs[k + 1][1:]) if k + 1 < len(jobs) else None
                w.add_tensor(t, raw, shard=i)
    except BaseException:
        w.abort()
        raise
    path = w.close()
    if verify:
        import xksv_runtime
        a = xksv_runtime.ResidentArchive(path, device)
        a.verify()
        a.close()
    return path


def _read_tensor(shard, t):
    raw = np.empty(t["size"], dtype=np.uint8)
    with open(shard["path"], "rb") as f:
        f.seek(8 + shard["header_size"] + t["start"])
        if t["size"] and f.readinto(memoryview(raw)) != t["size"]:
            fail("unexpected end of file")
    return raw


def _sha_file(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(1 << 24)
            if not b:
                return h.hexdigest()
            h.update(b)
