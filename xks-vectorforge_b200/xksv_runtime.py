"""Device-resident archive runtime: the callers of the decode and fused-GEMV
path, moved onto the batched plan interface.

The reference's callers (python/runtime.py:31-117 ``load_archive`` with
``--gpu-decode``; :248-287 ``install_fused_gemv``) re-read each block from the
file, stage it through ``ctypes.create_string_buffer`` and make one blocking
ABI call per block, on every load and on every token.  Here an archive's block
region is uploaded to HBM once (``ResidentArchive``); a whole checkpoint
decodes in one plan launch; integrity is checked on the device against the
index's SHA-256 digests (replacing the CPU ``xksv.verify`` that precedes every
load, python/xksv.py:311-386); and each fused linear layer is one resident
plan whose call enqueues on the caller's stream, for batch 1 (CUDA-core GEMV)
and batch > 1 (tensor-core GEMM) alike, where the reference falls back to a
decoded-weight ``F.linear`` (python/runtime.py:265-266).

Archive format (python/xksv.py:18-19, 302-308; written by compile_model,
:197-300): ``b"XKSV\\x00\\x01\\r\\n"``, a little-endian u64 index offset, the
assets and blocks back to back from byte 16, then the JSON index at the
offset.  The index lists shards, each with tensors (name, dtype, shape, start,
size, sha256) and their blocks (offset, size, raw_size, codec, rows, cols,
sha256) in tensor byte order.  Errors raise ``ArchiveError`` (a ValueError,
like the reference's ``fail``) with the reference's messages.
"""
import hashlib
import json
import os
import struct
import tempfile
from pathlib import Path

import xksv_gpu

MAGIC = b"XKSV\x00\x01\r\n"
HEADER = struct.Struct("<8sQ")
MAX_INDEX = 1_000_000_000
RAW_CHUNK = 1 << 20
CODED = ("bf16-huffman-tile16", "bf16-huffman-parallel32")
CODECS = ("raw",) + CODED
# bytes per element (python/xksv.py:20)
DTYPE_SIZES = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E4M3": 1, "F8_E5M2": 1, "I16": 2, "U16": 2, "F16": 2,
               "BF16": 2, "I32": 4, "U32": 4, "F32": 4, "I64": 8, "U64": 8, "F64": 8}
TENSOR_ALIGN = 256  # byte alignment of each decoded tensor inside a flat buffer


class ArchiveError(ValueError):
    pass


def fail(msg):
    raise ArchiveError(msg)


def torch_dtype(name):
    import torch
    table = {"BOOL": torch.bool, "U8": torch.uint8, "I8": torch.int8, "I16": torch.int16,
             "U16": torch.uint16, "F16": torch.float16, "BF16": torch.bfloat16, "I32": torch.int32,
             "U32": torch.uint32, "F32": torch.float32, "I64": torch.int64, "U64": torch.uint64,
             "F64": torch.float64, "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2}
    if name not in table:
        fail(f"backend cannot load dtype {name}")
    return table[name]


# ------------------------------------------------------------------ index
def load_index(f):
    """(index, data limit) of an open archive; python/xksv.py:302-308."""
    size = os.fstat(f.fileno()).st_size
    head = f.read(HEADER.size)
    if len(head) != HEADER.size:
        fail("unexpected end of file")
    magic, offset = HEADER.unpack(head)
    if magic != MAGIC or offset < HEADER.size or offset > size or size - offset > MAX_INDEX:
        fail("invalid archive header")
    f.seek(offset)
    try:
        index = json.loads(f.read(size - offset))
    except (ValueError, UnicodeDecodeError):
        fail("invalid JSON")
    if not isinstance(index, dict) or index.get("version") != 1 or index.get("format") != "safetensors":
        fail("unsupported archive")
    return index, offset


def _is_int(v):
    return type(v) is int


def check_index(index, limit):
    """The metadata checks of the reference's verify (python/xksv.py:316-356,
    381-385, the ``metadata_only`` branch): names, descriptors, block extents
    and codecs, and that assets and blocks tile [16, limit) exactly.  Returns
    {name: tensor} in archive order."""
    spans, tensors, assets = [], {}, set()
    for a in index.get("assets", []):
        name, off, n = a.get("name"), a.get("offset"), a.get("size")
        if (not isinstance(name, str) or Path(name).name != name or name in assets or not _is_int(off)
                or not _is_int(n) or off < HEADER.size or n < 0 or n > 100_000_000 or off > limit
                or n > limit - off):
            fail("invalid asset")
        assets.add(name)
        spans.append((off, off + n))
    shards = set()
    for shard in index.get("shards", []):
        if shard.get("name") in shards or Path(str(shard.get("name"))).name != shard.get("name"):
            fail("invalid archive shard name")
        shards.add(shard["name"])
        for t in shard.get("tensors", []):
            if t.get("name") in tensors:
                fail("duplicate archive tensor")
            shape, dtype = t.get("shape"), t.get("dtype")
            if dtype not in DTYPE_SIZES or not isinstance(shape, list) or any(not _is_int(x) or x < 0 for x in shape):
                fail("invalid tensor descriptor")
            count = 1
            for dim in shape:
                count *= dim
            if count * DTYPE_SIZES[dtype] != t.get("size"):
                fail("tensor descriptor conflicts with stored header")
            total = 0
            for b in t.get("blocks", []):
                off, n, raw = b.get("offset"), b.get("size"), b.get("raw_size")
                if (not _is_int(off) or not _is_int(n) or off < HEADER.size or n < 0 or off > limit
                        or n > limit - off or n > RAW_CHUNK or not _is_int(raw) or raw < 0 or raw > RAW_CHUNK):
                    fail("invalid block extent")
                spans.append((off, off + n))
                if b.get("codec") == "raw":
                    if n != raw:
                        fail("invalid raw block length")
                elif b.get("codec") in CODED:
                    r, c = b.get("rows"), b.get("cols")
                    if not _is_int(r) or not _is_int(c) or r <= 0 or c <= 0 or r * c * 2 != raw:
                        fail("invalid compressed block dimensions")
                else:
                    fail("unknown codec")
                total += raw
            if total != t["size"]:
                fail(f"tensor verification failed: {t['name']}")
            tensors[t["name"]] = t
    spans.sort()
    cursor = HEADER.size
    for start, end in spans:
        if start != cursor:
            fail("overlapping or unreferenced archive data")
        cursor = end
    if cursor != limit:
        fail("unreferenced archive data")
    return tensors


def decode_entries(blocks, base=0):
    """Plan rows that decode `blocks` (one tensor, in order) to byte offset
    `base` of the output; payload offsets are relative to archive byte 16."""
    out, dst = [], base
    for b in blocks:
        codec = xksv_gpu.CODEC_BY_NAME[b["codec"]]
        coded = codec != xksv_gpu.CODEC_RAW
        out.append(dict(src_offset=b["offset"] - HEADER.size, src_size=b["size"],
                        rows=b["rows"] if coded else 0, cols=b["cols"] if coded else 0,
                        dst_offset=dst, codec=codec))
        dst += b["raw_size"]
    return out


def gemm_entries(t):
    """Plan rows for y = W x of a 2-D BF16 weight (output rows at dst_offset);
    raw blocks carry their row count, python/runtime.py:275, 281."""
    cols = t["shape"][1]
    out, row = [], 0
    for b in t["blocks"]:
        codec = xksv_gpu.CODEC_BY_NAME[b["codec"]]
        rows = b["raw_size"] // (cols * 2)
        out.append(dict(src_offset=b["offset"] - HEADER.size, src_size=b["size"], rows=rows, cols=cols,
                        dst_offset=row, codec=codec))
        row += rows
    return out


def fusable(t):
    """The reference's eligibility test for a fused layer's weight
    (python/runtime.py:258-263): BF16, 2-D, some coded block, whole rows per
    block and coded blocks of the tensor's width."""
    if not t or t["dtype"] != "BF16" or len(t["shape"]) != 2:
        return False
    rows, cols = t["shape"]
    if not cols or not any(b["codec"] in CODED for b in t["blocks"]):
        return False
    return not any(b["raw_size"] % (cols * 2) or b["codec"] not in CODECS
                   or (b["codec"] != "raw" and b["cols"] != cols) for b in t["blocks"])


def fused_candidates(model, tensors):
    """Names of the linear layers install_fused_gemv replaces: bias-free
    nn.Linear modules other than lm_head whose weight is fusable
    (python/runtime.py:256-263)."""
    import torch
    names = []
    for name, module in model.named_modules():
        if not isinstance(module, torch.nn.Linear) or module.bias is not None or name == "lm_head":
            continue
        if fusable(tensors.get(name + ".weight")):
            names.append(name)
    return names


# -------------------------------------------------------- resident archive
class ResidentArchive:
    """An archive whose block region (bytes 16 .. index offset) lives in one
    device buffer for the archive's lifetime.

    ``verify()`` hashes every decoded block and tensor on the device;
    ``decode_all()`` decodes the checkpoint with one plan; ``tensor(name)``
    decodes one; ``fused(name)`` returns a resident fused-GEMV/GEMM weight.
    """

    def __init__(self, path, device="cuda", chunk_bytes=32 << 20, readers=8):
        import numpy as np
        import torch
        self.path = str(path)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            fail("GPU decode requires a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.lib = xksv_gpu.load()
        with open(self.path, "rb") as f:
            self.index, self.limit = load_index(f)
        self.tensors = check_index(self.index, self.limit)
        self.assets = {a["name"]: a for a in self.index.get("assets", [])}
        # every block once, as a slab-table template: payload offsets relative
        # to byte 16, rows/cols 0 for raw blocks; per tensor its first block,
        # block count, and each block's byte offset inside the tensor
        blocks = [b for t in self.tensors.values() for b in t["blocks"]]
        tab = np.zeros(len(blocks), dtype=xksv_gpu.slab_dtype())
        if blocks:
            tab["src_offset"] = np.fromiter((b["offset"] for b in blocks), np.uint64, len(blocks)) - HEADER.size
            tab["src_size"] = np.fromiter((b["size"] for b in blocks), np.uint64, len(blocks))
            tab["rows"] = np.fromiter((b["rows"] for b in blocks), np.uint64, len(blocks))
            tab["cols"] = np.fromiter((b["cols"] for b in blocks), np.uint64, len(blocks))
            tab["codec"] = np.fromiter((xksv_gpu.CODEC_BY_NAME[b["codec"]] for b in blocks), np.uint32, len(blocks))
        raw = np.fromiter((b["raw_size"] for b in blocks), np.uint64, len(blocks))
        self._raw = raw
        self._block_sha = [b.get("sha256") for b in blocks]
        self._table, self._first, self._nblocks = tab, {}, {}
        self._local = np.zeros(len(blocks), dtype=np.uint64)
        k = 0
        for name, t in self.tensors.items():
            n = len(t["blocks"])
            self._first[name], self._nblocks[name] = k, n
            if n:
                self._local[k + 1:k + n] = np.cumsum(raw[k:k + n - 1])
            k += n
        self.payload = self._upload(chunk_bytes, readers)
        self._check_parallel_headers()
        self.verified = False
        self._plans = {}
        # one BF16 scratch shared by the fused weights' tensor-core path
        # (their calls are serialised on the caller's stream)
        self._tc_scratch, self._tc_need = None, 0

    def _upload(self, chunk, readers):
        """Reads the block region into HBM: `readers` threads each pread
        chunk after chunk into their own two pinned buffers and copy them on
        their own stream, so file reads and host->device copies overlap."""
        import torch
        from concurrent.futures import ThreadPoolExecutor
        n = self.limit - HEADER.size
        dev = torch.empty(max(n, 1), dtype=torch.uint8, device=self.device)
        if not n:
            return dev
        chunk = max(1 << 20, min(chunk, n))
        chunks = [(pos, min(chunk, n - pos)) for pos in range(0, n, chunk)]
        readers = max(1, min(readers, len(chunks), os.cpu_count() or 1))
        fd = os.open(self.path, os.O_RDONLY)

        def reader(tid):
            with torch.cuda.device(self.device):
                stream = torch.cuda.Stream(self.device)
                pins = [torch.empty(chunk, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
                done = [None, None]
                k = 0
                for pos, m in chunks[tid::readers]:
                    if done[k] is not None:
                        done[k].synchronize()  # the copy that last used this buffer
                    view = memoryview(pins[k].numpy())[:m]
                    got = 0
                    while got < m:
                        r = os.preadv(fd, [view[got:]], HEADER.size + pos + got)
                        if r <= 0:
                            fail("unexpected end of file")
                        got += r
                    with torch.cuda.stream(stream):
                        dev[pos:pos + m].copy_(pins[k][:m], non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record(stream)
                    done[k] = ev
                    k ^= 1
                stream.synchronize()

        try:
            with ThreadPoolExecutor(max_workers=readers) as ex:
                for fut in [ex.submit(reader, i) for i in range(readers)]:
                    fut.result()
        finally:
            os.close(fd)
        return dev

    def _check_parallel_headers(self):
        """Parallel blocks' stored rows/cols must match the index
        (python/runtime.py:93, python/xksv.py:369)."""
        import numpy as np
        import torch
        tab = self._table
        sel = np.nonzero(tab["codec"] == xksv_gpu.CODEC_PARALLEL32)[0]
        if not len(sel):
            return
        if (tab["src_size"][sel] < 24).any():
            fail("parallel block dimensions disagree with index")
        off = torch.from_numpy((tab["src_offset"][sel] + 8).astype(np.int64)).to(self.device)
        idx = off[:, None] + torch.arange(16, device=self.device)
        got = self.payload[idx].cpu().numpy().view("<u8").reshape(-1, 2)
        if (got[:, 0] != tab["rows"][sel]).any() or (got[:, 1] != tab["cols"][sel]).any():
            fail("parallel block dimensions disagree with index")

    @property
    def payload_ptr(self):
        return self.payload.data_ptr()

    def asset(self, name):
        """An asset's bytes, checked against the index (python/xksv.py:322-323)."""
        a = self.assets.get(name)
        if a is None:
            fail(f"archive lacks {name}")
        with open(self.path, "rb") as f:
            f.seek(a["offset"])
            data = f.read(a["size"])
        if len(data) != a["size"] or hashlib.sha256(data).hexdigest() != a["sha256"]:
            fail("asset checksum failed")
        return data

    def _layout(self, names):
        """Byte offsets of `names` in one flat, TENSOR_ALIGN-aligned buffer."""
        offs, pos = {}, 0
        for name in names:
            offs[name] = pos
            pos += -(-self.tensors[name]["size"] // TENSOR_ALIGN) * TENSOR_ALIGN
        return offs, pos

    def _decode_table(self, names, offs):
        """(slab table decoding `names` to their offsets `offs`, the blocks'
        indices in archive order)."""
        import numpy as np
        idx = [np.arange(self._first[n], self._first[n] + self._nblocks[n]) for n in names]
        idx = np.concatenate(idx) if idx else np.zeros(0, np.int64)
        tab = self._table[idx]
        counts = [self._nblocks[n] for n in names]
        base = np.repeat(np.array([offs[n] for n in names], dtype=np.uint64), counts)
        tab["dst_offset"] = base + self._local[idx]
        return tab, idx

    def _decode_plan(self, names, offs):
        key = tuple(names)
        plan = self._plans.get(key)
        if plan is None:
            tab, _ = self._decode_table(names, offs)
            if not len(tab):
                return None
            plan = xksv_gpu.Plan(tab, lib=self.lib)
            self._plans[key] = plan
        return plan

    def _decode_into(self, names, offs, out, stream, keep=True):
        plan = self._decode_plan(names, offs)
        if plan is None:
            return
        try:
            plan.decode(self.payload, out, stream)
            if plan.status(stream):
                fail(f"GPU block decode failed: {names[0] if len(names) == 1 else 'archive'}")
        finally:
            if not keep:
                self._plans.pop(tuple(names), None)
                plan.close()

    def _stream(self):
        import torch
        return torch.cuda.current_stream(self.device).cuda_stream

    def decode_all(self, names=None):
        """{name: device tensor} for `names` (default: every tensor), decoded
        by one plan into one flat buffer that the tensors view."""
        import torch
        names = list(self.tensors) if names is None else list(names)
        offs, total = self._layout(names)
        flat = torch.empty(max(total, 1), dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            self._decode_into(names, offs, flat, self._stream())
        out = {}
        for name in names:
            t = self.tensors[name]
            view = flat[offs[name]:offs[name] + t["size"]]
            out[name] = view.view(torch_dtype(t["dtype"])).reshape(t["shape"])
        return out

    def tensor(self, name):
        if name not in self.tensors:
            fail(f"archive lacks tensor {name}")
        return self.decode_all([name])[name]

    def verify(self, max_scratch=4 << 30):
        """Decodes every block on the device and checks the SHA-256 of each
        block and of each tensor against the index (python/xksv.py:361-375),
        plus the assets on the host.  Block digests (at most 1 MiB each, many
        independent messages) run on the device, one thread per block; a
        tensor digest is one sequential message of up to gigabytes, which one
        GPU thread hashes at tens of MB/s against GB/s for a host core with
        SHA instructions, so those run on host threads over one device->host
        copy of the decoded group.  Tensors are processed in groups whose
        decoded bytes fit `max_scratch`.  Returns (tensors, bytes)."""
        import numpy as np
        import torch
        from concurrent.futures import ThreadPoolExecutor
        for name in self.assets:
            self.asset(name)
        names = list(self.tensors)
        groups, cur, cur_bytes = [], [], 0
        for name in names:
            size = self.tensors[name]["size"]
            if cur and cur_bytes + size > max_scratch:
                groups.append(cur)
                cur, cur_bytes = [], 0
            cur.append(name)
            cur_bytes += -(-size // TENSOR_ALIGN) * TENSOR_ALIGN
        if cur:
            groups.append(cur)
        nbytes = 0
        pool = ThreadPoolExecutor(max_workers=max(1, min(32, os.cpu_count() or 1)))
        try:
            with torch.cuda.device(self.device):
                stream = self._stream()
                for group in groups:
                    offs, total = self._layout(group)
                    flat = torch.empty(max(total, 1), dtype=torch.uint8, device=self.device)
                    self._decode_into(group, offs, flat, stream, keep=len(groups) == 1)
                    # block digests on the device, one thread per block
                    tab, idx = self._decode_table(group, offs)
                    if len(idx):
                        ranges = np.stack([tab["dst_offset"], self._raw[idx]], axis=1)
                        dig = torch.empty(32 * len(idx), dtype=torch.uint8, device=self.device)
                        xksv_gpu.sha256_ranges(ranges, flat.data_ptr(), dig.data_ptr(), stream, lib=self.lib)
                        got = dig.cpu().numpy().tobytes()
                        for j, i in enumerate(idx):
                            if got[32 * j:32 * j + 32].hex() != self._block_sha[i]:
                                name = next(n for n in group
                                            if self._first[n] <= i < self._first[n] + self._nblocks[n])
                                fail(f"block checksum failed: {name}")
                    # tensor digests on host threads, largest first; each
                    # tensor's copy overlaps the hashing of the previous ones
                    order = sorted(group, key=lambda n: -self.tensors[n]["size"])
                    futs = []
                    for n in order:
                        host = flat[offs[n]:offs[n] + self.tensors[n]["size"]].cpu().numpy()
                        futs.append(pool.submit(lambda h=host: hashlib.sha256(memoryview(h)).hexdigest()))
                    for name, fut in zip(order, futs):
                        if fut.result() != self.tensors[name].get("sha256"):
                            fail(f"tensor verification failed: {name}")
                    nbytes += sum(self.tensors[n]["size"] for n in group)
                    del flat
        finally:
            pool.shutdown()
        self.verified = True
        return len(names), nbytes

    def fused(self, name):
        """A FusedWeight for the 2-D BF16 tensor `name`."""
        t = self.tensors.get(name)
        if not fusable(t):
            fail(f"tensor {name} is not a fusable BF16 matrix")
        return FusedWeight(self, t)

    def shared_scratch(self):
        """The tensor-core scratch shared by this archive's fused weights,
        (re)allocated to the largest need registered so far."""
        import torch
        if self._tc_scratch is None or self._tc_scratch.numel() < self._tc_need:
            self._tc_scratch = torch.empty(self._tc_need, dtype=torch.uint8, device=self.device)
        return self._tc_scratch

    def close(self):
        """Releases the resident payload, the cached decode plans and the
        shared scratch."""
        for plan in self._plans.values():
            plan.close()
        self._plans.clear()
        self._tc_scratch = None
        self.payload = None


class FusedWeight:
    """y = x W^T for a weight that stays compressed in HBM: one plan over the
    weight's blocks (tile index built once for its 16-row serial blocks).
    Calls enqueue on the current stream and do not synchronise once the
    archive has been verified; before that, each call checks the plan's
    device status like the reference's per-call return code
    (python/runtime.py:278-279)."""

    def __init__(self, archive, t):
        import torch
        self.archive = archive
        self.name = t["name"]
        self.rows, self.cols = t["shape"]
        self.plan = xksv_gpu.Plan(gemm_entries(t), lib=archive.lib)
        with torch.cuda.device(archive.device):
            if self.plan.index(archive.payload, archive._stream()):
                fail(f"fused GEMV failed: {self.name}")
        # batch >= TC_MIN_BATCH decodes the weight into a BF16 scratch for the tensor
        # cores: borrow the archive's shared one instead of keeping a
        # decoded copy per weight
        self._scratch_need = self.plan.scratch_bytes()
        archive._tc_need = max(archive._tc_need, self._scratch_need)
        self._lent = None

    def __call__(self, x):
        import torch
        if x.shape[-1] != self.cols:
            raise ValueError(f"{self.name}: input width {x.shape[-1]} != {self.cols}")
        lead = x.shape[:-1]
        xb = x.reshape(-1, self.cols)
        batch = xb.shape[0]
        if batch == 0:
            return x.new_empty(*lead, self.rows)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        if batch >= xksv_gpu.TC_MIN_BATCH and self._scratch_need:
            buf = self.archive.shared_scratch()
            if self._lent is not buf:  # keeps the lent buffer alive while the plan points at it
                self.plan.set_scratch(buf.data_ptr(), buf.numel())
                self._lent = buf
        if batch == 1:  # x [cols] and y [rows]: the ABI's [cols, 1] and [rows, 1]
            xt = xb.reshape(self.cols).float().contiguous()
            y = torch.empty(self.rows, device=x.device, dtype=torch.float32)
        else:           # the ABI takes X [cols, batch] and returns Y [rows, batch]
            xt = xb.t().float().contiguous()
            y = torch.empty(self.rows, batch, device=x.device, dtype=torch.float32)
        self.plan.gemm(self.archive.payload, xt, y, batch, stream)
        if not self.archive.verified and self.plan.status(stream):
            fail(f"fused GEMV failed: {self.name}")
        out = y if batch == 1 else y.t()
        return out.to(x.dtype).reshape(*lead, self.rows)

    def close(self):
        self.plan.close()


def install_fused_gemv(model, archive):
    """Replaces the forward of every eligible linear layer with its resident
    FusedWeight (python/runtime.py:248-287); returns how many."""
    installed = 0
    modules = dict(model.named_modules())
    for name in fused_candidates(model, archive.tensors):
        fw = archive.fused(name + ".weight")
        modules[name].forward = fw
        modules[name].xksv_fused = fw
        installed += 1
    return installed


# ------------------------------------------------------------- loading
def assign_tensors(model, tensors, archive_names=None):
    """Places decoded tensors into a model's parameters and buffers with the
    reference's checks (python/runtime.py:72-117): every archive tensor must
    be a parameter or buffer of the model, and every model weight (up to tied
    aliases) must be supplied."""
    import torch
    expected = set(model.state_dict().keys())
    aliases = {}
    for n, p in model.named_parameters(remove_duplicate=False):
        aliases.setdefault(id(p), set()).add(n)
    supplied = set()
    for name, tensor in tensors.items():
        if name not in expected:
            fail(f"backend does not accept tensor {name}")
        module_name, _, leaf = name.rpartition(".")
        module = model.get_submodule(module_name) if module_name else model
        if leaf in module._parameters:
            old = module._parameters[leaf]
            module._parameters[leaf] = torch.nn.Parameter(tensor, requires_grad=old.requires_grad)
        elif leaf in module._buffers:
            module._buffers[leaf] = tensor
        else:
            fail(f"backend tensor is not a parameter or buffer: {name}")
        supplied.add(name)
    missing = expected - supplied
    for group in aliases.values():
        if group & supplied:
            missing -= group
    if missing:
        fail(f"archive is missing backend weights: {sorted(missing)[:10]}")
    if hasattr(model, "tie_weights"):
        model.tie_weights()
    return model


def backend_class(config):
    from transformers import AutoModelForCausalLM, AutoModelForImageTextToText
    architectures = getattr(config, "architectures", None) or []
    if any(name.endswith("ForConditionalGeneration") for name in architectures):
        return AutoModelForImageTextToText
    return AutoModelForCausalLM


def load_archive(path, device, model=None, verify=True, fused_gemv=False):
    """The ``load_archive(..., gpu_decode=True)`` flow (python/runtime.py:31-117)
    on a resident archive: upload, device verification, one-launch decode into
    the model, optional fused linear layers.  Without `model`, the model is
    built from the archive's config.json asset with Transformers, as the
    reference does, and a tokenizer is loaded when the assets hold one.
    Returns (model, tokenizer or None, archive)."""
    import torch
    archive = ResidentArchive(path, device)
    if verify:
        archive.verify()
    tokenizer = None
    if model is None:
        from transformers import AutoConfig, AutoTokenizer
        with tempfile.TemporaryDirectory(prefix="xksv-assets-") as assets:
            for name in archive.assets:
                (Path(assets) / name).write_bytes(archive.asset(name))
            if not (Path(assets) / "config.json").is_file():
                fail("archive lacks config.json")
            config = AutoConfig.from_pretrained(assets, local_files_only=True, trust_remote_code=False)
            model = backend_class(config).from_config(config, trust_remote_code=False)
            if any((Path(assets) / n).is_file() for n in ("tokenizer.json", "tokenizer.model", "vocab.json")):
                tokenizer = AutoTokenizer.from_pretrained(assets, local_files_only=True, trust_remote_code=False)
    model.eval()
    # fused linears keep their weights compressed in HBM: those tensors are
    # not decoded, and the parameter becomes a zero-element placeholder (the
    # fused forward never reads it), so the model holds the compressed bytes
    # once instead of compressed + decoded
    fused = [n + ".weight" for n in fused_candidates(model, archive.tensors)] if fused_gemv else []
    if fused_gemv and not fused:
        fail("no compatible linear layers for fused GEMV")
    keep = [n for n in archive.tensors if n not in set(fused)]
    tensors = archive.decode_all(keep)
    for name in fused:
        tensors[name] = torch.empty(0, dtype=torch.bfloat16, device=archive.device)
    assign_tensors(model, tensors)
    model.to(archive.device)
    if fused_gemv:
        install_fused_gemv(model, archive)
    torch.cuda.synchronize(archive.device)
    return model, tokenizer, archive
