"""ctypes binding of libxksv_cuda.so (include/xksv_cuda.h).

``load()`` returns the CDLL with the argument types the reference's own
callers declare for the five GPU entry points (python/runtime.py:40-44 and
251-255, python/tune.py:16-19, tests/test_cuda.py:11-12, 24-25, 35-36, 48-49,
66-67), plus the batched plan interface.  ``Plan`` wraps a plan for torch
callers.  There is no fallback: a missing library raises.
"""
import ctypes
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEFAULT_LIB = HERE / "libxksv_cuda.so"

CODEC_RAW, CODEC_TILE16, CODEC_PARALLEL32 = 0, 1, 2
CODEC_BY_NAME = {"raw": CODEC_RAW, "bf16-huffman-tile16": CODEC_TILE16,
                 "bf16-huffman-parallel32": CODEC_PARALLEL32}


class Slab(ctypes.Structure):
    _fields_ = [("src_offset", ctypes.c_uint64), ("src_size", ctypes.c_uint64),
                ("rows", ctypes.c_uint64), ("cols", ctypes.c_uint64),
                ("dst_offset", ctypes.c_uint64), ("x_offset", ctypes.c_uint64),
                ("codec", ctypes.c_uint32), ("flags", ctypes.c_uint32)]


_SIGS = {
    "xksv_cuda_decode": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                          ctypes.c_void_p], ctypes.c_int),
    "xksv_cuda_gemv": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                        ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "xksv_cuda_gemm": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                        ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "xksv_cuda_decode_parallel": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "xksv_cuda_gemv_parallel": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                 ctypes.c_void_p], ctypes.c_int),
    "xksv_plan_create": ([ctypes.POINTER(Slab), ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)],
                         ctypes.c_int),
    "xksv_plan_destroy": ([ctypes.c_void_p], None),
    "xksv_plan_decode": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                          ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "xksv_plan_decode_host": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                               ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "xksv_plan_gemm": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                        ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                        ctypes.c_void_p], ctypes.c_int),
    "xksv_plan_status": ([ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "xksv_plan_scratch_bytes": ([ctypes.c_void_p], ctypes.c_size_t),
    "xksv_plan_set_scratch": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t], ctypes.c_int),
    "xksv_plan_launches": ([ctypes.c_void_p], ctypes.c_int),
    "xksv_plan_set_gemm_route": ([ctypes.c_void_p, ctypes.c_int], ctypes.c_int),
    "xksv_plan_fused_ready": ([ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "xksv_plan_index": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "xksv_cuda_sha256": ([ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t, ctypes.c_void_p,
                          ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "xksv_plan_sha256": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                          ctypes.c_void_p], ctypes.c_int),
    "xksv_cuda_pack_tensor": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int,
                               ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p),
                               ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_void_p),
                               ctypes.POINTER(ctypes.c_size_t), ctypes.c_void_p], ctypes.c_int),
    "xksv_cuda_free": ([ctypes.c_void_p], None),
    "xksv_tp_fused_create": ([ctypes.c_int, ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t,
                              ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p], ctypes.c_int),
    "xksv_tp_fused_open": ([ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "xksv_tp_fused_gemm": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                            ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                            ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p],
                           ctypes.c_int),
    "xksv_tp_fused_destroy": ([ctypes.c_void_p], None),
    "xksv_tp_unique_id": ([ctypes.c_void_p], ctypes.c_int),
    "xksv_tp_comm_create": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                             ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "xksv_tp_comm_destroy": ([ctypes.c_void_p], None),
    "xksv_tp_gemm": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                      ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                      ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "xksv_host_pack": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                        ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                        ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "xksv_host_free": ([ctypes.c_void_p], None),
    "xksv_host_pack_tensor": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                               ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                               ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_size_t),
                               ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_size_t)],
                              ctypes.c_int),
    "xksv_cuda_decode_noalloc": ([ctypes.POINTER(Slab), ctypes.c_size_t, ctypes.c_void_p,
                                  ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                  ctypes.c_void_p], ctypes.c_int),
}

NOALLOC_MAX_SLABS = 4096
# xksv_plan_set_gemm_route
GEMM_AUTO, GEMM_SCRATCH, GEMM_FUSED = 0, 1, 2
# the fused decode -> tensor-core GEMM takes batches up to this size
FUSED_MAX_BATCH = 128
# xksv_plan_gemm: batches from this size run on the tensor cores (X rounded
# to BF16) when the plan has a tensor-core path (xksv_plan_scratch_bytes > 0)
TC_MIN_BATCH = 4

EXPORTS = tuple(_SIGS)
_lib = None


def library_path():
    return Path(os.environ.get("XKSV_CUDA_LIBRARY", DEFAULT_LIB))


def load(path=None):
    """Loads (once) and returns the CDLL with argtypes/restype set."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else library_path()
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: build it with xks-vectorforge_b200/build.py")
    lib = ctypes.CDLL(str(p))
    for name, (args, res) in _SIGS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    if path is None:
        _lib = lib
    return lib


def slab_dtype():
    """numpy structured dtype with the memory layout of xksv_slab."""
    import numpy as np
    return np.dtype({"names": [f for f, _ in Slab._fields_],
                     "formats": ["<u8"] * 6 + ["<u4"] * 2,
                     "offsets": [getattr(Slab, f).offset for f, _ in Slab._fields_],
                     "itemsize": ctypes.sizeof(Slab)})


def slab_table(entries):
    """entries: iterable of dicts/tuples with the xksv_slab fields, or a
    numpy array of slab_dtype() (used in place, no per-row Python work)."""
    if hasattr(entries, "dtype") and entries.dtype == slab_dtype():
        import numpy as np
        arr = np.ascontiguousarray(entries)
        # the pointer keeps a reference to the array
        return arr.ctypes.data_as(ctypes.POINTER(Slab)), len(arr)
    entries = list(entries)
    arr = (Slab * max(1, len(entries)))()
    for i, e in enumerate(entries):
        if isinstance(e, dict):
            arr[i] = Slab(e["src_offset"], e["src_size"], e.get("rows", 0), e.get("cols", 0),
                          e.get("dst_offset", 0), e.get("x_offset", 0), e["codec"], 0)
        else:
            arr[i] = Slab(*e)
    return arr, len(entries)


def host_pack(raw, rows, cols, codec, lib=None):
    """Encodes one slab on the host (xksv_host_pack); returns bytes."""
    lib = lib or load()
    buf = ctypes.create_string_buffer(bytes(raw), max(1, len(raw)))
    out, size = ctypes.c_void_p(), ctypes.c_size_t()
    if lib.xksv_host_pack(buf, len(raw), rows, cols, codec, ctypes.byref(out), ctypes.byref(size)):
        raise ValueError("xksv_host_pack failed")
    try:
        return ctypes.string_at(out, size.value)
    finally:
        lib.xksv_host_free(out)


def host_pack_tensor(ptr, nbytes, rows, cols, codec, threads=0, dst_base=0, lib=None):
    """Encodes a row-major BF16 tensor at host address `ptr` into compiler
    slabs.  Returns (payload bytes as a numpy uint8 array, list of slab dicts)."""
    import numpy as np
    lib = lib or load()
    pay, psize = ctypes.c_void_p(), ctypes.c_size_t()
    tab, ns = ctypes.c_void_p(), ctypes.c_size_t()
    if lib.xksv_host_pack_tensor(ptr, nbytes, rows, cols, codec, threads, dst_base,
                                 ctypes.byref(pay), ctypes.byref(psize), ctypes.byref(tab),
                                 ctypes.byref(ns)):
        raise ValueError("xksv_host_pack_tensor failed")
    try:
        payload = np.ctypeslib.as_array((ctypes.c_uint8 * max(1, psize.value)).from_address(pay.value))[:psize.value].copy()
        arr = (Slab * max(1, ns.value)).from_address(tab.value)
        slabs = [dict(src_offset=s.src_offset, src_size=s.src_size, rows=s.rows, cols=s.cols,
                      dst_offset=s.dst_offset, x_offset=s.x_offset, codec=s.codec)
                 for s in arr[:ns.value]]
    finally:
        lib.xksv_host_free(pay)
        lib.xksv_host_free(tab)
    return payload, slabs


def cuda_pack_tensor(d_ptr, rows, cols, codec, dst_base=0, stream=0, lib=None):
    """GPU encoder (xksv_cuda_pack_tensor) of a row-major BF16 tensor at device
    address `d_ptr`.  Returns (device payload address, payload bytes, slab
    dicts); release the payload with free_device()."""
    lib = lib or load()
    pay, psize = ctypes.c_void_p(), ctypes.c_size_t()
    tab, ns = ctypes.c_void_p(), ctypes.c_size_t()
    if lib.xksv_cuda_pack_tensor(d_ptr, rows, cols, codec, dst_base, ctypes.byref(pay), ctypes.byref(psize),
                                 ctypes.byref(tab), ctypes.byref(ns), stream):
        raise ValueError("xksv_cuda_pack_tensor failed")
    try:
        arr = (Slab * max(1, ns.value)).from_address(tab.value)
        slabs = [dict(src_offset=s.src_offset, src_size=s.src_size, rows=s.rows, cols=s.cols,
                      dst_offset=s.dst_offset, x_offset=s.x_offset, codec=s.codec)
                 for s in arr[:ns.value]]
    finally:
        lib.xksv_host_free(tab)
    return pay.value, psize.value, slabs


def free_device(d_ptr, lib=None):
    (lib or load()).xksv_cuda_free(d_ptr)


def dev_buffer(buf, nbytes=None, what="buffer"):
    """(address, byte size) of a device buffer given to a plan call: a torch
    tensor (its own size, or `nbytes` when that is smaller) or an integer
    device address with its byte size.  The library refuses a call whose
    slabs fall outside the sizes it is given."""
    if hasattr(buf, "data_ptr"):
        n = buf.numel() * buf.element_size()
        return buf.data_ptr(), n if nbytes is None else min(int(nbytes), n)
    if nbytes is None:
        raise TypeError(f"{what}: an integer device address needs its byte size")
    return int(buf), int(nbytes)


def _rows(buf, nrows, batch, what):
    """(address, rows) of an FP32 [rows, batch] matrix (tensor or address)."""
    if hasattr(buf, "data_ptr"):
        n = buf.numel() * buf.element_size() // (4 * max(1, batch))
        return buf.data_ptr(), n if nrows is None else min(int(nrows), n)
    if nrows is None:
        raise TypeError(f"{what}: an integer device address needs its row count")
    return int(buf), int(nrows)


class Plan:
    """A device-resident plan over one payload buffer (see include/xksv_cuda.h).
    Device buffers are torch tensors (their sizes bound the call) or integer
    addresses with explicit sizes (payload_bytes, out_bytes, x_rows, y_rows)."""

    def __init__(self, entries, lib=None):
        self.lib = lib or load()
        arr, n = slab_table(entries)
        h = ctypes.c_void_p()
        if self.lib.xksv_plan_create(arr, n, ctypes.byref(h)):
            raise ValueError("xksv_plan_create rejected the slab table")
        self.handle = h
        self.n = n

    def decode(self, d_payload, d_out, stream=0, payload_bytes=None, out_bytes=None):
        pay, npay = dev_buffer(d_payload, payload_bytes, "payload")
        out, nout = dev_buffer(d_out, out_bytes, "output")
        if self.lib.xksv_plan_decode(self.handle, pay, npay, out, nout, stream):
            raise RuntimeError("xksv_plan_decode refused the call or failed to launch")

    def decode_host(self, h_payload, size, d_payload, d_out, stream=0, out_bytes=None):
        """Host payload (`size` bytes at host address h_payload) -> d_payload
        -> decode, copy and decode overlapped (xksv_plan_decode_host)."""
        pay, npay = dev_buffer(d_payload, None if hasattr(d_payload, "data_ptr") else size, "payload")
        out, nout = dev_buffer(d_out, out_bytes, "output")
        if npay < size:
            raise ValueError("device payload buffer smaller than the host payload")
        if self.lib.xksv_plan_decode_host(self.handle, h_payload, size, pay, out, nout, stream):
            raise RuntimeError("xksv_plan_decode_host refused the call or failed")

    def gemm(self, d_payload, d_x, d_y, batch, stream=0, payload_bytes=None, x_rows=None, y_rows=None):
        pay, npay = dev_buffer(d_payload, payload_bytes, "payload")
        x, nx = _rows(d_x, x_rows, batch, "x")
        y, ny = _rows(d_y, y_rows, batch, "y")
        if self.lib.xksv_plan_gemm(self.handle, pay, npay, x, nx, y, ny, batch, stream):
            raise RuntimeError("xksv_plan_gemm refused the call or failed to launch")

    def index(self, d_payload, stream=0, payload_bytes=None):
        """Builds the tile index (xksv_plan_index); returns 0, or 1 on a bad slab."""
        pay, npay = dev_buffer(d_payload, payload_bytes, "payload")
        return self.lib.xksv_plan_index(self.handle, pay, npay, stream)

    def sha256(self, d_out, d_digests, stream=0, out_bytes=None):
        """Enqueues the SHA-256 of every slab's decoded bytes (xksv_plan_sha256)."""
        out, nout = dev_buffer(d_out, out_bytes, "output")
        dig = d_digests.data_ptr() if hasattr(d_digests, "data_ptr") else d_digests
        if self.lib.xksv_plan_sha256(self.handle, out, nout, dig, stream):
            raise RuntimeError("xksv_plan_sha256 failed")

    def scratch_bytes(self):
        """Bytes of BF16 scratch the tensor-core path needs (0: none)."""
        return self.lib.xksv_plan_scratch_bytes(self.handle)

    def set_scratch(self, d_scratch, nbytes):
        """Lends the plan a caller-owned scratch (xksv_plan_set_scratch)."""
        if self.lib.xksv_plan_set_scratch(self.handle, d_scratch, nbytes):
            raise ValueError("scratch too small or misaligned")

    def set_gemm_route(self, route):
        """GEMM_AUTO, GEMM_SCRATCH or GEMM_FUSED (xksv_plan_set_gemm_route)."""
        if self.lib.xksv_plan_set_gemm_route(self.handle, int(route)):
            raise ValueError(f"unknown GEMM route {route}")

    def fused_ready(self, d_payload):
        """True when the fused decode -> tensor-core GEMM applies to this
        plan on d_payload (indexed, all 16-row serial slabs)."""
        pay = d_payload.data_ptr() if hasattr(d_payload, "data_ptr") else d_payload
        return bool(self.lib.xksv_plan_fused_ready(self.handle, pay))

    def status(self, stream=0):
        """0 when no slab reported an error since the last call, else 1."""
        return self.lib.xksv_plan_status(self.handle, stream)

    def launches(self):
        return self.lib.xksv_plan_launches(self.handle)

    def close(self):
        if self.handle:
            self.lib.xksv_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------- tensor parallel
TP_ID_BYTES = 128


def shard_rows(rows, world, rank, align=16):
    """Row range [r0, r1) of `rank` when `rows` rows are split over `world`
    ranks in whole 16-row slabs (the first ranks take one slab more when the
    slab count does not divide)."""
    nslab = (rows + align - 1) // align
    base, extra = divmod(nslab, world)
    s0 = rank * base + min(rank, extra)
    s1 = s0 + base + (1 if rank < extra else 0)
    return min(rows, s0 * align), min(rows, s1 * align)


def shard_entries(entries, world, rank, rows_of):
    """The slab entries of this rank's rows, for TP GEMV/GEMM.

    `entries` are GEMV slab entries whose dst_offset is the slab's first row
    in the full Y (a plan may cover several tensors); `rows_of(e)` gives the
    (first row, row count) of the tensor the slab belongs to.  Each tensor is
    split separately with shard_rows; returns (local entries with dst_offset
    rebased to the rank's shard of Y, rows in the shard, and the list of
    (full_row0, local_row0, nrows) runs that map the shard back)."""
    out, runs, local = [], [], 0
    seen = {}
    for e in entries:
        t0, trows = rows_of(e)
        if t0 not in seen:
            r0, r1 = shard_rows(trows, world, rank)
            seen[t0] = (r0, r1, local)
            runs.append((t0 + r0, local, r1 - r0))
            local += r1 - r0
        r0, r1, l0 = seen[t0]
        row = e["dst_offset"] - t0
        if r0 <= row < r1:
            d = dict(e)
            d["dst_offset"] = l0 + row - r0
            out.append(d)
    return out, local, runs


def gathered_to_full(gathered, world, runs_per_rank, rows_shard):
    """Row indices: full_row -> row of the all-gathered buffer
    ([world * rows_shard] rows in rank order), from each rank's runs."""
    import numpy as np
    total = sum(n for runs in runs_per_rank for _, _, n in runs)
    idx = np.empty(total, dtype=np.int64)
    for g, runs in enumerate(runs_per_rank):
        for full0, local0, n in runs:
            idx[full0:full0 + n] = g * rows_shard + local0 + np.arange(n)
    return idx


class TPComm:
    """NCCL communicator for xksv_tp_gemm over the ranks of a torch.distributed
    group (which only carries the unique id)."""

    def __init__(self, rank, world, lib=None):
        import torch.distributed as dist
        self.lib = lib or load()
        uid = ctypes.create_string_buffer(TP_ID_BYTES)
        if rank == 0 and self.lib.xksv_tp_unique_id(uid):
            raise RuntimeError("xksv_tp_unique_id failed (NCCL not available?)")
        obj = [bytes(uid.raw) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = ctypes.create_string_buffer(obj[0], TP_ID_BYTES)
        h = ctypes.c_void_p()
        if self.lib.xksv_tp_comm_create(uid, world, rank, ctypes.byref(h)):
            raise RuntimeError("xksv_tp_comm_create failed")
        self.handle = h
        self.rank, self.world = rank, world

    def gemm(self, plan, d_payload, d_x, d_y_shard, rows_shard, d_y_full, batch, stream=0,
             payload_bytes=None, x_rows=None):
        pay, npay = dev_buffer(d_payload, payload_bytes, "payload")
        x, nx = _rows(d_x, x_rows, batch, "x")
        ys = d_y_shard.data_ptr() if hasattr(d_y_shard, "data_ptr") else d_y_shard
        yf = d_y_full.data_ptr() if hasattr(d_y_full, "data_ptr") else d_y_full
        if self.lib.xksv_tp_gemm(plan.handle, pay, npay, x, nx, ys, rows_shard, yf, batch, self.handle, stream):
            raise RuntimeError("xksv_tp_gemm failed")

    def close(self):
        if self.handle:
            self.lib.xksv_tp_comm_destroy(self.handle)
            self.handle = None


def sha256_ranges(ranges, d_base, d_digests, stream=0, lib=None):
    """SHA-256 of device byte ranges [(offset, length), ...] (or an n x 2
    integer array) at d_base into d_digests (n * 32 bytes, device);
    xksv_cuda_sha256."""
    import numpy as np
    lib = lib or load()
    flat = np.ascontiguousarray(np.asarray(ranges, dtype=np.uint64).reshape(-1))
    n = flat.size // 2
    ptr = flat.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))
    if lib.xksv_cuda_sha256(ptr, n, d_base, d_digests, stream):
        raise RuntimeError("xksv_cuda_sha256 failed")


class TPFused:
    """Fused tensor-parallel GEMV/GEMM (xksv_tp_fused_*): the GEMV epilogue
    stores each output row into every rank's gathered buffer over NVLink; the
    IPC handles travel over a torch.distributed group."""

    IPC_BYTES = 64

    def __init__(self, rank, world, max_rows_shard, max_batch=1, lib=None):
        import torch.distributed as dist
        self.lib = lib or load()
        h = ctypes.create_string_buffer(self.IPC_BYTES)
        ctx = ctypes.c_void_p()
        if self.lib.xksv_tp_fused_create(world, rank, max_rows_shard, max_batch, ctypes.byref(ctx), h):
            raise RuntimeError("xksv_tp_fused_create failed")
        self.handle = ctx
        handles = [None] * world
        dist.all_gather_object(handles, bytes(h.raw))
        joined = ctypes.create_string_buffer(b"".join(handles), self.IPC_BYTES * world)
        if self.lib.xksv_tp_fused_open(ctx, joined):
            self.close()
            raise RuntimeError("xksv_tp_fused_open failed")
        dist.barrier()

    def gemm(self, plan, d_payload, d_x, rows_shard, batch, stream=0, d_y_full=None, payload_bytes=None,
             x_rows=None):
        """Enqueues the fused call (and a copy of the gathered Y to d_y_full
        when given); returns the device address of the gathered Y."""
        pay, npay = dev_buffer(d_payload, payload_bytes, "payload")
        x, nx = _rows(d_x, x_rows, batch, "x")
        yf = d_y_full.data_ptr() if hasattr(d_y_full, "data_ptr") else d_y_full
        y = ctypes.c_void_p()
        if self.lib.xksv_tp_fused_gemm(self.handle, plan.handle, pay, npay, x, nx, rows_shard, batch,
                                       yf, ctypes.byref(y), stream):
            raise RuntimeError("xksv_tp_fused_gemm failed")
        return y.value

    def close(self):
        if self.handle:
            self.lib.xksv_tp_fused_destroy(self.handle)
            self.handle = None
