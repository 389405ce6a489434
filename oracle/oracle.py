"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU parity checkers.

* ``Oracle()``    -- this repository's C restatement (oracle/xksv_oracle.c) of
  the reference slab codec (src/c_api.cpp:17-85, src/codec.cpp:11-74,
  src/layout.cpp:32-53).
* ``Reference()`` -- the reference CPU library itself, compiled from its own
  sources into oracle/_ref/libxksv_native.so by oracle/Makefile (absent when
  that build was not possible).

Both expose the reference Python binding's shape (python/xksv.py:138-162):
``call(op, data, rows, cols)`` and ``unpack_parallel(data)`` returning bytes, or
raising ``CodecError`` where the C function returned non-zero.
Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use this.
"""
import ctypes
import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent


class CodecError(RuntimeError):
    pass


def build():
    """Compile liboracle.so (and _ref when the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


class _Lib:
    prefix = ""

    def __init__(self, path):
        self.path = str(path)
        self.lib = ctypes.CDLL(self.path)
        P = ctypes.POINTER
        four = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                P(ctypes.c_void_p), P(ctypes.c_size_t)]
        for op in ("pack", "unpack", "pack_parallel"):
            f = getattr(self.lib, self.prefix + op)
            f.argtypes = four
            f.restype = ctypes.c_int
        f = getattr(self.lib, self.prefix + "unpack_parallel")
        f.argtypes = [ctypes.c_void_p, ctypes.c_size_t, P(ctypes.c_void_p), P(ctypes.c_size_t)]
        f.restype = ctypes.c_int
        self._free = getattr(self.lib, self.prefix + "free")
        self._free.argtypes = [ctypes.c_void_p]

    def _take(self, rc, out, size):
        if rc:
            raise CodecError(f"{self.path}: codec call failed")
        try:
            return ctypes.string_at(out, size.value)
        finally:
            self._free(out)

    def call(self, op, data, rows, cols):
        buf = ctypes.create_string_buffer(bytes(data), max(len(data), 1))
        out, size = ctypes.c_void_p(), ctypes.c_size_t()
        rc = getattr(self.lib, self.prefix + op)(buf, len(data), rows, cols, ctypes.byref(out),
                                                 ctypes.byref(size))
        return self._take(rc, out, size)

    def unpack_parallel(self, data):
        buf = ctypes.create_string_buffer(bytes(data), max(len(data), 1))
        out, size = ctypes.c_void_p(), ctypes.c_size_t()
        rc = getattr(self.lib, self.prefix + "unpack_parallel")(buf, len(data), ctypes.byref(out),
                                                                ctypes.byref(size))
        return self._take(rc, out, size)

    # convenience wrappers
    def pack(self, raw, rows, cols):
        return self.call("pack", raw, rows, cols)

    def unpack(self, blob, rows, cols):
        return self.call("unpack", blob, rows, cols)

    def pack_parallel(self, raw, rows, cols):
        return self.call("pack_parallel", raw, rows, cols)


class Oracle(_Lib):
    prefix = "oracle_"

    def __init__(self):
        path = HERE / "liboracle.so"
        if not path.exists():
            build()
        super().__init__(path)
        self.lib.oracle_decode_into.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                                ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
        self.lib.oracle_decode_into.restype = ctypes.c_int


class Reference(_Lib):
    prefix = "xksv_"

    def __init__(self):
        path = Path(os.environ.get("XKSV_LIBRARY", HERE / "_ref" / "libxksv_native.so"))
        if not path.exists():
            raise FileNotFoundError(path)
        super().__init__(path)


def reference_available():
    try:
        Reference()
        return True
    except OSError:
        return False
