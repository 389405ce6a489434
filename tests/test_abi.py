"""CPU: the C-ABI library builds for sm_100a, loads without a GPU, and exports
every function include/*.h declares (no compute calls here)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:int|void|size_t|const char\s*\*)\s+(xksv_\w+)\s*\(", text, flags=re.M)
    return names


@pytest.fixture(scope="module")
def lib():
    import build as b  # xks-vectorforge_b200/build.py
    b.build()
    import xksv_gpu
    return xksv_gpu.load()


def test_header_declares_reference_entry_points():
    names = set(declared_functions())
    for ref in ("xksv_cuda_decode", "xksv_cuda_gemv", "xksv_cuda_gemm",
                "xksv_cuda_decode_parallel", "xksv_cuda_gemv_parallel"):
        assert ref in names


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 11
    for n in names:
        assert hasattr(lib, n), n
        assert isinstance(getattr(lib, n), ctypes._CFuncPtr)


def test_binding_covers_header(lib):
    import xksv_gpu
    assert set(declared_functions()) == set(xksv_gpu.EXPORTS)


def test_null_arguments_rejected_without_device(lib):
    # argument checks happen before any CUDA call (cuda/decode.cu:49, 90, 96)
    assert lib.xksv_cuda_decode(None, 0, 1, 1, None) == 1
    assert lib.xksv_cuda_gemv(b"x" * 300, 300, 1, 1, None, None) == 1
    assert lib.xksv_cuda_gemm(b"x" * 300, 300, 1, 1, 1, None, None) == 1
    assert lib.xksv_cuda_decode_parallel(None, 0, None) == 1
    assert lib.xksv_cuda_gemv_parallel(b"x" * 40, 40, None, None) == 1


def test_header_compiles_as_c99(tmp_path):
    """The boundary is plain C: the header compiles under -std=c99 -pedantic."""
    import subprocess
    src = tmp_path / "h.c"
    src.write_text('#include "xksv_cuda.h"\nint main(void) { return 0; }\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-fsyntax-only",
                    "-I", str(ROOT / "include"), str(src)], check=True)


def test_c_caller_links_and_encodes(tmp_path, lib):
    """A C program linked against libxksv_cuda.so calls a host-side entry
    point (xksv_host_pack of a 1x4 slab) and gets the reference layout."""
    import subprocess
    src = tmp_path / "c.c"
    src.write_text(r"""
#include <stdio.h>
#include <string.h>
#include "xksv_cuda.h"
int main(void) {
  unsigned short w[4] = {0x3f80, 0x3f80, 0xbf80, 0x4000};
  void* out = NULL; size_t n = 0;
  if (xksv_host_pack(w, sizeof w, 1, 4, XKSV_CODEC_TILE16, &out, &n)) return 2;
  unsigned long long count; memcpy(&count, out, 8);
  printf("%zu %llu\n", n, count);
  xksv_host_free(out);
  return 0;
}
""")
    exe = tmp_path / "c"
    libdir = str(ROOT / "xks-vectorforge_b200")
    subprocess.run(["gcc", "-std=c99", "-I", str(ROOT / "include"), str(src), "-L", libdir, "-lxksv_cuda",
                    "-Wl,-rpath," + libdir, "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, check=True)
    size, count = map(int, r.stdout.split())
    assert count == 4 and size == 272 + 4 + 1  # header, 4 sign/mantissa bytes, 1 byte of codes
