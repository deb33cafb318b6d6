"""CPU checks of the C ABI: the library loads, exports every symbol include/b2g.h declares,
the Python descriptor matches the C struct layout, and calls fail loudly without a GPU."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from conftest import PKG, REPO, cuda_available

HEADER = REPO / "include" / "b2g.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2g_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("b2g_init", "b2g_gemm", "b2g_linear_lt", "b2g_linear_gated_residual", "b2g_batched_matmul_Bt",
                 "b2g_last_error", "b2g_check_device_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    import b2g

    lib = b2g.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"libb2g.so lacks {missing}"
    assert b"sm_100a" in lib.b2g_version()


def test_gemm_desc_layout_matches_c(tmp_path):
    """ctypes GemmDesc must have the C struct's size and field offsets."""
    import b2g

    src = tmp_path / "layout.c"
    fields = [f[0] for f in b2g.GemmDesc._fields_]
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(b2g_gemm_desc, {f}));' for f in fields)
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "b2g.h"\nint main(void){\n'
                   f'  printf("size %zu\\n", sizeof(b2g_gemm_desc));\n{body}\n  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["/usr/bin/gcc", "-I", str(REPO / "include"), "-I", "/usr/local/cuda/include", str(src), "-o",
                    str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(b2g.GemmDesc)
    for f in fields:
        assert int(out[f]) == getattr(b2g.GemmDesc, f).offset, f


def test_missing_library_fails_loudly(tmp_path):
    import b2g

    saved = b2g._lib
    try:
        b2g._lib = None
        with pytest.raises(b2g.B2GError):
            b2g.load(tmp_path / "nope.so")
    finally:
        b2g._lib = saved


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU behaviour")
def test_no_device_is_an_error_not_a_fallback():
    import b2g

    lib = b2g.load()
    assert lib.b2g_init() != 0
    assert len(lib.b2g_last_error()) > 0
    # a GEMM call must refuse rather than compute anything on the CPU
    d = b2g.GemmDesc()
    d.M = d.N = d.K = 8
    d.a = d.b = d.d = 16
    d.lda = d.ldb = d.ldd = 8
    d.a_dtype = d.b_dtype = b2g.BF16
    d.d_dtype = b2g.F32
    assert lib.b2g_gemm(ctypes.byref(d), None) != 0


def test_invalid_arguments_rejected_before_any_device_work():
    import b2g

    lib = b2g.load()
    assert lib.b2g_gemm(None, None) == 1  # B2G_ERR_INVALID
    d = b2g.GemmDesc()
    d.M, d.N, d.K = -1, 4, 4
    assert lib.b2g_gemm(ctypes.byref(d), None) == 1
    d.M, d.N, d.K = 4, 4, 4
    d.a = d.b = d.d = 16
    d.lda, d.ldb, d.ldd = 2, 4, 4   # lda < K
    assert lib.b2g_gemm(ctypes.byref(d), None) == 1
    d.lda = 4
    d.a_dtype, d.b_dtype = b2g.BF16, b2g.F16  # mixed 16-bit operands
    assert lib.b2g_gemm(ctypes.byref(d), None) == 2  # B2G_ERR_UNSUPPORTED
    # M == 0 is a no-op success, like an empty cuBLAS call
    d.M = 0
    assert lib.b2g_gemm(ctypes.byref(d), None) == 0
