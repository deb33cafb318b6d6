"""b2g_gemm_noalloc (F32 activations cast into the library's static scratch, K never split)
against b2g_gemm, the entry point that casts into its growable workspace.  Collected last so
it also runs after every other test has used the library.

Both paths cast the same way and run the same tensor-core kernels, so they agree to
max|d|/max|ref| <= 1e-6 (the kernel variant may differ only in accumulation order).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def lib_and_desc(engine):
    lib = engine.load()
    lib.b2g_gemm_noalloc.argtypes = [ctypes.POINTER(engine.GemmDesc), ctypes.c_void_p]
    lib.b2g_gemm_noalloc.restype = ctypes.c_int
    return lib


def desc(engine, x, w, bias, out, epilogue=0, gate=None):
    M, K = x.shape
    N = w.shape[0]
    d = engine.GemmDesc()
    d.M, d.N, d.K = M, N, K
    d.a, d.a_dtype, d.lda = x.data_ptr(), 0, x.stride(0)
    d.b, d.b_dtype, d.ldb = w.data_ptr(), 2, w.stride(0)
    d.bias, d.bias_dtype = (bias.data_ptr() if bias is not None else None), 0
    d.d, d.d_dtype, d.ldd = out.data_ptr(), 0, out.stride(0)
    d.epilogue = epilogue
    d.gate = gate.data_ptr() if gate is not None else None
    return d


@pytest.mark.parametrize("M,K,N,epilogue", [(384, 1000, 520, 0), (1024, 4096, 768, 2), (77, 3072, 3072, 0)])
def test_noalloc_matches_gemm_twice(engine, M, K, N, epilogue):
    lib = lib_and_desc(engine)
    engine.set_gemm_variant(-1, 0)
    g = torch.Generator().manual_seed(M + K + N)
    x = torch.randn((M, K), generator=g).to(DEV)
    w = (torch.randn((N, K), generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    bias = (torch.randn(N, generator=g) * 0.02).to(DEV)
    gate = torch.randn(N, generator=g).to(DEV) if epilogue == 2 else None
    res0 = torch.randn((M, N), generator=g).to(DEV)
    st = torch.cuda.current_stream().cuda_stream
    want, got = res0.clone(), res0.clone()
    for call in range(2):   # two calls in a row on each path (gated residual accumulates)
        dw = desc(engine, x, w, bias, want, epilogue, gate)
        assert lib.b2g_gemm(ctypes.byref(dw), ctypes.c_void_p(st)) == 0, engine.load().b2g_last_error()
        dg = desc(engine, x, w, bias, got, epilogue, gate)
        assert lib.b2g_gemm_noalloc(ctypes.byref(dg), ctypes.c_void_p(st)) == 0, engine.load().b2g_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert rel_err(got.cpu().numpy(), want.cpu().numpy()) <= 1e-6, f"call {call}"
    engine.check_device_error()


def test_noalloc_rejects_oversize_before_launching(engine):
    lib = lib_and_desc(engine)
    M, K, N = 1025, 4096, 64        # 1025 * 4096 * 2 bytes > 8 MiB of static scratch
    x = torch.zeros((M, K), device=DEV)
    w = torch.zeros((N, K), dtype=torch.bfloat16, device=DEV)
    out = torch.full((M, N), 7.0, device=DEV)
    n0 = engine.launch_count()
    d = desc(engine, x, w, None, out)
    assert lib.b2g_gemm_noalloc(ctypes.byref(d), None) == 1          # B2G_ERR_INVALID
    assert b"8388608" in lib.b2g_last_error()
    assert engine.launch_count() == n0
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)
