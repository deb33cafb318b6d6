"""b2g_gemm_noalloc (F32 activations cast into the library's static scratch, K never split)
against b2g_gemm, the entry point that casts into its growable workspace, and against the C
oracle.  Collected last so it also runs after every other test has used the library.

Both paths cast the same way and run the same tensor-core kernels, so they agree to
max|d|/max|ref| <= 1e-6 (the kernel variant may differ only in accumulation order).  The
entry point exists for callers that cannot let a library allocate device memory, so one test
runs in a fresh process, forces split-K (which makes b2g_gemm allocate partial sums) and
checks that the device's free memory does not move across no-alloc calls.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

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


def test_noalloc_matches_oracle(engine, oracle):
    """The no-alloc path against the C restatement of linear(): F32 activations rounded to
    bf16 as the reference's linear() casts them, bf16 weights, F32 bias and output."""
    lib = lib_and_desc(engine)
    M, K, N = 200, 768, 384
    g = torch.Generator().manual_seed(3)
    x = torch.randn((M, K), generator=g)
    w = (torch.randn((N, K), generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.randn(N, generator=g) * 0.02
    xb = oracle.to_bf16_bits(x.numpy())
    wb = w.view(torch.int16).numpy().view(np.uint16)
    want = oracle.linear(xb, 2, wb, 2, bias.numpy())
    xd, wd, bd = x.to(DEV), w.to(DEV), bias.to(DEV)
    out = torch.empty((M, N), device=DEV)
    for _ in range(2):
        out.fill_(float("nan"))
        d = desc(engine, xd, wd, bd, out)
        assert lib.b2g_gemm_noalloc(ctypes.byref(d), None) == 0, engine.load().b2g_last_error()
        torch.cuda.synchronize()
        assert rel_err(out.cpu().numpy(), want) <= 1e-4


def _fresh_process_worker() -> int:
    """Run as a script: a process in which nothing has used the library yet."""
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "chroma-radiance_b200"))
    import b2g

    b2g.init()
    lib = lib_and_desc(b2g)
    b2g.set_gemm_variant(-1, 4)   # force 4-way split-K: b2g_gemm then needs partial-sum workspace
    M, K, N = 512, 3072, 3072
    g = torch.Generator().manual_seed(7)
    x = torch.randn((M, K), generator=g).to(DEV)           # F32 activations: the cast path
    w = (torch.randn((N, K), generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    bias = (torch.randn(N, generator=g) * 0.02).to(DEV)
    got, want = torch.empty((M, N), device=DEV), torch.empty((M, N), device=DEV)
    dg, dw = desc(b2g, x, w, bias, got), desc(b2g, x, w, bias, want)
    # The first call loads the kernels' module and looks up the array's address.
    assert lib.b2g_gemm_noalloc(ctypes.byref(dg), None) == 0, lib.b2g_last_error()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert lib.b2g_gemm_noalloc(ctypes.byref(dg), None) == 0, lib.b2g_last_error()
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, f"b2g_gemm_noalloc changed free device memory by {free0 - free1} bytes"
    # The same request through b2g_gemm grows its workspaces (cast operand, split-K partials):
    # the measurement above would have seen an allocation.
    assert lib.b2g_gemm(ctypes.byref(dw), None) == 0, lib.b2g_last_error()
    torch.cuda.synchronize()
    free2 = torch.cuda.mem_get_info()[0]
    assert free2 < free1, "b2g_gemm was expected to allocate its workspace in a fresh process"
    # b2g_gemm summed K in 4 split parts, the no-alloc call in one: fp32 accumulation order
    # differs, so the tolerance is the F32-output one of the GEMM tests (1e-4 of max|ref|).
    err = rel_err(got.cpu().numpy(), want.cpu().numpy())
    assert err <= 1e-4, err
    b2g.check_device_error()
    print("no-alloc fresh process ok", free0 - free2, err)
    return 0


def test_noalloc_allocates_nothing_in_fresh_process():
    r = subprocess.run([sys.executable, os.path.abspath(__file__)], capture_output=True, text=True, timeout=600)
    print(r.stdout[-2000:], r.stderr[-2000:])
    assert r.returncode == 0 and "no-alloc fresh process ok" in r.stdout


if __name__ == "__main__":
    sys.exit(_fresh_process_worker())
