"""TEST INFRASTRUCTURE ONLY: ctypes access to the two checkers built by oracle/Makefile.

  Oracle (liboracle.so)   fp32 C restatement of the reference's GEMM path, numpy in/out.
  Ref    (_ref/libref_cublaslt.so)  the reference's own cublas_ops.cuh / kernels.cu compiled
                           from its sources; device pointers in, runs on the GPU.

Only tests/, __graft_entry__.smoke() and bench.py (its CPU-baseline leg and its
--impl reference arm) use this module.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_PATH = HERE / "liboracle.so"
REF_PATH = HERE / "_ref" / "libref_cublaslt.so"

F32, F16, BF16 = 0, 1, 2          # reference DType codes (tensor.cuh:116)
TF32 = 3                          # oracle rounding target only
CUDA_R_32F, CUDA_R_16F, CUDA_R_16BF = 0, 2, 14

_c_p = ctypes.c_void_p
_i64 = ctypes.c_int64


def _np_ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


class Oracle:
    """fp32 CPU oracle (oracle.c)."""

    def __init__(self, path: str | os.PathLike = ORACLE_PATH):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        lib = ctypes.CDLL(str(path))
        lib.oracle_linear.argtypes = [_i64, _i64, _i64, _c_p, ctypes.c_int, _i64, _c_p, ctypes.c_int, _i64, _c_p,
                                      _c_p, _i64, ctypes.c_int]
        lib.oracle_linear.restype = ctypes.c_int
        lib.oracle_batched_matmul_bt.argtypes = [_c_p, _c_p, _c_p, _i64, _i64, _i64, _i64, ctypes.c_int,
                                                 ctypes.c_int]
        lib.oracle_batched_matmul_bt.restype = ctypes.c_int
        for name in ("oracle_gelu",):
            getattr(lib, name).argtypes = [_c_p, _c_p, _i64]
        lib.oracle_gelu_to_bf16.argtypes = [_c_p, _c_p, _i64]
        lib.oracle_gated_residual.argtypes = [_c_p, _c_p, _c_p, _c_p, _i64, _i64]
        lib.oracle_modulate.argtypes = [_c_p, _c_p, _c_p, _c_p, _i64, _i64, ctypes.c_float]
        lib.oracle_rms_norm.argtypes = [_c_p, _c_p, _c_p, _i64, _i64, ctypes.c_float]
        lib.oracle_rope.argtypes = [_c_p, _c_p, _c_p, _i64, _i64, _i64]
        lib.oracle_round.argtypes = [_c_p, ctypes.c_int, _c_p, _i64]
        lib.oracle_f32_to_e4m3_array.argtypes = [_c_p, _c_p, _i64]
        lib.oracle_e4m3_to_f32_array.argtypes = [_c_p, _c_p, _i64]
        lib.oracle_quantize_rows_e4m3.argtypes = [_c_p, _i64, _i64, _c_p, _c_p]
        lib.oracle_f32_to_bf16_array.argtypes = [_c_p, _c_p, _i64]
        lib.oracle_f32_to_f16_array.argtypes = [_c_p, _c_p, _i64]
        lib.oracle_to_f32.argtypes = [_c_p, ctypes.c_int, _c_p, _i64]
        lib.oracle_num_threads.restype = ctypes.c_int
        lib.oracle_attention_rope.argtypes = [_c_p] * 6 + [_i64] * 3
        lib.oracle_attention_rope.restype = ctypes.c_int
        self.lib = lib

    def num_threads(self) -> int:
        return int(self.lib.oracle_num_threads())

    # --- formats -----------------------------------------------------------------
    def to_bf16_bits(self, a: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.float32)
        out = np.empty(a.shape, dtype=np.uint16)
        self.lib.oracle_f32_to_bf16_array(_np_ptr(a), _np_ptr(out), a.size)
        return out

    def to_f16_bits(self, a: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.float32)
        out = np.empty(a.shape, dtype=np.uint16)
        self.lib.oracle_f32_to_f16_array(_np_ptr(a), _np_ptr(out), a.size)
        return out

    def to_f32(self, bits: np.ndarray, dtype: int) -> np.ndarray:
        bits = np.ascontiguousarray(bits)
        out = np.empty(bits.shape, dtype=np.float32)
        self.lib.oracle_to_f32(_np_ptr(bits), dtype, _np_ptr(out), bits.size)
        return out

    def round(self, a: np.ndarray, dtype: int) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.float32)
        out = np.empty_like(a)
        self.lib.oracle_round(_np_ptr(a), dtype, _np_ptr(out), a.size)
        return out

    # --- GEMM --------------------------------------------------------------------
    def linear(self, x: np.ndarray, xdt: int, w: np.ndarray, wdt: int, bias: np.ndarray | None = None,
               nthreads: int = 0) -> np.ndarray:
        """linear_lt semantics: x [M,K], w [N,K] given as F32 arrays or uint16 bit arrays of
        dtype xdt/wdt; returns F32 [M,N] = x.w^T + bias."""
        x = np.ascontiguousarray(x)
        w = np.ascontiguousarray(w)
        M, K = x.shape
        N = w.shape[0]
        out = np.empty((M, N), dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        rc = self.lib.oracle_linear(M, K, N, _np_ptr(x), xdt, K, _np_ptr(w), wdt, K, _np_ptr(b), _np_ptr(out), N,
                                    nthreads)
        if rc != 0:
            raise MemoryError("oracle_linear")
        return out

    def batched_matmul_bt(self, A: np.ndarray, B: np.ndarray, rounding: int = TF32,
                          nthreads: int = 0) -> np.ndarray:
        """rounding: TF32 (the reference's behaviour on B200), BF16, or 0 for exact fp32."""
        A = np.ascontiguousarray(A, dtype=np.float32)
        B = np.ascontiguousarray(B, dtype=np.float32)
        batch, M, K = A.shape
        N = B.shape[1]
        C = np.empty((batch, M, N), dtype=np.float32)
        self.lib.oracle_batched_matmul_bt(_np_ptr(A), _np_ptr(B), _np_ptr(C), batch, M, K, N, int(rounding),
                                          nthreads)
        return C

    # --- elementwise ---------------------------------------------------------------
    def gelu(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.oracle_gelu(_np_ptr(x), _np_ptr(out), x.size)
        return out

    def gelu_to_bf16(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, dtype=np.uint16)
        self.lib.oracle_gelu_to_bf16(_np_ptr(x), _np_ptr(out), x.size)
        return out

    def gated_residual(self, x: np.ndarray, y: np.ndarray, gate: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.ascontiguousarray(y, dtype=np.float32)
        gate = np.ascontiguousarray(gate, dtype=np.float32)
        M, C = x.shape
        out = np.empty_like(x)
        self.lib.oracle_gated_residual(_np_ptr(x), _np_ptr(y), _np_ptr(gate), _np_ptr(out), M, C)
        return out

    def modulate(self, x, shift, scale, eps=1e-6):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        M, C = x.shape
        self.lib.oracle_modulate(_np_ptr(x), _np_ptr(np.ascontiguousarray(shift, np.float32)),
                                 _np_ptr(np.ascontiguousarray(scale, np.float32)), _np_ptr(out), M, C, eps)
        return out

    def attention_rope(self, Q, K, V, pe, mask=None):
        """Q, K, V F32 [L, H, D]; pe [L, D/2, 4]; mask [L] or None -> F32 [L, H*D]."""
        Q, K, V, pe = (np.ascontiguousarray(a, np.float32) for a in (Q, K, V, pe))
        L, H, D = Q.shape
        out = np.empty((L, H * D), dtype=np.float32)
        m = None if mask is None else np.ascontiguousarray(mask, np.float32)
        if self.lib.oracle_attention_rope(_np_ptr(Q), _np_ptr(K), _np_ptr(V), _np_ptr(pe), _np_ptr(m), _np_ptr(out),
                                          L, H, D) != 0:
            raise MemoryError("oracle_attention_rope")
        return out

    # ---------------------------------------------------------------- FP8 E4M3
    def to_e4m3_bits(self, a: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.float32)
        out = np.empty(a.shape, dtype=np.uint8)
        self.lib.oracle_f32_to_e4m3_array(_np_ptr(a), _np_ptr(out), a.size)
        return out

    def e4m3_to_f32(self, bits: np.ndarray) -> np.ndarray:
        bits = np.ascontiguousarray(bits, dtype=np.uint8)
        out = np.empty(bits.shape, dtype=np.float32)
        self.lib.oracle_e4m3_to_f32_array(_np_ptr(bits), _np_ptr(out), bits.size)
        return out

    def quantize_rows_e4m3(self, x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        """Per-row E4M3 quantisation: (codes [rows, cols] uint8, scales [rows] f32)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, cols = x.shape
        q = np.empty((rows, cols), dtype=np.uint8)
        s = np.empty(rows, dtype=np.float32)
        self.lib.oracle_quantize_rows_e4m3(_np_ptr(x), rows, cols, _np_ptr(q), _np_ptr(s))
        return q, s

    def gemm_fp8(self, qa, sa, qb, sb, bias=None) -> np.ndarray:
        """(sum_k a.b over the E4M3 values, exact products, float64 sums) * sa[m] * sb[n] + bias."""
        acc = self.e4m3_to_f32(qa).astype(np.float64) @ self.e4m3_to_f32(qb).astype(np.float64).T
        out = acc * sa.astype(np.float64)[:, None] * sb.astype(np.float64)[None, :]
        if bias is not None:
            out = out + bias.astype(np.float64)[None, :]
        return out

    def rope(self, x, pe, n_head):
        """RoPE rotation of F32 [L, H*D] rows by pe [L, D/2, 4], kept in fp32."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        pe = np.ascontiguousarray(pe, dtype=np.float32)
        L, HD = x.shape
        out = np.empty_like(x)
        self.lib.oracle_rope(_np_ptr(x), _np_ptr(pe), _np_ptr(out), L, n_head, HD // n_head)
        return out

    def rms_norm(self, x, scale, eps=1e-6):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        rows, C = x.shape
        self.lib.oracle_rms_norm(_np_ptr(x), _np_ptr(np.ascontiguousarray(scale, np.float32)), _np_ptr(out), rows,
                                 C, eps)
        return out


class Ref:
    """The reference's own GEMM path (cuBLASLt), built from its sources; device pointers."""

    def __init__(self, path: str | os.PathLike = REF_PATH):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} missing: it is built by `make -C oracle` where the reference "
                                    "sources are present")
        lib = ctypes.CDLL(str(path))
        sig = {
            "ref_init": [],
            "ref_sync": [],
            "ref_cublaslt_version": [],
            "ref_linear_lt": [_i64, _i64, _i64, _c_p, ctypes.c_int, _c_p, ctypes.c_int, _c_p, _c_p],
            "ref_linear": [_c_p, ctypes.c_int, _c_p, ctypes.c_int, _c_p, _c_p, _i64, _i64, _i64],
            "ref_linear_gated_residual": [_c_p, ctypes.c_int, _c_p, ctypes.c_int, _c_p, _c_p, _c_p, _i64, _i64,
                                          _i64],
            "ref_batched_matmul_Bt": [_c_p, _c_p, _c_p, _i64, _i64, _i64, _i64],
            "ref_gelu": [_c_p, _c_p, _i64],
            "ref_gelu_to_bf16": [_c_p, _c_p, _i64],
            "ref_gated_residual": [_c_p, _c_p, _c_p, _c_p, _i64, _i64],
            "ref_f32_to_bf16": [_c_p, _c_p, _i64],
            "ref_f32_to_fp16": [_c_p, _c_p, _i64],
            "ref_modulate_to_bf16": [_c_p, _c_p, _c_p, _c_p, _i64, _i64, ctypes.c_float],
            "ref_rms_norm": [_c_p, _c_p, _c_p, _i64, _i64, ctypes.c_float],
            "ref_concat_last_dim_to_bf16": [_c_p, _c_p, _c_p, _i64, _i64, _i64],
            "ref_bench_linear_lt": [_i64, _i64, _i64, ctypes.c_int, _c_p, _c_p, _c_p, ctypes.c_int, ctypes.c_int,
                                    _i64, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)],
        }
        for name, args in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        self.lib = lib
        self.lib.ref_init()

    def __getattr__(self, name):
        return getattr(self.lib, "ref_" + name)


ATTN_REF_PATH = HERE / "_ref" / "libref_attention.so"
# The reference's whole forward_cfg, stock (oracle/Makefile builds it from the drop-in
# directory's harness and the reference's own headers); bound by chroma-radiance_b200/harness.py.
MODEL_REF_PATH = HERE / "_ref" / "libref_model.so"


class AttnRef:
    """The reference's attention (cuDNN-frontend flash SDPA with RoPE), built from its sources."""

    def __init__(self, path: str | os.PathLike = ATTN_REF_PATH):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} missing: built by `make -C oracle` where the reference sources are present")
        lib = ctypes.CDLL(str(path))
        lib.ref_attn_init.restype = ctypes.c_int
        lib.ref_attention_with_rope.argtypes = [_c_p] * 4 + [ctypes.c_int, ctypes.c_int, _i64, _c_p, _c_p]
        lib.ref_attention_with_rope.restype = ctypes.c_int
        lib.ref_bench_attention.argtypes = [_c_p] * 4 + [ctypes.c_int, ctypes.c_int, _i64, _c_p, ctypes.c_int,
                                                         ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
        lib.ref_bench_attention.restype = ctypes.c_int
        pp = ctypes.POINTER(ctypes.c_void_p)
        lib.ref_double_block.argtypes = [pp, _i64, _i64]
        lib.ref_double_block_attn.argtypes = [pp, _i64, _i64]
        lib.ref_double_block_mlp.argtypes = [pp, _i64, _i64]
        lib.ref_single_block.argtypes = [pp, _i64]
        lib.ref_alloc_blocks.argtypes = [ctypes.c_ulonglong, _i64, _i64, _i64, pp, pp]
        lib.ref_bench_blocks.argtypes = [pp, pp, _i64, _i64, ctypes.c_int, ctypes.c_int, _i64,
                                         ctypes.POINTER(ctypes.c_double)]
        for f in ("ref_double_block", "ref_double_block_attn", "ref_double_block_mlp", "ref_single_block",
                  "ref_alloc_blocks", "ref_bench_blocks"):
            getattr(lib, f).restype = ctypes.c_int
        lib.ref_t5_attention.argtypes = [_c_p] * 4 + [ctypes.c_int, ctypes.c_int, _i64, ctypes.c_float, _c_p, _c_p]
        lib.ref_t5_attention.restype = ctypes.c_int
        lib.ref_bench_t5_attention.argtypes = [_c_p] * 4 + [ctypes.c_int, ctypes.c_int, _i64, ctypes.c_float, _c_p,
                                                            ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
        lib.ref_bench_t5_attention.restype = ctypes.c_int
        lib.ref_sdpa_bf16.argtypes = [_c_p] * 5 + [ctypes.c_int] * 3
        lib.ref_sdpa_bf16.restype = ctypes.c_int
        lib.ref_bench_sdpa_bf16.argtypes = [_c_p] * 5 + [ctypes.c_int] * 5 + [_c_p, _i64,
                                                                            ctypes.POINTER(ctypes.c_double)]
        lib.ref_bench_sdpa_bf16.restype = ctypes.c_int
        lib.ref_bench_t5_leg.argtypes = [ctypes.c_int, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         _c_p, _i64, ctypes.POINTER(ctypes.c_double)]
        lib.ref_bench_t5_leg.restype = ctypes.c_int
        lib.ref_attn_init()
        self.lib = lib

    @staticmethod
    def ptr_array(ptrs):
        """ctypes void* array from device addresses (ints or None)."""
        return (ctypes.c_void_p * len(ptrs))(*ptrs)

    def double_block(self, ptrs, T, I):
        return self.lib.ref_double_block(self.ptr_array(ptrs), T, I)

    def double_block_attn(self, ptrs, T, I):
        return self.lib.ref_double_block_attn(self.ptr_array(ptrs), T, I)

    def double_block_mlp(self, ptrs, T, I):
        return self.lib.ref_double_block_mlp(self.ptr_array(ptrs), T, I)

    def single_block(self, ptrs, L):
        return self.lib.ref_single_block(self.ptr_array(ptrs), L)

    def attention_with_rope(self, Q, K, V, pe, n_head, d_head, L, mask, out):
        return self.lib.ref_attention_with_rope(Q, K, V, pe, n_head, d_head, L, mask, out)

    def sdpa_bf16(self, Q, K, V, bias, O, n_head, L, d_head):
        """cudnn_sdpa_forward on bf16 [n_head, L, d_head] device buffers (addresses)."""
        return self.lib.ref_sdpa_bf16(Q, K, V, bias, O, n_head, L, d_head)

    def bench_t5_leg(self, layers, L, d, ff, heads, iters, warmup, flush, flush_bytes):
        """Per-pass milliseconds of the reference's T5 GEMMs + t5_attention leg (ref_bench_t5_leg)."""
        ms = (ctypes.c_double * iters)()
        rc = self.lib.ref_bench_t5_leg(layers, L, d, ff, heads, iters, warmup, flush, flush_bytes, ms)
        if rc != 0:
            raise RuntimeError(f"ref_bench_t5_leg: CUDA error {rc}")
        return list(ms)

    def bench_sdpa_bf16(self, Q, K, V, bias, O, n_head, L, d_head, iters, warmup, flush, flush_bytes):
        """Per-call milliseconds of cudnn_sdpa_forward alone (events on stream 0, L2 flushed
        before each call outside the events)."""
        ms = (ctypes.c_double * iters)()
        rc = self.lib.ref_bench_sdpa_bf16(Q, K, V, bias, O, n_head, L, d_head, iters, warmup, flush, flush_bytes, ms)
        if rc != 0:
            raise RuntimeError(f"ref_bench_sdpa_bf16: CUDA error {rc}")
        return list(ms)


def available() -> dict:
    return {"oracle": ORACLE_PATH.exists(), "ref": REF_PATH.exists()}
