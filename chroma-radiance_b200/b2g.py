"""Python host side of the B200 GEMM engine, over its C ABI (include/b2g.h).

The functions mirror the reference's GEMM interface in cublas_ops.cuh — same names,
argument meaning and dtype rules — on torch CUDA tensors (torch is only the device-memory
and stream plumbing here; every byte of math runs in libb2g.so's kernels):

    linear(x, W, bias, out)                          cublas_ops.cuh:359-500
    linear_lt(M, K, N, x, x_type, w, w_type, bias, out)   cublas_ops.cuh:214-288
    linear_gated_residual(x, W, bias, residual, gate, M, N_out)   cublas_ops.cuh:684-723
    batched_matmul_Bt(A, B, C)                       cublas_ops.cuh:558-585

plus the engine's own fused entry point `gemm(...)` (bias / GELU / gated residual fused
into the tensor-core epilogue, bf16/fp16/F32 output).  Where the reference prints and
calls exit(1) on an error, these raise B2GError with the engine's message.  There is no
CPU fallback: without the library or a B200 every call raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libb2g.so"

# b2g_dtype
F32, F16, BF16, E4M3 = 0, 1, 2, 3
# cudaDataType_t values used by linear_lt's signature
CUDA_R_32F, CUDA_R_16F, CUDA_R_16BF = 0, 2, 14
# b2g_epilogue
EPI_NONE, EPI_GELU, EPI_GATED_RESIDUAL, EPI_SILU = 0, 1, 2, 3

_TORCH_TO_B2G = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
_TORCH_TO_CUDA = {torch.float32: CUDA_R_32F, torch.float16: CUDA_R_16F, torch.bfloat16: CUDA_R_16BF}
_EPILOGUES = {"none": EPI_NONE, "gelu": EPI_GELU, "gated_residual": EPI_GATED_RESIDUAL, "silu": EPI_SILU}


class B2GError(RuntimeError):
    """A non-OK b2g_status, with the library's message."""


class GemmDesc(ctypes.Structure):
    """Mirror of b2g_gemm_desc."""

    _fields_ = [
        ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
        ("a", ctypes.c_void_p), ("a_dtype", ctypes.c_int), ("lda", ctypes.c_int64),
        ("b", ctypes.c_void_p), ("b_dtype", ctypes.c_int), ("ldb", ctypes.c_int64),
        ("bias", ctypes.c_void_p), ("bias_dtype", ctypes.c_int),
        ("d", ctypes.c_void_p), ("d_dtype", ctypes.c_int), ("ldd", ctypes.c_int64),
        ("epilogue", ctypes.c_int),
        ("gate", ctypes.c_void_p),
    ]


class TpResidualSeg(ctypes.Structure):
    """Mirror of b2g_tp_residual_seg."""

    _fields_ = [("row0", ctypes.c_int64), ("rows", ctypes.c_int64), ("bias", ctypes.c_void_p),
                ("gate", ctypes.c_void_p), ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64)]


class TpReduceDesc(ctypes.Structure):
    """Mirror of b2g_tp_reduce_desc."""

    _fields_ = [
        ("world", ctypes.c_int), ("rank", ctypes.c_int),
        ("part_ptrs", ctypes.c_void_p), ("res_ptrs", ctypes.c_void_p),
        ("ld_part", ctypes.c_int64), ("ld_res", ctypes.c_int64),
        ("counters", ctypes.c_void_p), ("counter_slots", ctypes.c_int64),
    ]


class QkvRopeDesc(ctypes.Structure):
    """b2g_qkv_rope_desc: RoPE rows and RMSNorm scales of one qkv projection problem."""
    _fields_ = [("pe", ctypes.c_void_p), ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
                ("gelu_out", ctypes.c_void_p), ("gelu_ld", ctypes.c_int64), ("pe_period", ctypes.c_int64),
                ("a_scale", ctypes.c_void_p), ("b_scale", ctypes.c_void_p), ("pe_compact", ctypes.c_int64)]


_lib = None

# Exported symbols of libb2g.so with their ctypes signatures (status-returning unless noted).
_SIGNATURES = {
    "b2g_init": ([], ctypes.c_int),
    "b2g_shutdown": ([], ctypes.c_int),
    "b2g_last_error": ([], ctypes.c_char_p),
    "b2g_version": ([], ctypes.c_char_p),
    "b2g_gemm": ([ctypes.POINTER(GemmDesc), ctypes.c_void_p], ctypes.c_int),
    "b2g_gemm_group": ([ctypes.POINTER(GemmDesc), ctypes.c_int, ctypes.c_void_p], ctypes.c_int),
    "b2g_quantize_e4m3": ([ctypes.c_void_p, ctypes.c_int] + [ctypes.c_int64] * 3 + [ctypes.c_void_p, ctypes.c_int64,
                                                                                   ctypes.c_void_p, ctypes.c_void_p],
                          ctypes.c_int),
    "b2g_gemm_fp8": ([ctypes.POINTER(GemmDesc), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "b2g_gemm_fp8_group": ([ctypes.POINTER(GemmDesc), ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                            ctypes.c_int, ctypes.c_void_p], ctypes.c_int),
    "b2g_gemm_tp_reduce": ([ctypes.POINTER(GemmDesc), ctypes.POINTER(ctypes.c_int64), ctypes.c_int,
                            ctypes.POINTER(TpReduceDesc), ctypes.c_void_p], ctypes.c_int),
    "b2g_tp_push_rows": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                          ctypes.c_int, ctypes.c_void_p], ctypes.c_int),
    "b2g_tp_push_sums": ([ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                          ctypes.c_void_p], ctypes.c_int),
    "b2g_tp_reduce_slots": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                             ctypes.c_int, ctypes.c_void_p], ctypes.c_int),
    "b2g_tp_barrier": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p],
                       ctypes.c_int),
    "b2g_tp_scatter_rows": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                             ctypes.c_int, ctypes.c_void_p], ctypes.c_int),
    "b2g_tp_reduce_slots_bcast": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                   ctypes.c_int, ctypes.c_void_p], ctypes.c_int),
    "b2g_tp_barrier_next": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                             ctypes.c_void_p], ctypes.c_int),
    "b2g_tp_reduce_shard": ([ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_int, ctypes.c_int,
                                                                                       ctypes.c_void_p], ctypes.c_int),
    "b2g_tp_gather_residual": ([ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_int, ctypes.c_void_p,
                                                                          ctypes.c_int, ctypes.c_void_p], ctypes.c_int),
    "b2g_t5_attention": ([ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "b2g_bias_gated_residual": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_void_p], ctypes.c_int),
    "b2g_linear_lt": ([ctypes.c_int64] * 3 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                               ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "b2g_linear_lt_stream": ([ctypes.c_int64] * 3 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
                             ctypes.c_int),
    "b2g_linear_gated_residual": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_int64], ctypes.c_int),
    "b2g_batched_matmul_Bt": ([ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4, ctypes.c_int),
    "b2g_batched_matmul_Bt_stream": ([ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4 + [ctypes.c_void_p], ctypes.c_int),
    "b2g_patchify_bf16": ([ctypes.c_void_p] + [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p],
                          ctypes.c_int),
    "b2g_timestep_vec": ([ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p],
                         ctypes.c_int),
    "b2g_rms_norm": ([ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                      ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p], ctypes.c_int),
    "b2g_nerf_input_bf16": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                             ctypes.c_int64, ctypes.c_void_p], ctypes.c_int),
    "b2g_nerf_glu_weights": ([ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64] + [ctypes.c_void_p] * 4, ctypes.c_int),
    "b2g_convert_f32": ([ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                                                 ctypes.c_void_p], ctypes.c_int),
    "b2g_nerf_glu_block": ([ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                            ctypes.c_void_p], ctypes.c_int),
    "b2g_silu_mul": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p], ctypes.c_int),
    "b2g_add_inplace": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p], ctypes.c_int),
    "b2g_nerf_final": ([ctypes.c_void_p] * 5 + [ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                                 ctypes.c_void_p], ctypes.c_int),
    "b2g_check_device_error": ([ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "b2g_launch_count": ([], ctypes.c_uint64),
    "b2g_set_gemm_variant": ([ctypes.c_int, ctypes.c_int], ctypes.c_int),
    "b2g_set_attention_splits": ([ctypes.c_int], ctypes.c_int),
    "b2g_attention_qknorm_rope": ([ctypes.c_void_p, ctypes.c_int64] * 3 + [ctypes.c_void_p] * 4 +
                                  [ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_void_p], ctypes.c_int),
    "b2g_gemm_qkv_rope": ([ctypes.POINTER(GemmDesc), ctypes.POINTER(QkvRopeDesc), ctypes.c_int, ctypes.c_int,
                           ctypes.c_float, ctypes.c_void_p], ctypes.c_int),
    "b2g_attention_bf16": ([ctypes.c_void_p, ctypes.c_int64] * 3 + [ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                                   ctypes.c_int64, ctypes.c_void_p], ctypes.c_int),
    "b2g_attention_bf16_batched": ([ctypes.c_void_p, ctypes.c_int64] * 3 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                                                           ctypes.c_int, ctypes.c_void_p,
                                                                           ctypes.c_int64, ctypes.c_void_p, ctypes.c_int,
                                                                           ctypes.c_int64, ctypes.c_void_p],
                                   ctypes.c_int),
    "b2g_modulate_to_bf16": ([ctypes.c_void_p] * 4 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p],
                             ctypes.c_int),
    "b2g_modulate_streams": ([ctypes.c_void_p] * 5 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int,
                                                       ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                                       ctypes.c_void_p], ctypes.c_int),
    "b2g_modulate_to_e4m3": ([ctypes.c_void_p] * 5 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p],
                             ctypes.c_int),
    "b2g_attention_with_rope": ([ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p,
                                 ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
}


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Loads libb2g.so (once) and declares its signatures.  Raises B2GError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise B2GError(f"{p} is missing: build it with `python chroma-radiance_b200/build.py`")
    lib = ctypes.CDLL(str(p))
    for name, (args, res) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def _check(status: int) -> None:
    if status != 0:
        msg = _lib.b2g_last_error().decode(errors="replace")
        raise B2GError(f"b2g status {status}: {msg}")


def init() -> None:
    """Replaces init_cublas() (cublas_ops.cuh:152): validates the device (sm_100)."""
    _check(load().b2g_init())


def launch_count() -> int:
    """How many of the engine's kernels have been launched in this process."""
    return int(load().b2g_launch_count())


def set_gemm_variant(variant: int, splits: int = 0) -> None:
    """variant -1 automatic, 0 = 1-CTA 128x128, 1 = 1-CTA 128x256, 2 = 2-CTA 256x256 tiles;
    splits 0 automatic, > 0 the split-K factor of every tile, < 0 (-S) only the tiles of the
    last, partial wave split S ways."""
    _check(load().b2g_set_gemm_variant(variant, splits))


def set_attention_splits(splits: int) -> None:
    """Fused-attention key splits: 0 automatic, -1 never, > 0 that many slices."""
    _check(load().b2g_set_attention_splits(splits))


def check_device_error() -> None:
    """Synchronises and raises if a kernel gave up on a pipeline wait (then clears it)."""
    code = ctypes.c_int(0)
    _check(load().b2g_check_device_error(ctypes.byref(code)))


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise B2GError("all tensors must be CUDA tensors")


def _operand_dtype(t: torch.Tensor) -> int:
    """b2g dtype of a GEMM operand: uint8 tensors hold E4M3 codes."""
    return E4M3 if t.dtype == torch.uint8 else _TORCH_TO_B2G[t.dtype]


def _gemm_desc(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, out: torch.Tensor | None,
               out_dtype: torch.dtype | None, epilogue: str, gate: torch.Tensor | None) -> tuple[GemmDesc, torch.Tensor]:
    _require_cuda(x, w, bias, out, gate)
    if x.dim() != 2 or w.dim() != 2 or x.stride(1) != 1 or w.stride(1) != 1:
        raise B2GError("gemm: x and w must be 2-D with unit stride along K")
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise B2GError(f"gemm: K mismatch {tuple(x.shape)} vs {tuple(w.shape)}")
    epi = _EPILOGUES[epilogue]
    if out is None:
        if epi == EPI_GATED_RESIDUAL:
            raise B2GError("gemm: gated_residual needs `out` (the residual)")
        out = torch.empty((M, N), device=x.device, dtype=out_dtype or torch.float32)
    if out.dim() != 2 or out.shape != (M, N) or out.stride(1) != 1:
        raise B2GError("gemm: out must be [M, N] with unit column stride")
    d = GemmDesc()
    d.M, d.N, d.K = M, N, K
    d.a, d.a_dtype, d.lda = x.data_ptr(), _operand_dtype(x), x.stride(0) if M > 1 else K
    d.b, d.b_dtype, d.ldb = w.data_ptr(), _operand_dtype(w), w.stride(0) if N > 1 else K
    d.bias = _ptr(bias)
    d.bias_dtype = _TORCH_TO_B2G[bias.dtype] if bias is not None else F32
    d.d, d.d_dtype, d.ldd = out.data_ptr(), _TORCH_TO_B2G[out.dtype], out.stride(0) if M > 1 else N
    d.epilogue = epi
    d.gate = _ptr(gate)
    return d, out


def gemm(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
         out_dtype: torch.dtype | None = None, epilogue: str = "none", gate: torch.Tensor | None = None,
         stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """out[M, N] = epilogue(x[M, K] . w[N, K]^T + bias) on the tensor-core path.

    x, w: 2-D, unit stride along K (row strides may exceed K).  epilogue: "none", "gelu"
    (tanh GELU), "silu" or "gated_residual" (out is an F32 residual updated in place:
    out += gate * (x.w^T + bias)).  Runs on `stream` (default: torch's current stream).
    """
    lib = load()
    d, out = _gemm_desc(x, w, bias, out, out_dtype, epilogue, gate)
    s = (stream or torch.cuda.current_stream(x.device)).cuda_stream
    _check(lib.b2g_gemm(ctypes.byref(d), ctypes.c_void_p(s)))
    return out


def gemm_group(problems: list[dict], stream: torch.cuda.Stream | None = None) -> list[torch.Tensor]:
    """Several gemm() problems (dicts of gemm's keyword arguments, x and w required) in one
    call; two to four that share N, K, dtypes and epilogue run as one tensor-core launch."""
    lib = load()
    descs, outs = [], []
    for pr in problems:
        d, out = _gemm_desc(pr["x"], pr["w"], pr.get("bias"), pr.get("out"), pr.get("out_dtype"),
                            pr.get("epilogue", "none"), pr.get("gate"))
        descs.append(d)
        outs.append(out)
    arr = (GemmDesc * len(descs))(*descs)
    dev = problems[0]["x"].device if problems else torch.device("cuda")
    s = (stream or torch.cuda.current_stream(dev)).cuda_stream
    _check(lib.b2g_gemm_group(arr, len(descs), ctypes.c_void_p(s)))
    return outs


def _q8_outputs(rows: int, cols: int, dev, out, scales, who: str) -> tuple[torch.Tensor, torch.Tensor]:
    """Caller-given (or new) uint8 [rows, cols] code and F32 [rows] scale buffers."""
    q = out if out is not None else torch.empty((rows, cols), dtype=torch.uint8, device=dev)
    sc = scales if scales is not None else torch.empty(rows, dtype=torch.float32, device=dev)
    _require_cuda(q, sc)
    if (q.dtype != torch.uint8 or q.shape != (rows, cols) or q.stride(1) != 1 or sc.dtype != torch.float32 or
            sc.shape != (rows,) or not sc.is_contiguous()):
        raise B2GError(f"{who}: out must be uint8 [rows, cols] (unit column stride), scales F32 [rows]")
    return q, sc


def quantize_e4m3(x: torch.Tensor, out: torch.Tensor | None = None, scales: torch.Tensor | None = None,
                  stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row E4M3 quantisation of a 2-D F32/BF16/F16 CUDA tensor: (codes uint8 [rows, cols],
    scales f32 [rows]) with scales = absmax/448 and codes = E4M3(x * 448/absmax); into `out` and
    `scales` when given."""
    lib = load()
    _require_cuda(x)
    if x.dim() != 2 or x.stride(1) != 1:
        raise B2GError("quantize_e4m3: 2-D tensor with unit column stride expected")
    rows, cols = x.shape
    q, sc = _q8_outputs(rows, cols, x.device, out, scales, "quantize_e4m3")
    s = (stream or torch.cuda.current_stream(x.device)).cuda_stream
    _check(lib.b2g_quantize_e4m3(x.data_ptr(), _TORCH_TO_B2G[x.dtype], rows, cols, x.stride(0) if rows > 1 else cols,
                                 q.data_ptr(), q.stride(0) if rows > 1 else cols, sc.data_ptr(), ctypes.c_void_p(s)))
    return q, sc


def gemm_fp8(x: torch.Tensor, wq: torch.Tensor, w_scale: torch.Tensor, bias: torch.Tensor | None = None,
             out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None, epilogue: str = "none",
             gate: torch.Tensor | None = None, x_scale: torch.Tensor | None = None,
             stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """FP8 linear: out = epilogue((x . wq^T) * x_scale[m] * w_scale[n] + bias).

    wq: uint8 E4M3 codes [N, K] from quantize_e4m3 (w_scale its scales).  x: uint8 E4M3 codes
    with x_scale, or F32/BF16/F16 activations that the library quantises per token."""
    lib = load()
    _require_cuda(x, wq, w_scale, bias, out, gate, x_scale)
    if x.dim() != 2 or wq.dim() != 2 or x.stride(1) != 1 or wq.stride(1) != 1 or wq.dtype != torch.uint8:
        raise B2GError("gemm_fp8: 2-D x and uint8 wq with unit stride along K expected")
    M, K = x.shape
    N = wq.shape[0]
    if wq.shape[1] != K:
        raise B2GError("gemm_fp8: K mismatch")
    epi = _EPILOGUES[epilogue]
    if out is None:
        if epi == EPI_GATED_RESIDUAL:
            raise B2GError("gemm_fp8: gated_residual needs `out` (the residual)")
        out = torch.empty((M, N), device=x.device, dtype=out_dtype or torch.float32)
    d = GemmDesc()
    d.M, d.N, d.K = M, N, K
    d.a, d.lda = x.data_ptr(), x.stride(0) if M > 1 else K
    d.a_dtype = E4M3 if x.dtype == torch.uint8 else _TORCH_TO_B2G[x.dtype]
    d.b, d.b_dtype, d.ldb = wq.data_ptr(), E4M3, wq.stride(0) if N > 1 else K
    d.bias = _ptr(bias)
    d.bias_dtype = _TORCH_TO_B2G[bias.dtype] if bias is not None else F32
    d.d, d.d_dtype, d.ldd = out.data_ptr(), _TORCH_TO_B2G[out.dtype], out.stride(0) if M > 1 else N
    d.epilogue = epi
    d.gate = _ptr(gate)
    s = (stream or torch.cuda.current_stream(x.device)).cuda_stream
    _check(lib.b2g_gemm_fp8(ctypes.byref(d), _ptr(x_scale), w_scale.data_ptr(), ctypes.c_void_p(s)))
    return out


def gemm_fp8_group(problems: list[dict], stream: torch.cuda.Stream | None = None) -> list[torch.Tensor]:
    """Up to four FP8 linears in one call (b2g_gemm_fp8_group): dicts with x (uint8 E4M3 codes),
    x_scale, w (uint8 codes), w_scale and gemm()'s bias / out / out_dtype / epilogue / gate;
    those that share N, K and epilogue run as one tensor-core launch."""
    lib = load()
    descs, outs, a_sc, b_sc = [], [], [], []
    for pr in problems:
        x, w = pr["x"], pr["w"]
        if x.dtype != torch.uint8 or w.dtype != torch.uint8:
            raise B2GError("gemm_fp8_group: uint8 E4M3 x and w expected")
        _require_cuda(pr["x_scale"], pr["w_scale"])
        d, out = _gemm_desc(x, w, pr.get("bias"), pr.get("out"), pr.get("out_dtype"), pr.get("epilogue", "none"),
                            pr.get("gate"))
        descs.append(d)
        outs.append(out)
        a_sc.append(pr["x_scale"].data_ptr())
        b_sc.append(pr["w_scale"].data_ptr())
    n = len(descs)
    arr = (GemmDesc * n)(*descs)
    dev = problems[0]["x"].device if problems else torch.device("cuda")
    s = (stream or torch.cuda.current_stream(dev)).cuda_stream
    _check(lib.b2g_gemm_fp8_group(arr, (ctypes.c_void_p * n)(*a_sc), (ctypes.c_void_p * n)(*b_sc), n,
                                  ctypes.c_void_p(s)))
    return outs


def gemm_tp_reduce(problems: list[dict], row0: list[int], tp: TpReduceDesc,
                   stream: torch.cuda.Stream | None = None) -> None:
    """Row-split layer with the tensor-parallel reduction fused in (b2g_gemm_tp_reduce):
    problems = [dict(x=, w=, bias=, gate=)] (this rank's K-slice), row0 = their first rows in
    the peer-mapped partial / residual buffers described by `tp`."""
    lib = load()
    descs = []
    for pr in problems:
        x, w = pr["x"], pr["w"]
        _require_cuda(x, w, pr.get("bias"), pr["gate"])
        if x.dim() != 2 or w.dim() != 2 or x.stride(1) != 1 or w.stride(1) != 1 or w.shape[1] != x.shape[1]:
            raise B2GError("gemm_tp_reduce: 2-D x [M, K] and w [N, K] with unit stride along K expected")
        d = GemmDesc()
        d.M, d.K, d.N = x.shape[0], x.shape[1], w.shape[0]
        d.a, d.a_dtype, d.lda = x.data_ptr(), _TORCH_TO_B2G[x.dtype], x.stride(0) if x.shape[0] > 1 else x.shape[1]
        d.b, d.b_dtype, d.ldb = w.data_ptr(), _TORCH_TO_B2G[w.dtype], w.stride(0)
        d.bias = _ptr(pr.get("bias"))
        d.bias_dtype = F32
        d.d, d.d_dtype, d.ldd = None, F32, d.N
        d.epilogue = EPI_GATED_RESIDUAL
        d.gate = pr["gate"].data_ptr()
        descs.append(d)
    arr = (GemmDesc * len(descs))(*descs)
    rows = (ctypes.c_int64 * len(row0))(*row0)
    s = (stream or torch.cuda.current_stream(problems[0]["x"].device)).cuda_stream
    _check(lib.b2g_gemm_tp_reduce(arr, rows, len(descs), ctypes.byref(tp), ctypes.c_void_p(s)))


def tp_push_rows(part: torch.Tensor, recv_ptrs: list[int], world: int, rank: int,
                 stream: torch.cuda.Stream | None = None) -> None:
    """Push form, step 1 (b2g_tp_push_rows): this rank's bf16 partial [rows, N] (contiguous) into
    every owner's receive slot `rank` by copy-engine copies (recv_ptrs: the ranks' addresses)."""
    rows, N = part.shape
    arr = (ctypes.c_void_p * world)(*recv_ptrs)
    s = (stream or torch.cuda.current_stream(part.device)).cuda_stream
    _check(load().b2g_tp_push_rows(part.data_ptr(), arr, rows, N, world, rank, ctypes.c_void_p(s)))


def tp_push_sums(sum_ptrs: list[int], sum_buf: torch.Tensor, world: int, rank: int,
                 stream: torch.cuda.Stream | None = None) -> None:
    """Push form, step 3 (b2g_tp_push_sums): this rank's rows of its sums into every other rank's
    by copy-engine copies (sum_ptrs: the ranks' addresses)."""
    rows, N = sum_buf.shape
    arr = (ctypes.c_void_p * world)(*sum_ptrs)
    s = (stream or torch.cuda.current_stream(sum_buf.device)).cuda_stream
    _check(load().b2g_tp_push_sums(arr, rows, N, world, rank, ctypes.c_void_p(s)))


def tp_reduce_slots(recv: torch.Tensor, sum_buf: torch.Tensor, world: int, rank: int,
                    stream: torch.cuda.Stream | None = None) -> None:
    """Phase 1 of the reduce-scatter form (b2g_tp_reduce_slots): recv this rank's bf16
    [world, shard, N] receive buffer, sum_buf its bf16 [rows, N] sums."""
    rows, N = sum_buf.shape
    s = (stream or torch.cuda.current_stream(sum_buf.device)).cuda_stream
    _check(load().b2g_tp_reduce_slots(recv.data_ptr(), sum_buf.data_ptr(), rows, N, world, rank, ctypes.c_void_p(s)))


def tp_scatter_rows(part: torch.Tensor, recv_ptrs: torch.Tensor, world: int, rank: int,
                    stream: torch.cuda.Stream | None = None) -> None:
    """Store form, step 1 (b2g_tp_scatter_rows): this rank's bf16 partial [rows, N] (contiguous)
    into every owner's receive slot `rank` by SM stores; recv_ptrs an int64 CUDA tensor of the
    ranks' receive-buffer addresses."""
    rows, N = part.shape
    s = (stream or torch.cuda.current_stream(part.device)).cuda_stream
    _check(load().b2g_tp_scatter_rows(part.data_ptr(), recv_ptrs.data_ptr(), rows, N, world, rank,
                                      ctypes.c_void_p(s)))


def tp_reduce_slots_bcast(recv: torch.Tensor, sum_ptrs: torch.Tensor, rows: int, N: int, world: int, rank: int,
                          stream: torch.cuda.Stream | None = None) -> None:
    """Store form, step 2 (b2g_tp_reduce_slots_bcast): the sum of this rank's receive slots
    (recv bf16 [world, shard, N]) stored into every rank's sum buffer [rows, N] (sum_ptrs an
    int64 CUDA tensor of their addresses)."""
    s = (stream or torch.cuda.current_stream(recv.device)).cuda_stream
    _check(load().b2g_tp_reduce_slots_bcast(recv.data_ptr(), sum_ptrs.data_ptr(), rows, N, world, rank,
                                            ctypes.c_void_p(s)))


def tp_reduce_shard(part_ptrs: torch.Tensor, sum_buf: torch.Tensor, world: int, rank: int,
                    stream: torch.cuda.Stream | None = None) -> None:
    """Phase 1 of the peer-memory all-reduce (b2g_tp_reduce_shard): part_ptrs an int64 CUDA
    tensor of every rank's bf16 partial [rows, N] address; sum_buf this rank's bf16 [rows, N]."""
    rows, N = sum_buf.shape
    s = (stream or torch.cuda.current_stream(sum_buf.device)).cuda_stream
    _check(load().b2g_tp_reduce_shard(part_ptrs.data_ptr(), sum_buf.data_ptr(), sum_buf.stride(0), rows, N, world,
                                      rank, ctypes.c_void_p(s)))


def tp_gather_residual(sum_ptrs: torch.Tensor, sum_buf: torch.Tensor, world: int, segments: list[dict],
                       stream: torch.cuda.Stream | None = None) -> None:
    """Phase 2 (b2g_tp_gather_residual): segments of dict(row0, bias, gate, residual) with the
    residual F32 [rows, N] of sum rows [row0, row0 + rows)."""
    rows, N = sum_buf.shape
    segs = (TpResidualSeg * len(segments))()
    for i, g in enumerate(segments):
        r = g["residual"]
        _require_cuda(r, g["gate"], g.get("bias"))
        segs[i] = TpResidualSeg(g["row0"], r.shape[0], _ptr(g.get("bias")), g["gate"].data_ptr(), r.data_ptr(),
                                r.stride(0))
    s = (stream or torch.cuda.current_stream(sum_buf.device)).cuda_stream
    _check(load().b2g_tp_gather_residual(sum_ptrs.data_ptr(), sum_buf.stride(0), rows, N, world, segs, len(segments),
                                         ctypes.c_void_p(s)))


def tp_barrier(flag_ptrs: torch.Tensor, own_flags: torch.Tensor, world: int, rank: int, epoch: int,
               stream: torch.cuda.Stream | None = None) -> None:
    """Cross-rank barrier (b2g_tp_barrier): flag_ptrs an int64 CUDA tensor of every rank's flag
    array address, own_flags this rank's int32 [world] array."""
    lib = load()
    s = (stream or torch.cuda.current_stream(own_flags.device)).cuda_stream
    _check(lib.b2g_tp_barrier(flag_ptrs.data_ptr(), own_flags.data_ptr(), world, rank, epoch, ctypes.c_void_p(s)))


def tp_barrier_next(flag_ptrs: torch.Tensor, own_flags: torch.Tensor, epoch_counter: torch.Tensor, world: int,
                    rank: int, stream: torch.cuda.Stream | None = None) -> None:
    """The cross-rank barrier with its epoch held in device memory (b2g_tp_barrier_next):
    epoch_counter this rank's own int32 [1] CUDA tensor, zero before the first call.  Safe to
    capture in a CUDA graph: every replay waits on the next epoch."""
    s = (stream or torch.cuda.current_stream(own_flags.device)).cuda_stream
    _check(load().b2g_tp_barrier_next(flag_ptrs.data_ptr(), own_flags.data_ptr(), epoch_counter.data_ptr(), world,
                                      rank, ctypes.c_void_p(s)))


def t5_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, rel_bias: torch.Tensor | None, n_head: int,
                 d_head: int, scale: float = 1.0, attn_mask: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """t5_attention (attention.cuh:34-91): Q, K, V F32 [L, n_head, d_head] contiguous; rel_bias
    [n_head, L, L] or None; attn_mask [L] or None -> F32 [L, n_head*d_head]."""
    lib = load()
    _require_cuda(Q, K, V, rel_bias, attn_mask, out)
    L = Q.shape[0]
    for t in (Q, K, V):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != L * n_head * d_head:
            raise B2GError("t5_attention: contiguous F32 [L, n_head, d_head] tensors expected")
    if out is None:
        out = torch.empty((L, n_head * d_head), dtype=torch.float32, device=Q.device)
    s = torch.cuda.current_stream(Q.device).cuda_stream
    _check(lib.b2g_t5_attention(Q.data_ptr(), K.data_ptr(), V.data_ptr(), _ptr(rel_bias), n_head, d_head, L, scale,
                                _ptr(attn_mask), out.data_ptr(), ctypes.c_void_p(s)))
    return out


def bias_gated_residual(y: torch.Tensor, bias: torch.Tensor | None, gate: torch.Tensor, residual: torch.Tensor,
                        stream: torch.cuda.Stream | None = None) -> None:
    """residual[m, n] += gate[n] * (y[m, n] + bias[n]) (y BF16 or F32 [M, N], residual F32)."""
    lib = load()
    _require_cuda(y, bias, gate, residual)
    M, N = residual.shape
    if y.shape != (M, N) or y.stride(1) != 1 or residual.stride(1) != 1 or residual.dtype != torch.float32:
        raise B2GError("bias_gated_residual: y [M, N] and F32 residual [M, N] with unit column stride expected")
    s = (stream or torch.cuda.current_stream(y.device)).cuda_stream
    _check(lib.b2g_bias_gated_residual(y.data_ptr(), _TORCH_TO_B2G[y.dtype], y.stride(0) if M > 1 else N, _ptr(bias),
                                       gate.data_ptr(), residual.data_ptr(), residual.stride(0) if M > 1 else N, M, N,
                                       ctypes.c_void_p(s)))


def linear_lt(M: int, K: int, N: int, x: torch.Tensor, x_type: int, w: torch.Tensor, w_type: int,
              bias: torch.Tensor | None, out: torch.Tensor) -> None:
    """linear_lt (cublas_ops.cuh:214): out[M,N] F32 = x[M,K] . w[N,K]^T + bias (F32 or None).

    x_type/w_type are cudaDataType_t codes (CUDA_R_32F, CUDA_R_16F, CUDA_R_16BF); runs on the
    legacy default stream like the reference.
    """
    lib = load()
    _require_cuda(x, w, bias, out)
    _check(lib.b2g_linear_lt(M, K, N, x.data_ptr(), x_type, w.data_ptr(), w_type, _ptr(bias), out.data_ptr()))


def linear(x: torch.Tensor, W: torch.Tensor, bias: torch.Tensor | None, output: torch.Tensor) -> None:
    """linear (cublas_ops.cuh:359): output (F32, numel M*N) = x . W^T + bias.

    M = x.numel() / x.shape[-1].  Like the reference, the bias is used only when it is an F32
    tensor, and F32 activations with BF16/FP16 weights are rounded to the weight dtype first.
    """
    lib = load()
    _require_cuda(x, W, bias, output)
    if W.dim() != 2 or x.shape[-1] != W.shape[1]:
        raise B2GError("linear: W must be [N, K] with K = x.shape[-1]")
    K = x.shape[-1]
    M = x.numel() // K if K else 0
    N = W.shape[0]
    if output.numel() != M * N or output.dtype != torch.float32:
        raise B2GError("linear: output must be F32 with M*N elements")
    if not (x.is_contiguous() and W.is_contiguous() and output.is_contiguous()):
        raise B2GError("linear: tensors must be contiguous")
    b = bias if (bias is not None and bias.dtype == torch.float32) else None
    xt, wt = x.dtype, W.dtype
    if not (xt == wt or (xt == torch.float32 and wt in (torch.bfloat16, torch.float16))):
        raise B2GError(f"Unsupported dtype combo in linear: x={xt} W={wt}")
    d = GemmDesc()
    d.M, d.N, d.K = M, N, K
    d.a, d.a_dtype, d.lda = x.data_ptr(), _TORCH_TO_B2G[xt], K
    d.b, d.b_dtype, d.ldb = W.data_ptr(), _TORCH_TO_B2G[wt], K
    d.bias, d.bias_dtype = _ptr(b), F32
    d.d, d.d_dtype, d.ldd = output.data_ptr(), F32, N
    d.epilogue = EPI_NONE
    _check(lib.b2g_gemm(ctypes.byref(d), ctypes.c_void_p(0)))


def linear_gated_residual(x: torch.Tensor, W: torch.Tensor, bias: torch.Tensor | None,
                          residual_inout: torch.Tensor, gate: torch.Tensor, M: int, N_out: int) -> None:
    """linear_gated_residual (cublas_ops.cuh:684): residual += gate * (x . W^T + bias), one kernel."""
    lib = load()
    _require_cuda(x, W, bias, residual_inout, gate)
    K = x.shape[-1]
    b = bias if (bias is not None and bias.dtype == torch.float32) else None
    _check(lib.b2g_linear_gated_residual(x.data_ptr(), _TORCH_TO_CUDA[x.dtype], W.data_ptr(),
                                         _TORCH_TO_CUDA[W.dtype], _ptr(b), residual_inout.data_ptr(),
                                         gate.data_ptr(), M, K, N_out))


def attention_with_rope(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, pe: torch.Tensor, n_head: int,
                        d_head: int, attn_mask: torch.Tensor | None = None,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """attention_with_rope (attention.cuh:23): F32 [L, n_head, d_head] Q/K/V -> F32 [L, n_head*d_head]."""
    lib = load()
    _require_cuda(Q, K, V, pe, attn_mask, out)
    L = Q.shape[0]
    for t in (Q, K, V, pe):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise B2GError("attention_with_rope: contiguous F32 tensors expected")
    if out is None:
        out = torch.empty((L, n_head * d_head), dtype=torch.float32, device=Q.device)
    s = torch.cuda.current_stream(Q.device).cuda_stream
    _check(lib.b2g_attention_with_rope(Q.data_ptr(), K.data_ptr(), V.data_ptr(), pe.data_ptr(), n_head, d_head, L,
                                       _ptr(attn_mask), out.data_ptr(), ctypes.c_void_p(s)))
    return out


def attention_qknorm_rope(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pe: torch.Tensor, n_head: int,
                          d_head: int, q_norm: torch.Tensor | None = None, k_norm: torch.Tensor | None = None,
                          attn_mask: torch.Tensor | None = None, out: torch.Tensor | None = None,
                          out_dtype: torch.dtype = torch.float32, eps: float = 1e-6,
                          q_norm2: torch.Tensor | None = None, k_norm2: torch.Tensor | None = None,
                          norm_split: int = -1) -> torch.Tensor:
    """Fused block-path attention: q/k/v are [L, n_head*d_head] F32 views (unit column
    stride, any row stride); optional per-head RMSNorm scales (q_norm2/k_norm2 for rows
    >= norm_split); output F32 or bf16 view."""
    lib = load()
    _require_cuda(q, k, v, pe, q_norm, k_norm, q_norm2, k_norm2, attn_mask, out)
    L = q.shape[0]
    for t in (q, k, v):
        if t.dtype != torch.float32 or t.stride(1) != 1:
            raise B2GError("attention_qknorm_rope: F32 views with unit column stride expected")
    if out is None:
        out = torch.empty((L, n_head * d_head), dtype=out_dtype, device=q.device)
    s = torch.cuda.current_stream(q.device).cuda_stream
    _check(lib.b2g_attention_qknorm_rope(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(),
                                         v.stride(0), _ptr(q_norm), _ptr(k_norm), _ptr(q_norm2), _ptr(k_norm2),
                                         norm_split, eps, pe.data_ptr(),
                                         _ptr(attn_mask), out.data_ptr(), _TORCH_TO_B2G[out.dtype], out.stride(0),
                                         L, n_head, d_head, ctypes.c_void_p(s)))
    return out


def gemm_qkv_rope(problems: list[dict], n_head: int, eps: float = 1e-6,
                  stream: torch.cuda.Stream | None = None) -> list[torch.Tensor]:
    """Attention input projections with qk_norm and RoPE in the GEMM epilogue.

    Each problem: x [M, K] and w [3*n_head*128, K] (bf16/fp16), bias (F32), out (bf16 [M, N]
    view with 16-byte aligned rows; allocated when absent), pe (F32 RoPE rows of the
    problem's tokens, [M, 64, 4] or [M, 256]), q_norm / k_norm ([128] F32 or None), and
    pe may also be [M, 64, 2] (cos, sin) per pair, for tables of the rotation form (cos, -sin,
    sin, cos): the same result from half the bytes (compact_rope_table).  Optionally
    pe_period P (row m uses pe row m % P; pe then needs P rows only: stacked
    guidance halves of one sequence).  Output columns [q | k | v]: q and k heads normed and
    rotated, v the plain product (+ bias).  Up to four problems (txt and img streams, times
    the guidance halves) run as one launch.  FP8 form: x and w uint8 E4M3 codes with x_scale
    (per row) and w_scale (per output channel, from quantize_e4m3).  One problem may carry gelu_out (a
    bf16 [M, N - 3*n_head*128] view): w then has more rows, and those columns get bias + GELU
    into gelu_out (the single block's linear1 in one launch); out holds the qkv columns.
    """
    lib = load()
    descs, ropes, outs, keep = [], [], [], []
    for pr in problems:
        out = pr.get("out")
        qkv_cols = 3 * n_head * 128
        tail = pr.get("gelu_out")
        if out is None:
            out = torch.empty((pr["x"].shape[0], qkv_cols if tail is not None else pr["w"].shape[0]),
                              device=pr["x"].device, dtype=torch.bfloat16)
        if tail is not None:
            _require_cuda(tail)
            if (tail.dtype != torch.bfloat16 or tail.stride(1) != 1 or
                    tail.shape != (pr["x"].shape[0], pr["w"].shape[0] - qkv_cols)):
                raise B2GError("gemm_qkv_rope: gelu_out must be a bf16 [M, N - 3*n_head*128] view")
            d, _ = _gemm_desc(pr["x"], pr["w"][:qkv_cols], pr.get("bias"), out, None, "none", None)
            d.N = pr["w"].shape[0]
        else:
            d, out = _gemm_desc(pr["x"], pr["w"], pr.get("bias"), out, None, "none", None)
        pe = pr["pe"]
        qn, kn = pr.get("q_norm"), pr.get("k_norm")
        _require_cuda(pe, qn, kn)
        for t in (pe, qn, kn):
            if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
                raise B2GError("gemm_qkv_rope: pe and norm scales must be contiguous F32")
        period = int(pr.get("pe_period") or 0)
        if period < 0:
            raise B2GError("gemm_qkv_rope: pe_period must be 0 or positive")
        compact = pe.dim() == 3 and pe.shape[-1] == 2
        if pe.numel() < (period or pr["x"].shape[0]) * (128 if compact else 256):
            raise B2GError("gemm_qkv_rope: pe must hold 256 floats ([64, 4]), or 128 ([64, 2] cos/sin), per row "
                           "of x (per pe_period row)")
        xs, ws = pr.get("x_scale"), pr.get("w_scale")
        if pr["x"].dtype == torch.uint8:
            _require_cuda(xs, ws)
            if xs is None or ws is None or pr["w"].dtype != torch.uint8:
                raise B2GError("gemm_qkv_rope: E4M3 x needs x_scale, and uint8 w with w_scale")
        descs.append(d)
        ropes.append(QkvRopeDesc(pe.data_ptr(), _ptr(qn), _ptr(kn), _ptr(tail),
                                 tail.stride(0) if tail is not None else 0, period, _ptr(xs), _ptr(ws),
                                 1 if compact else 0))
        outs.append(out)
        keep.append(pe)
    arr = (GemmDesc * len(descs))(*descs)
    rarr = (QkvRopeDesc * len(ropes))(*ropes)
    dev = problems[0]["x"].device
    s = (stream or torch.cuda.current_stream(dev)).cuda_stream
    _check(lib.b2g_gemm_qkv_rope(arr, rarr, len(descs), n_head, eps, ctypes.c_void_p(s)))
    return outs


def attention_bf16(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, n_head: int, d_head: int,
                   attn_mask: torch.Tensor | None = None, out: torch.Tensor | None = None,
                   out_dtype: torch.dtype = torch.float32, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Fused attention on bf16 [L, n_head*d_head] views (unit column stride, row strides a
    multiple of 8): softmax(q k^T / sqrt(d_head) + attn_mask[key]) v per head."""
    lib = load()
    _require_cuda(q, k, v, attn_mask, out)
    L = q.shape[0]
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or t.stride(1) != 1 or t.shape[0] != L:
            raise B2GError("attention_bf16: bf16 [L, H*D] views with unit column stride expected")
    if out is None:
        out = torch.empty((L, n_head * d_head), dtype=out_dtype, device=q.device)
    s = (stream or torch.cuda.current_stream(q.device)).cuda_stream
    _check(lib.b2g_attention_bf16(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                                  L, n_head, d_head, _ptr(attn_mask), out.data_ptr(), _TORCH_TO_B2G[out.dtype],
                                  out.stride(0), ctypes.c_void_p(s)))
    return out


def attention_bf16_batched(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, n_head: int, d_head: int,
                           batch: int, attn_mask: torch.Tensor | None = None, out: torch.Tensor | None = None,
                           out_dtype: torch.dtype = torch.float32,
                           stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """attention_bf16 over `batch` sequences stacked in the rows of q, k, v (and out): sequence
    b is rows [b*L, (b+1)*L) with L = rows / batch and attends only within itself.  attn_mask:
    None, one [L] bias for every sequence, or [batch, L] (contiguous)."""
    lib = load()
    _require_cuda(q, k, v, attn_mask, out)
    R = q.shape[0]
    if batch < 1 or R % batch != 0:
        raise B2GError("attention_bf16_batched: rows must be whole sequences")
    L = R // batch
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or t.stride(1) != 1 or t.shape[0] != R:
            raise B2GError("attention_bf16_batched: bf16 [batch*L, H*D] views with unit column stride expected")
    stride = 0
    if attn_mask is not None:
        if attn_mask.dtype != torch.float32 or not attn_mask.is_contiguous():
            raise B2GError("attention_bf16_batched: attn_mask must be contiguous F32")
        if attn_mask.dim() == 2:
            if tuple(attn_mask.shape) != (batch, L):
                raise B2GError("attention_bf16_batched: attn_mask must be [L] or [batch, L]")
            stride = L
        elif attn_mask.numel() != L:
            raise B2GError("attention_bf16_batched: attn_mask must be [L] or [batch, L]")
    if out is None:
        out = torch.empty((R, n_head * d_head), dtype=out_dtype, device=q.device)
    s = (stream or torch.cuda.current_stream(q.device)).cuda_stream
    _check(lib.b2g_attention_bf16_batched(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(),
                                          v.stride(0), L, batch, n_head, d_head, _ptr(attn_mask), stride,
                                          out.data_ptr(), _TORCH_TO_B2G[out.dtype], out.stride(0),
                                          ctypes.c_void_p(s)))
    return out


def _modulate_args(x, shift, scale):
    _require_cuda(x, shift, scale)
    for t in (x, shift, scale):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise B2GError("modulate: contiguous F32 x, shift and scale expected")
    if x.dim() != 2 or shift.numel() != x.shape[1] or scale.numel() != x.shape[1]:
        raise B2GError("modulate: x [M, C] with shift and scale [C]")
    return x.shape


def modulate_to_bf16(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6,
                     out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """modulate_to_bf16 (kernels.cu:552-599): bf16(LayerNorm(x) * (1 + scale) + shift), x [M, C] F32."""
    lib = load()
    M, C = _modulate_args(x, shift, scale)
    if out is None:
        out = torch.empty((M, C), dtype=torch.bfloat16, device=x.device)
    if out.dtype != torch.bfloat16 or not out.is_contiguous() or out.shape != (M, C):
        raise B2GError("modulate_to_bf16: contiguous bf16 out [M, C] expected")
    s = (stream or torch.cuda.current_stream(x.device)).cuda_stream
    _check(lib.b2g_modulate_to_bf16(x.data_ptr(), shift.data_ptr(), scale.data_ptr(), out.data_ptr(), M, C, eps,
                                    ctypes.c_void_p(s)))
    return out


def modulate_to_e4m3(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6,
                     out: torch.Tensor | None = None, scales: torch.Tensor | None = None,
                     stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """The modulated rows quantised per row to E4M3: (codes uint8 [M, C], row scales f32 [M]),
    into `out` (contiguous) and `scales` when given."""
    lib = load()
    M, C = _modulate_args(x, shift, scale)
    codes, rs = _q8_outputs(M, C, x.device, out, scales, "modulate_to_e4m3")
    if not codes.is_contiguous():
        raise B2GError("modulate_to_e4m3: out must be contiguous")
    s = (stream or torch.cuda.current_stream(x.device)).cuda_stream
    _check(lib.b2g_modulate_to_e4m3(x.data_ptr(), shift.data_ptr(), scale.data_ptr(), codes.data_ptr(),
                                    rs.data_ptr(), M, C, eps, ctypes.c_void_p(s)))
    return codes, rs


def batched_matmul_Bt(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
                      stream: torch.cuda.Stream | None = None) -> None:
    """batched_matmul_Bt (cublas_ops.cuh:558): C[b] = A[b] . B[b]^T, F32, operands rounded to TF32
    (as cuBLAS runs the reference's CUBLAS_COMPUTE_32F_FAST_16BF on B200), fp32 accumulation.
    On `stream` (default: torch's current stream)."""
    lib = load()
    _require_cuda(A, B, C)
    if A.dim() != 3 or B.dim() != 3 or C.dim() != 3:
        raise B2GError("batched_matmul_Bt: 3-D tensors expected")
    batch, M, K = A.shape
    N = B.shape[1]
    if B.shape != (batch, N, K) or C.shape != (batch, M, N):
        raise B2GError("batched_matmul_Bt: shape mismatch")
    if not all(t.dtype == torch.float32 and t.is_contiguous() for t in (A, B, C)):
        raise B2GError("batched_matmul_Bt: contiguous F32 tensors expected")
    s = (stream or torch.cuda.current_stream(A.device)).cuda_stream
    _check(lib.b2g_batched_matmul_Bt_stream(A.data_ptr(), B.data_ptr(), C.data_ptr(), batch, M, K, N,
                                            ctypes.c_void_p(s)))


def modulate_streams(x: torch.Tensor, txt_shift: torch.Tensor, txt_scale: torch.Tensor, img_shift: torch.Tensor,
                     img_scale: torch.Tensor, seq: int, txt_rows: int, out: torch.Tensor | None = None,
                     scales: torch.Tensor | None = None, fp8: bool = False, eps: float = 1e-6,
                     stream: torch.cuda.Stream | None = None):
    """Both streams of a double block in one launch (b2g_modulate_streams): x [M, C] F32 holds
    whole sequences of `seq` rows, the first `txt_rows` of each modulated with the txt vectors,
    the rest with the img vectors.  Returns bf16 [M, C], or (codes, row scales) with fp8."""
    lib = load()
    M, C = _modulate_args(x, txt_shift, txt_scale)
    _modulate_args(x, img_shift, img_scale)
    if fp8:
        codes, rs = _q8_outputs(M, C, x.device, out, scales, "modulate_streams")
        dst, dt, rsp = codes, E4M3, rs.data_ptr()
    else:
        codes = out if out is not None else torch.empty((M, C), dtype=torch.bfloat16, device=x.device)
        _require_cuda(codes)
        if codes.dtype != torch.bfloat16 or codes.shape != (M, C):
            raise B2GError("modulate_streams: out must be bf16 [M, C]")
        dst, dt, rsp, rs = codes, BF16, None, None
    if not dst.is_contiguous():
        raise B2GError("modulate_streams: out must be contiguous")
    s = (stream or torch.cuda.current_stream(x.device)).cuda_stream
    _check(lib.b2g_modulate_streams(x.data_ptr(), txt_shift.data_ptr(), txt_scale.data_ptr(), img_shift.data_ptr(),
                                    img_scale.data_ptr(), seq, txt_rows, dst.data_ptr(), dt, rsp, M, C, eps,
                                    ctypes.c_void_p(s)))
    return (codes, rs) if fp8 else codes


def compact_rope_table(pe: torch.Tensor) -> torch.Tensor | None:
    """[L, 64, 2] (cos, sin) form of a RoPE table [L, 64, 4] = (cos, -sin, sin, cos) per pair,
    for gemm_qkv_rope; None if the table is not of that form (then pass it as it is)."""
    p = pe.reshape(pe.shape[0], -1, 4)
    if not (torch.equal(p[..., 0], p[..., 3]) and torch.equal(p[..., 1], -p[..., 2])):
        return None
    return torch.stack([p[..., 0], p[..., 2]], -1).contiguous()


# ---------------------------------------------------------------------------- rest of the step
def _stream(t: torch.Tensor, stream: torch.cuda.Stream | None) -> ctypes.c_void_p:
    return ctypes.c_void_p((stream or torch.cuda.current_stream(t.device)).cuda_stream)


def patchify_bf16(x: torch.Tensor, p: int, out: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """im2col of conv2d_img_in + linear()'s cast (chroma.cuh:1311-1327): x F32 [C, H, W] (or
    [1, C, H, W]) -> out bf16 [(H/p)(W/p), >= C*p*p]."""
    _require_cuda(x, out)
    C, H, W = x.shape[-3:]
    if x.dtype != torch.float32 or not x.is_contiguous() or out.dtype != torch.bfloat16 or out.stride(1) != 1:
        raise B2GError("patchify_bf16: contiguous F32 image and a bf16 output with unit column stride")
    _check(load().b2g_patchify_bf16(x.data_ptr(), C, H, W, p, out.data_ptr(), out.stride(0), _stream(x, stream)))
    return out


def timestep_vec(timestep: torch.Tensor, guidance: float, out: torch.Tensor,
                 stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """compute_modulation's approximator input (chroma.cuh:467-505) into out F32 [rows, 64];
    timestep: a one-element F32 device tensor."""
    _require_cuda(timestep, out)
    if out.dtype != torch.float32 or not out.is_contiguous() or out.shape[-1] != 64:
        raise B2GError("timestep_vec: contiguous F32 [rows, 64] output")
    _check(load().b2g_timestep_vec(timestep.data_ptr(), float(guidance), out.data_ptr(), out.shape[0],
                                   _stream(out, stream)))
    return out


def rms_norm(x: torch.Tensor, scale: torch.Tensor, out: torch.Tensor, eps: float = 1e-6,
             stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """rms_norm_cuda (kernels.cu:174-212) over the last dim of x [rows, C] (F32, row stride any)
    into out (F32 or bf16)."""
    _require_cuda(x, scale, out)
    rows, C = x.shape
    if x.dtype != torch.float32 or x.stride(1) != 1 or out.stride(1) != 1 or out.shape != x.shape:
        raise B2GError("rms_norm: F32 x and an output of the same shape, unit column strides")
    _check(load().b2g_rms_norm(x.data_ptr(), x.stride(0), scale.data_ptr(), out.data_ptr(), _operand_dtype(out),
                               out.stride(0), rows, C, eps, _stream(x, stream)))
    return out


def nerf_input_bf16(x: torch.Tensor, dct: torch.Tensor, out: torch.Tensor,
                    stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """The NeRF embedder's input rows [pixel rgb | DCT features | zeros] (chroma.cuh:1170-1200)."""
    _require_cuda(x, dct, out)
    H, W = x.shape[-2:]
    _check(load().b2g_nerf_input_bf16(x.data_ptr(), dct.data_ptr(), H, W, out.data_ptr(), out.stride(0),
                                      _stream(x, stream)))
    return out


def nerf_glu_weights(params: torch.Tensor, gate: torch.Tensor, value: torch.Tensor, fc2: torch.Tensor,
                     stream: torch.cuda.Stream | None = None) -> None:
    """slice_transpose + l2_norm of one NeRF GLU block's generated weights (chroma.cuh:1264-1281):
    params F32 [P, 49152] -> gate, value [P, 256, 64], fc2 [P, 64, 256]."""
    _require_cuda(params, gate, value, fc2)
    _check(load().b2g_nerf_glu_weights(params.data_ptr(), params.stride(0), params.shape[0], gate.data_ptr(),
                                       value.data_ptr(), fc2.data_ptr(), _stream(params, stream)))


def convert_f32(src: torch.Tensor, out: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """out (bf16 or fp16) = src (F32 [rows, cols]) rounded to nearest, as linear() casts
    activations (f32_to_bf16_cuda); unit column strides, any row strides."""
    _require_cuda(src, out)
    if src.dtype != torch.float32 or src.shape != out.shape or src.stride(1) != 1 or out.stride(1) != 1:
        raise B2GError("convert_f32: F32 source and an output of the same 2-D shape")
    _check(load().b2g_convert_f32(src.data_ptr(), src.stride(0), src.shape[0], src.shape[1], out.data_ptr(),
                                  _operand_dtype(out), out.stride(0), _stream(src, stream)))
    return out


def nerf_glu_block(params: torch.Tensor, norm_scale: torch.Tensor, x: torch.Tensor,
                   stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """One NeRF GLU block fused (chroma.cuh:1253-1306): params F32 [P, >= 49152] (the
    param_generator output), x F32 [P, 256, 64] updated in place."""
    _require_cuda(params, norm_scale, x)
    P = params.shape[0]
    if params.dtype != torch.float32 or params.stride(1) != 1 or x.dtype != torch.float32 or not x.is_contiguous() \
            or x.numel() != P * 256 * 64:
        raise B2GError("nerf_glu_block: F32 params [P, >= 49152] and a contiguous F32 state [P, 256, 64]")
    _check(load().b2g_nerf_glu_block(params.data_ptr(), params.stride(0), norm_scale.data_ptr(), x.data_ptr(), P,
                                     _stream(x, stream)))
    return x


def silu_mul(a: torch.Tensor, b: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
    """a = silu(a) * b (silu_mul_cuda), F32, contiguous."""
    _require_cuda(a, b)
    _check(load().b2g_silu_mul(a.data_ptr(), b.data_ptr(), a.numel(), _stream(a, stream)))


def add_inplace(x: torch.Tensor, y: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
    """x += y (add_cuda), F32, contiguous."""
    _require_cuda(x, y)
    _check(load().b2g_add_inplace(x.data_ptr(), y.data_ptr(), x.numel(), _stream(x, stream)))


def nerf_final(feat_cond: torch.Tensor, feat_uncond: torch.Tensor | None, norm_scale: torch.Tensor,
               conv_w: torch.Tensor, conv_b: torch.Tensor, cfg_scale: float, H: int, W: int,
               out: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """NeRF final layer of both guidance halves + cfg_blend (chroma.cuh:1225-1250, 1581) into out
    F32 [3, H, W], one kernel."""
    _require_cuda(feat_cond, norm_scale, conv_w, conv_b, out)
    _check(load().b2g_nerf_final(feat_cond.data_ptr(), _ptr(feat_uncond), norm_scale.data_ptr(), conv_w.data_ptr(),
                                 conv_b.data_ptr(), float(cfg_scale), H, W, out.data_ptr(), _stream(out, stream)))
    return out
