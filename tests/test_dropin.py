"""The drop-in headers (cublas_ops.cuh, cudnn_attention.cuh, attention.cuh): the reference's
chroma.cuh / t5.cuh compile unchanged against libb2g.so (CPU), and every routed entry point
matches the original cuBLASLt / cuDNN / cuBLAS code inside the same binary (GPU)."""
from __future__ import annotations

import json
import re
import subprocess

import pytest

from conftest import PKG

BIN = PKG / "dropin" / "build" / "ab_check"
DROPIN = PKG / "dropin" / "cublas_ops.cuh"
DROPIN_ATTN = PKG / "dropin" / "cudnn_attention.cuh"
DROPIN_T5 = PKG / "dropin" / "attention.cuh"


def test_dropin_keeps_every_routed_signature():
    text = DROPIN.read_text()
    for sig in [
        r"static void linear\(const Tensor& x, const Tensor& W, const Tensor\* bias, Tensor& output\)",
        r"static void linear_lt\(int64_t M, int64_t K, int64_t N, const void\* x_data, cudaDataType_t x_type,\s+"
        r"const void\* w_data, cudaDataType_t w_type, const void\* bias_data, void\* out_data\)",
        r"static void linear_gated_residual\(const Tensor& x, const Tensor& W, const Tensor\* bias, "
        r"float\* residual_inout,\s+const float\* gate, int64_t M, int64_t N_out\)",
        r"static void batched_matmul_Bt\(const Tensor& A, const Tensor& B, Tensor& C\)",
        r"static void init_cublas\(\)",
    ]:
        assert re.search(sig, text), sig


def test_attention_dropins_keep_the_routed_signatures():
    assert re.search(r"static Tensor cudnn_attention_with_rope\(const Tensor& Q, const Tensor& K, const Tensor& V, "
                     r"const Tensor& pe,\s+int n_head, int d_head, const float\* attn_mask = nullptr\)",
                     DROPIN_ATTN.read_text())
    assert re.search(r"static Tensor t5_attention\(const Tensor& Q, const Tensor& K, const Tensor& V, "
                     r"const float\* rel_bias, int n_head,\s+int d_head, float scale, "
                     r"const float\* attn_mask = nullptr\)", DROPIN_T5.read_text())


def test_reference_model_links_against_engine():
    if not BIN.exists():
        pytest.skip("drop-in build needs the reference sources at build time")
    syms = subprocess.run(["nm", "-D", str(BIN)], capture_output=True, text=True, check=True).stdout
    for name in ("b2g_gemm", "b2g_init", "b2g_linear_gated_residual", "b2g_batched_matmul_Bt",
                 "b2g_attention_with_rope", "b2g_t5_attention"):
        assert re.search(rf"\bU {name}\b", syms), name


@pytest.mark.gpu
def test_reference_model_ab_check_on_gpu():
    if not BIN.exists():
        pytest.skip("drop-in build needs the reference sources at build time")
    r = subprocess.run([str(BIN)], capture_output=True, text=True, timeout=300)
    lines = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    entries = {d["entry"]: d for d in lines if "entry" in d}
    assert set(entries) == {"linear bf16", "linear f32x fp16w", "linear_gated_residual", "batched_matmul_Bt",
                            "cudnn_attention_with_rope", "t5_attention"}
    for d in entries.values():
        assert d["rel_diff"] <= d["tol"], d
    assert r.returncode == 0, r.stdout + r.stderr
