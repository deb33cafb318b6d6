"""Pins the C oracle (oracle/oracle.c) to the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by running the reference's cublas_ops.cuh / kernels.cu (compiled
from its sources) on a B200 — see tests/golden/make_golden.py.  Runs on CPU only.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, rel_err

FIXTURES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load(name):
    path = GOLDEN / f"{name}.npz"
    if not path.exists():
        pytest.skip(f"golden fixture {name} not generated yet")
    return dict(np.load(path))


def test_fixtures_present():
    expected = {"linear_lt_bf16_bias", "linear_lt_bf16_nobias", "linear_lt_fp16", "linear_lt_f32_k67",
                "linear_f32x_bf16w", "linear_f32x_fp16w", "linear_gated_residual_bf16", "gelu",
                "gated_residual", "batched_matmul_Bt", "modulate_to_bf16", "rms_norm", "attention_rope"}
    missing = expected - set(FIXTURES)
    assert not missing, f"missing golden fixtures: {sorted(missing)}"


@pytest.mark.parametrize("name", ["linear_lt_bf16_bias", "linear_lt_bf16_nobias", "linear_lt_fp16",
                                  "linear_lt_f32_k67"])
def test_linear_lt(oracle, name):
    g = load(name)
    dt = int(g["dtype"])
    got = oracle.linear(g["x"], dt, g["w"], dt, g.get("bias"))
    # Both sides accumulate exactly-represented products in fp32; only the order differs.
    assert rel_err(got, g["out"]) < 1e-5


@pytest.mark.parametrize("name", ["linear_f32x_bf16w", "linear_f32x_fp16w"])
def test_linear_casts_f32_activations(oracle, name):
    g = load(name)
    wdt = int(g["wdtype"])
    x16 = oracle.round(g["x"], wdt)  # linear() casts x to the weight dtype first
    got = oracle.linear(x16, 0, g["w"], wdt, g["bias"])
    assert rel_err(got, g["out"]) < 1e-5
    # Without the cast the result is measurably different: the fixture really pins it.
    uncast = oracle.linear(g["x"], 0, oracle.to_f32(g["w"], wdt), 0, g["bias"])
    assert rel_err(uncast, g["out"]) > rel_err(got, g["out"])


def test_linear_gated_residual(oracle):
    g = load("linear_gated_residual_bf16")
    y = oracle.linear(g["x"], 2, g["w"], 2, g["bias"])
    got = oracle.gated_residual(g["resid"], y, g["gate"])
    assert rel_err(got, g["out"]) < 1e-5


def test_gelu(oracle):
    g = load("gelu")
    got = oracle.gelu(g["x"])
    # The reference is built with --use_fast_math (approximate tanhf); the oracle uses libm.
    assert np.abs(got - g["out"]).max() < 2e-6 * (1 + np.abs(g["x"]).max())
    got16 = oracle.to_f32(oracle.gelu_to_bf16(g["x"]), 2).astype(np.float64)
    want16 = oracle.to_f32(g["out_bf16"], 2).astype(np.float64)
    # One bf16 ulp where the two tanh evaluations straddle a rounding boundary; on the far
    # negative tail (|gelu| < 1e-4) the approximate tanhf rounds 1 + tanh to exactly 0.
    assert np.all(np.abs(got16 - want16) <= np.maximum(2.0 ** -7 * np.abs(want16), 1e-4))
    assert (got16 == want16).mean() > 0.9


def test_gated_residual(oracle):
    g = load("gated_residual")
    got = oracle.gated_residual(g["x"], g["y"], g["gate"])
    assert rel_err(got, g["out"]) < 1e-6


def test_batched_matmul_bt(oracle):
    """CUBLAS_COMPUTE_32F_FAST_16BF on B200 is TF32 with round-to-nearest operands."""
    from oracle import BF16, TF32

    g = load("batched_matmul_Bt")
    got = oracle.batched_matmul_bt(g["A"], g["B"], rounding=TF32)
    assert rel_err(got, g["out"]) < 1e-5
    # Neither exact fp32 nor bf16 operands reproduce it: the fixture pins the rounding.
    assert rel_err(oracle.batched_matmul_bt(g["A"], g["B"], rounding=0), g["out"]) > 1e-4
    assert rel_err(oracle.batched_matmul_bt(g["A"], g["B"], rounding=BF16), g["out"]) > 1e-3


def test_modulate_to_bf16(oracle):
    g = load("modulate_to_bf16")
    got = oracle.to_bf16_bits(oracle.modulate(g["x"], g["shift"], g["scale"], 1e-6)).astype(np.int32)
    want = g["out_bf16"].astype(np.int32)
    assert np.abs(got - want).max() <= 1


def test_attention_rope(oracle):
    """The oracle's attention restatement against the reference's cuDNN SDPA path."""
    g = load("attention_rope")
    got = oracle.attention_rope(g["q"], g["k"], g["v"], g["pe"], g["mask"])
    # bf16 operands and probabilities on both sides, different accumulation order and
    # normalisation point: agreement to a few bf16 ulps of the largest output.
    assert rel_err(got, g["out"]) < 1e-2
    a, b = got.ravel().astype(np.float64), g["out"].ravel().astype(np.float64)
    assert a @ b / np.sqrt((a @ a) * (b @ b)) > 0.9999


def test_rms_norm(oracle):
    g = load("rms_norm")
    got = oracle.rms_norm(g["x"], g["scale"], 1e-6)
    assert rel_err(got, g["out"]) < 1e-5
