"""CPU self-checks of the oracle's number formats and GEMM against numpy/torch (no GPU)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err


def test_bf16_rounding_matches_torch(oracle):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10,
                        np.array([0.0, -0.0, 1e-40, -1e-40, 3.4e38, -3.4e38, np.inf, -np.inf], np.float32)])
    got = oracle.to_bf16_bits(x)
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, want)


def test_f16_rounding_matches_torch(oracle):
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 100,
                        rng.standard_normal(20000).astype(np.float32) * 1e-5,   # subnormal halves
                        np.array([0.0, -0.0, 65504.0, 65520.0, 70000.0, -1e9, 2.0 ** -25, 2.0 ** -24,
                                  1.5 * 2.0 ** -24, np.inf], np.float32)])
    got = oracle.to_f16_bits(x)
    want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
    back = oracle.to_f32(got, 1)
    assert np.array_equal(back, want.view(np.float16).astype(np.float32))


@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (5, 17, 3), (64, 256, 96), (33, 3000, 7)])
def test_linear_matches_float64(oracle, M, K, N):
    rng = np.random.default_rng(M * 1000 + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((N, K)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    got = oracle.linear(x, 0, w, 0, b)
    want = x.astype(np.float64) @ w.astype(np.float64).T + b
    assert rel_err(got, want) < 1e-5


def test_linear_bf16_inputs_are_exact(oracle):
    rng = np.random.default_rng(3)
    x = oracle.to_bf16_bits(rng.standard_normal((20, 100)).astype(np.float32))
    w = oracle.to_bf16_bits(rng.standard_normal((30, 100)).astype(np.float32))
    got = oracle.linear(x, 2, w, 2)
    want = oracle.to_f32(x, 2).astype(np.float64) @ oracle.to_f32(w, 2).astype(np.float64).T
    assert rel_err(got, want) < 1e-5


def test_gelu_formula(oracle):
    x = np.linspace(-10, 10, 2001, dtype=np.float32)
    xd = x.astype(np.float64)
    want = 0.5 * xd * (1 + np.tanh(0.7978845608 * (xd + 0.044715 * xd ** 3)))
    assert np.abs(oracle.gelu(x) - want).max() < 1e-5


def test_modulate_and_rms_norm(oracle):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 64)).astype(np.float32)
    sh = rng.standard_normal(64).astype(np.float32)
    sc = rng.standard_normal(64).astype(np.float32)
    xd = x.astype(np.float64)
    ln = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + 1e-6)
    assert rel_err(oracle.modulate(x, sh, sc), ln * (1 + sc) + sh) < 1e-5
    rms = xd / np.sqrt((xd ** 2).mean(1, keepdims=True) + 1e-6) * sc
    assert rel_err(oracle.rms_norm(x, sc), rms) < 1e-5


def test_attention_matches_float64_within_bf16(oracle):
    rng = np.random.default_rng(5)
    L, H, D = 24, 2, 16
    Q, K, V = (rng.standard_normal((L, H, D)).astype(np.float32) for _ in range(3))
    ang = rng.uniform(0, 2 * np.pi, (L, D // 2))
    pe = np.stack([np.cos(ang), -np.sin(ang), np.sin(ang), np.cos(ang)], -1).astype(np.float32)
    mask = np.zeros(L, np.float32)
    mask[5:9] = -np.inf
    got = oracle.attention_rope(Q, K, V, pe, mask)

    def rope(x):
        e, o = x[..., 0::2].astype(np.float64), x[..., 1::2].astype(np.float64)
        c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
        r = np.empty(x.shape)
        r[..., 0::2], r[..., 1::2] = e * c - o * s, e * s + o * c
        return r

    q, k = rope(Q), rope(K)
    want = np.empty((L, H * D))
    for h in range(H):
        s_ = q[:, h] @ k[:, h].T / np.sqrt(D) + mask[None, :]
        p = np.exp(s_ - s_.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        want[:, h * D:(h + 1) * D] = p @ V[:, h].astype(np.float64)
    assert rel_err(got, want) < 2e-2
    assert np.all(got[:, :] == got[:, :])  # no NaN from the -inf keys


def test_e4m3_decode_all_codes_matches_torch(oracle):
    codes = np.arange(256, dtype=np.uint8)
    mine = oracle.e4m3_to_f32(codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(mine), np.isnan(theirs))
    fin = ~np.isnan(mine)
    assert np.array_equal(mine[fin], theirs[fin])
    assert mine[fin].max() == 448.0 and np.isnan(mine[0x7F]) and np.isnan(mine[0xFF])


def test_e4m3_encode_matches_torch_in_range_and_saturates(oracle):
    rng = np.random.default_rng(11)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 50,
                        rng.standard_normal(20000).astype(np.float32) * 1e-2,   # subnormal range
                        rng.uniform(-448, 448, 50000).astype(np.float32),
                        oracle.e4m3_to_f32(np.arange(0, 126, dtype=np.uint8)),  # exact codes and midpoints
                        (oracle.e4m3_to_f32(np.arange(0, 125, dtype=np.uint8)) +
                         oracle.e4m3_to_f32(np.arange(1, 126, dtype=np.uint8))) / 2])
    mine = oracle.to_e4m3_bits(x)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mine, theirs)
    big = np.array([449.0, 464.0, 1e30, np.inf, -600.0], np.float32)   # satfinite: clamp to +-448
    assert np.array_equal(oracle.e4m3_to_f32(oracle.to_e4m3_bits(big)), [448, 448, 448, 448, -448])


def test_quantize_rows_e4m3_restates_absmax_scaling(oracle):
    rng = np.random.default_rng(12)
    x = rng.standard_normal((7, 40)).astype(np.float32) * np.float32(3.0)
    x[3] = 0.0
    q, s = oracle.quantize_rows_e4m3(x)
    amax = np.abs(x).max(1)
    assert np.array_equal(s, np.where(amax > 0, amax / np.float32(448), np.float32(1)).astype(np.float32))
    inv = np.where(amax > 0, np.float32(448) / amax, np.float32(1)).astype(np.float32)
    want = torch.from_numpy((x * inv[:, None]).astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(q, want)
    assert np.abs(oracle.e4m3_to_f32(q).max(1)[amax > 0]).max() == 448.0


def test_e4m3_quantisation_error_is_inherent(oracle):
    """Per-row absmax/448 E4M3 quantisation of N(0,1) activations and N(0,0.02) weights, GEMM in
    exact arithmetic on the quantised values: the error against the unquantised product is the
    format's own (about 2.65% RMS per element, 3.7% RMS on a K=3072 product)."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((128, 3072)).astype(np.float32)
    w = (rng.standard_normal((256, 3072)) * 0.02).astype(np.float32)
    qx, sx = oracle.quantize_rows_e4m3(x)
    qw, sw = oracle.quantize_rows_e4m3(w)
    per_elem = np.sqrt(np.mean((oracle.e4m3_to_f32(qx) * sx[:, None] - x) ** 2) / np.mean(x ** 2))
    y8 = oracle.gemm_fp8(qx, sx, qw, sw)
    y = x.astype(np.float64) @ w.astype(np.float64).T
    rms = np.sqrt(np.mean((y8 - y) ** 2) / np.mean(y ** 2))
    assert 0.024 < per_elem < 0.029
    assert 0.033 < rms < 0.041


def test_rope_is_the_attention_rotation(oracle):
    """oracle.rope rotates each (even, odd) pair by its pe row: pair norms are kept, the
    inverse table (cos, sin, -sin, cos) undoes it, and it agrees with the pair formula of
    apply_rope_fused_bf16 in numpy (to an fp32 ulp: the C code may contract into FMAs)."""
    rng = np.random.default_rng(5)
    L, H, D = 9, 3, 16
    x = rng.standard_normal((L, H * D)).astype(np.float32)
    ang = rng.uniform(0, 2 * np.pi, (L, D // 2))
    pe = np.stack([np.cos(ang), -np.sin(ang), np.sin(ang), np.cos(ang)], -1).astype(np.float32)
    inv = np.stack([np.cos(ang), np.sin(ang), -np.sin(ang), np.cos(ang)], -1).astype(np.float32)
    y = oracle.rope(x, pe, H)
    pairs = lambda a: np.hypot(a[:, 0::2], a[:, 1::2])
    assert np.allclose(pairs(y), pairs(x), rtol=1e-6, atol=1e-6)
    assert np.allclose(oracle.rope(y, inv, H), x, rtol=1e-5, atol=1e-5)
    e, o = x.reshape(L, H, D // 2, 2)[..., 0], x.reshape(L, H, D // 2, 2)[..., 1]
    p = pe[:, None]
    want = np.stack([e * p[..., 0] + o * p[..., 1], e * p[..., 2] + o * p[..., 3]], -1).reshape(L, H * D)
    assert np.allclose(y, want, rtol=1e-6, atol=1e-6)

