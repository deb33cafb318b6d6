"""The block GEMMs' A-operand producer, b2g_modulate_to_bf16 (the reference's
modulate_to_bf16, kernels.cu:552-599) and its per-row E4M3 form, against the reference's own
output (golden fixture made by tests/golden/make_golden.py on a B200) and the C oracle.

Tolerances: bf16 codes within 1 unit of the reference's (the row statistics are summed in a
different order, which can move a value across a rounding boundary), as the oracle's own
golden test allows, and values within one bf16 ulp of the oracle's fp32 result; E4M3 codes equal to the oracle's quantisation of its fp32 modulated
values except at rounding ties of that kind (at most 1 code, in at most 0.1% of elements).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16).astype(np.int32)


def assert_within_bf16_ulp(got: torch.Tensor, want_f32: np.ndarray):
    """|got - want| <= one bf16 ulp of want (+1e-6 for values next to zero, whose sign the
    rounding of the row statistics can decide)."""
    g = got.float().cpu().numpy().astype(np.float64)
    w = want_f32.astype(np.float64)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(w), 1e-30))) - 7)
    assert np.all(np.abs(g - w) <= ulp + 1e-6)


def test_modulate_matches_reference_golden(engine):
    g = dict(np.load(GOLDEN / "modulate_to_bf16.npz"))
    x, sh, sc = (torch.from_numpy(g[k]).to(DEV) for k in ("x", "shift", "scale"))
    out = engine.modulate_to_bf16(x, sh, sc, 1e-6)
    torch.cuda.synchronize()
    assert np.abs(bf16_bits(out) - g["out_bf16"].astype(np.int32)).max() <= 1


@pytest.mark.parametrize("M,C", [(1536, 3072), (37, 3072), (5, 200), (9, 4096), (1, 4), (0, 3072)])
def test_modulate_vs_oracle(engine, oracle, M, C):
    rng = np.random.default_rng(M * 7 + C)
    x = (rng.standard_normal((M, C)) * 2.0 + 0.5).astype(np.float32)
    sh = (rng.standard_normal(C) * 0.1).astype(np.float32)
    sc = (rng.standard_normal(C) * 0.1).astype(np.float32)
    out = engine.modulate_to_bf16(torch.from_numpy(x).to(DEV), torch.from_numpy(sh).to(DEV),
                                  torch.from_numpy(sc).to(DEV))
    torch.cuda.synchronize()
    if M == 0:
        assert out.shape == (0, C)
        return
    assert_within_bf16_ulp(out, oracle.modulate(x, sh, sc, 1e-6))


@pytest.mark.parametrize("M,C", [(1536, 3072), (33, 200)])
def test_modulate_e4m3_vs_oracle(engine, oracle, M, C):
    rng = np.random.default_rng(C)
    x = rng.standard_normal((M, C)).astype(np.float32)
    x[min(3, M - 1)] = 0.25  # a constant row: LayerNorm gives 0, modulated values are the shift
    sh = (rng.standard_normal(C) * 0.1).astype(np.float32)
    sc = (rng.standard_normal(C) * 0.1).astype(np.float32)
    codes, rs = engine.modulate_to_e4m3(torch.from_numpy(x).to(DEV), torch.from_numpy(sh).to(DEV),
                                        torch.from_numpy(sc).to(DEV))
    torch.cuda.synchronize()
    y = oracle.modulate(x, sh, sc, 1e-6)
    q, s = oracle.quantize_rows_e4m3(y)
    np.testing.assert_allclose(rs.cpu().numpy(), s, rtol=1e-6)
    got = codes.cpu().numpy()
    # E4M3 magnitude codes are monotonic in |value|: compare the 7-bit magnitudes and signs.
    diff = np.abs(got.astype(np.int32) & 0x7F) - (q.astype(np.int32) & 0x7F)
    assert np.abs(diff).max() <= 1
    assert (diff != 0).mean() <= 1e-3


def test_modulate_rejects_unsupported(engine):
    x = torch.zeros((4, 6), device=DEV)
    v = torch.zeros(6, device=DEV)
    with pytest.raises(engine.B2GError):
        engine.modulate_to_bf16(x, v, v)  # C % 4 != 0


@pytest.mark.parametrize("fp8", [False, True])
def test_modulate_streams_equals_per_stream_calls(engine, fp8):
    """b2g_modulate_streams over two half-major sequences of [txt | img] rows gives, row for
    row, the same bits as modulate_to_bf16 / modulate_to_e4m3 on each stream's rows with that
    stream's vectors."""
    T, I, C = 40, 88, 3072
    L = T + I
    g = torch.Generator(device=DEV).manual_seed(21)
    x = torch.randn((2 * L, C), generator=g, device=DEV) * 3 + 0.5
    vec = [torch.randn(C, generator=g, device=DEV) * 0.3 for _ in range(4)]
    got = engine.modulate_streams(x, vec[0], vec[1], vec[2], vec[3], L, T, fp8=fp8)
    torch.cuda.synchronize()
    one = engine.modulate_to_e4m3 if fp8 else engine.modulate_to_bf16
    for b in range(2):
        for r0, r1, sh, sc in ((b * L, b * L + T, vec[0], vec[1]), (b * L + T, (b + 1) * L, vec[2], vec[3])):
            want = one(x[r0:r1].contiguous(), sh, sc)
            if fp8:
                assert torch.equal(got[0][r0:r1], want[0]) and torch.equal(got[1][r0:r1], want[1])
            else:
                assert torch.equal(got[r0:r1], want)


def test_modulate_streams_rejects_partial_sequences(engine):
    x = torch.zeros((100, 64), device=DEV)
    v = torch.zeros(64, device=DEV)
    with pytest.raises(engine.B2GError):
        engine.modulate_streams(x, v, v, v, v, 64, 10)      # 100 rows are not whole sequences of 64
