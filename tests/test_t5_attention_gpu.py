"""T5 attention (attention.cuh:34-91) on the engine: fp32-level scores from TF32 hi/lo operand
splits on the tensor cores, TF32 P.V.  Checked against a float64 numpy restatement (small
sizes) and the reference's own fp32 cuBLAS path at BASELINE config 5's size (512 tokens, 64
heads x 64).  Tolerance: max|d|/max|ref| <= 2e-3 (the north star's per-GEMM bound; measured
errors are far below it)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def t5_inputs(L, H, D, seed, bias=True, masked=0):
    g = torch.Generator().manual_seed(seed)
    Q, K, V = (torch.randn((L, H, D), generator=g) for _ in range(3))
    rb = torch.randn((H, L, L), generator=g) * 3.0 if bias else None
    mask = None
    if masked:
        mask = torch.zeros(L)
        mask[L - masked:] = float("-inf")
    return Q, K, V, rb, mask


def fp64_t5(Q, K, V, rb, mask, scale):
    q, k, v = (t.double().numpy() for t in (Q, K, V))
    L, H, D = q.shape
    out = np.empty((L, H * D))
    for h in range(H):
        s = scale * q[:, h] @ k[:, h].T
        if rb is not None:
            s = s + rb[h].double().numpy()
        if mask is not None:
            s = s + mask.double().numpy()[None, :]
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        out[:, h * D:(h + 1) * D] = p @ v[:, h]
    return out


@pytest.mark.parametrize("L,H,D,bias,masked,scale", [(64, 4, 64, True, 0, 1.0), (200, 3, 64, True, 17, 1.0),
                                                      (128, 2, 128, False, 5, 0.125)])
def test_t5_attention_vs_fp64(engine, L, H, D, bias, masked, scale):
    Q, K, V, rb, mask = t5_inputs(L, H, D, L + H, bias, masked)
    out = engine.t5_attention(Q.to(DEV), K.to(DEV), V.to(DEV), rb.to(DEV) if rb is not None else None, H, D, scale,
                              mask.to(DEV) if mask is not None else None)
    torch.cuda.synchronize()
    want = fp64_t5(Q, K, V, rb, mask, scale)
    assert rel_err(out.cpu().numpy(), want) <= 2e-3


def test_t5_attention_vs_reference_fp32(engine):
    from oracle import ATTN_REF_PATH, AttnRef

    if not ATTN_REF_PATH.exists():
        pytest.skip("reference attention library not built")
    ref = AttnRef()
    L, H, D = 512, 64, 64
    Q, K, V, rb, mask = t5_inputs(L, H, D, 3, True, 40)
    dq, dk, dv, drb, dm = (t.to(DEV) for t in (Q, K, V, rb, mask))
    mine = engine.t5_attention(dq, dk, dv, drb, H, D, 1.0, dm)
    theirs = torch.empty((L, H * D), device=DEV)
    assert ref.lib.ref_t5_attention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), drb.data_ptr(), H, D, L, 1.0,
                                    dm.data_ptr(), theirs.data_ptr()) == 0
    torch.cuda.synchronize()
    err = rel_err(mine.cpu().numpy(), theirs.cpu().numpy())
    print("t5 attention vs reference fp32:", err)
    assert err <= 2e-3
