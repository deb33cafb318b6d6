"""The kernels of the denoising step around the blocks (csrc/model.cu, csrc/model_fastmath.cu and
the GEMM's SiLU epilogue), each against a plain torch statement of the reference's kernel on
the same inputs (fp64 where the reference's fp32 rounding order is not the point):
patchify (kernels.cu:975-1019), the NeRF input rows (chroma.cuh:1170-1200), rms_norm
(kernels.cu:174-212), the GLU weight preparation (slice_transpose + l2_norm, chroma.cuh:
1264-1281), silu_mul / add, the final norm + 3x3 conv + cfg_blend (chroma.cuh:1225-1250, 1581)
and the approximator input (kernels.cu:608-631)."""
from __future__ import annotations

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def gen(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


def test_patchify_bf16(engine):
    x = torch.randn((1, 3, 64, 96), generator=gen(1), device=DEV)
    out = torch.full((24, 776), 7.0, dtype=torch.bfloat16, device=DEV)   # ldo > 768: padding untouched
    engine.patchify_bf16(x, 16, out)
    want = x[0].reshape(3, 4, 16, 6, 16).permute(1, 3, 0, 2, 4).reshape(24, 768).to(torch.bfloat16)
    assert torch.equal(out[:, :768], want)
    assert torch.all(out[:, 768:] == 7.0)


def test_nerf_input_rows(engine):
    H, W = 32, 48
    x = torch.randn((1, 3, H, W), generator=gen(2), device=DEV)
    dct = torch.randn((256, 64), generator=gen(3), device=DEV)
    out = torch.full((6 * 256, 72), 5.0, dtype=torch.bfloat16, device=DEV)
    engine.nerf_input_bf16(x, dct, out)
    pix = x[0].reshape(3, 2, 16, 3, 16).permute(1, 3, 2, 4, 0).reshape(6 * 256, 3)     # [patch, py, px, c]
    want = torch.cat([pix, dct.repeat(6, 1), torch.zeros((6 * 256, 5), device=DEV)], 1).to(torch.bfloat16)
    assert torch.equal(out, want)


@pytest.mark.parametrize("rows,C,odt", [(300, 64, torch.float32), (129, 192, torch.bfloat16),
                                         (344, 5120, torch.bfloat16), (17, 12288, torch.float32)])
def test_rms_norm(engine, rows, C, odt):
    x = torch.randn((rows, C), generator=gen(C), device=DEV) * 3
    scale = torch.randn(C, generator=gen(C + 1), device=DEV) * 0.1 + 1
    out = torch.empty((rows, C), dtype=odt, device=DEV)
    engine.rms_norm(x, scale, out, eps=1e-6)
    xd = x.double()
    want = xd * torch.rsqrt((xd * xd).mean(1, keepdim=True) + 1e-6) * scale.double()
    tol = 2.0 ** -8 if odt == torch.bfloat16 else 1e-5
    assert rel_err(out.float().cpu().numpy(), want.cpu().numpy()) <= tol


def test_nerf_glu_weights(engine):
    P = 5
    params = torch.randn((P, 49152), generator=gen(4), device=DEV)
    gate, value = (torch.empty((P, 256, 64), device=DEV) for _ in range(2))
    fc2 = torch.empty((P, 64, 256), device=DEV)
    engine.nerf_glu_weights(params, gate, value, fc2)
    pd = params.double()

    def l2(t):
        return t / t.norm(dim=-1, keepdim=True).clamp_min(1e-12)

    want_g = l2(pd[:, :16384].view(P, 64, 256).transpose(1, 2))
    want_v = l2(pd[:, 16384:32768].view(P, 64, 256).transpose(1, 2))
    want_f = l2(pd[:, 32768:].view(P, 256, 64).transpose(1, 2))
    for got, want in ((gate, want_g), (value, want_v), (fc2, want_f)):
        assert (got.double() - want).abs().max().item() <= 1e-6


def test_silu_mul_and_add(engine):
    a = torch.randn(4096, generator=gen(5), device=DEV) * 4
    b = torch.randn(4096, generator=gen(6), device=DEV)
    want = (a.double() / (1 + torch.exp(-a.double()))) * b.double()
    engine.silu_mul(a, b)
    assert (a.double() - want).abs().max().item() <= 1e-5 * want.abs().max().item()
    c = torch.randn(4096, generator=gen(7), device=DEV)
    want2 = a + c
    engine.add_inplace(a, c)
    assert torch.equal(a, want2)


@pytest.mark.parametrize("halves", [1, 2])
def test_nerf_final(engine, halves):
    H, W, cfg = 48, 32, 3.5
    P = (H // 16) * (W // 16)
    feats = [torch.randn((P * 256, 64), generator=gen(10 + z), device=DEV) for z in range(halves)]
    scale = torch.randn(64, generator=gen(20), device=DEV) * 0.1 + 1
    cw = torch.randn((3, 64, 3, 3), generator=gen(21), device=DEV) * 0.05
    cb = torch.randn(3, generator=gen(22), device=DEV) * 0.05
    out = torch.empty((3, H, W), device=DEV)
    engine.nerf_final(feats[0], feats[1] if halves == 2 else None, scale, cw, cb, cfg, H, W, out)

    def ref(f):   # unpatchify to [64, H, W], RMS norm over channels, 3x3 conv with zero padding
        img = f.double().view(H // 16, W // 16, 16, 16, 64).permute(4, 0, 2, 1, 3).reshape(64, H, W)
        img = img * torch.rsqrt((img * img).mean(0, keepdim=True) + 1e-6) * scale.double()[:, None, None]
        return torch.nn.functional.conv2d(img[None], cw.double(), cb.double(), padding=1)[0]

    want = ref(feats[0]) if halves == 1 else ref(feats[1]) + cfg * (ref(feats[0]) - ref(feats[1]))
    assert rel_err(out.cpu().numpy(), want.cpu().numpy()) <= 1e-5


def test_timestep_vec_structure(engine):
    """Rows = [timestep embedding (16) | guidance embedding (16) | row-index embedding (32)]:
    cos then sin halves; the guidance is 0 and row 0's index is 0, so those parts are exactly
    [1]*8 + [0]*8 and [1]*16 + [0]*16, and the timestep part is the same in every row."""
    t = torch.tensor([0.25], device=DEV)
    out = torch.empty((344, 64), device=DEV)
    engine.timestep_vec(t, 0.0, out)
    assert torch.equal(out[:, 16:32], torch.tensor([1.0] * 8 + [0.0] * 8, device=DEV).expand(344, 16))
    assert torch.equal(out[0, 32:], torch.tensor([1.0] * 16 + [0.0] * 16, device=DEV))
    assert torch.equal(out[:, :16], out[:1, :16].expand(344, 16))
    f = torch.exp(-torch.log(torch.tensor(10000.0, dtype=torch.float64)) * torch.arange(8) / 8)
    want = torch.cat([torch.cos(250.0 * f), torch.sin(250.0 * f)]).to(DEV)
    assert (out[0, :16].double() - want).abs().max().item() <= 1e-3   # fast-math cos/sin at |x| <= 250


def test_gemm_silu_epilogue(engine):
    g = torch.Generator().manual_seed(31)
    x = torch.randn((344, 640), generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn((1280, 640), generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    b = (torch.randn(1280, generator=g) * 0.05).to(DEV)
    y = x.double() @ w.double().t() + b.double()
    want = y / (1 + torch.exp(-y))
    got = engine.gemm(x, w, b, out_dtype=torch.bfloat16, epilogue="silu")
    got32 = engine.gemm(x, w, b, out_dtype=torch.float32, epilogue="silu")
    torch.cuda.synchronize()
    assert rel_err(got32.cpu().numpy(), want.cpu().numpy()) <= 1e-5
    assert rel_err(got.float().cpu().numpy(), want.cpu().numpy()) <= 2.0 ** -8


def _tf32(t: torch.Tensor) -> torch.Tensor:
    """Round fp32 values to TF32 (10 mantissa bits), nearest even (finite inputs)."""
    i = t.float().contiguous().view(torch.int32)
    return ((i + (((i >> 13) & 1) + 0x0FFF)) & ~0x1FFF).view(torch.float32)


def test_nerf_glu_block_fused(engine):
    """The fused GLU block against fp64 with the operands rounded to TF32 where the reference's
    cuBLAS rounds them (normalised weights, normed state, silu * mul), and against the engine's
    own unfused sequence (weights, rms_norm, three batched products, silu_mul, add)."""
    P = 301                                     # more patches than SMs: the persistent loop wraps
    params = torch.randn((P, 49152), generator=gen(40), device=DEV) * 0.05
    x = torch.randn((P, 256, 64), generator=gen(41), device=DEV)
    scale = torch.randn(64, generator=gen(42), device=DEV) * 0.1 + 1
    x0 = x.clone()
    engine.nerf_glu_block(params, scale, x)
    # unfused engine sequence
    gate, value = (torch.empty((P, 256, 64), device=DEV) for _ in range(2))
    fc2 = torch.empty((P, 64, 256), device=DEV)
    xn, x1, x2, xo = (torch.empty(s, device=DEV) for s in ((P, 256, 64), (P, 256, 256), (P, 256, 256), (P, 256, 64)))
    y = x0.clone()
    engine.nerf_glu_weights(params, gate, value, fc2)
    engine.rms_norm(y.view(-1, 64), scale, xn.view(-1, 64))
    engine.batched_matmul_Bt(xn, gate, x1)
    engine.batched_matmul_Bt(xn, value, x2)
    engine.silu_mul(x1, x2)
    engine.batched_matmul_Bt(x1, fc2, xo)
    engine.add_inplace(y, xo)
    torch.cuda.synchronize()
    engine.check_device_error()
    # fp64 with TF32 operand rounding
    pd = params.double()

    def l2(t):
        return t / t.norm(dim=-1, keepdim=True).clamp_min(1e-12)

    wg = _tf32(l2(pd[:, :16384].view(P, 64, 256).transpose(1, 2))).double()
    wv = _tf32(l2(pd[:, 16384:32768].view(P, 64, 256).transpose(1, 2))).double()
    wf = _tf32(l2(pd[:, 32768:].view(P, 256, 64).transpose(1, 2))).double()
    xd = x0.double()
    n = _tf32(xd * torch.rsqrt((xd * xd).mean(-1, keepdim=True) + 1e-6) * scale.double()).double()
    a1, a2 = n @ wg.transpose(1, 2), n @ wv.transpose(1, 2)
    h = _tf32((a1 / (1 + torch.exp(-a1))) * a2).double()
    want = xd + h @ wf.transpose(1, 2)
    d = want - xd
    assert ((x.double() - want).abs().max() / d.abs().max()).item() <= 2e-3
    assert ((x.double() - y.double()).abs().max() / d.abs().max()).item() <= 2e-3
