"""BASELINE config 2 through the engine's block path (chroma-radiance_b200/blocks.py) against
the reference's own block code (qkv linears, qk_norm, cuDNN attention, gated residuals,
GELU, concat) on identical inputs: one double-stream and one single-stream block at 512^2,
24 heads x 128, key mask on 400 of the 512 text tokens.

Tolerance: the residual-stream update (x_out - x_in) of each stream, compared over the whole
block, within 1e-2 of its max and cosine >= 0.9999 (bf16 operands and activations throughout,
different rounding points between the fused and unfused paths).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def attn_ref():
    from oracle import ATTN_REF_PATH, AttnRef

    if not ATTN_REF_PATH.exists():
        pytest.skip("reference attention/block library not built")
    return AttnRef()


def cos(a, b):
    a, b = a.double().cpu().numpy().ravel(), b.double().cpu().numpy().ravel()
    return a @ b / np.sqrt((a @ a) * (b @ b))


def check_delta(mine, theirs, x0):
    dm, dt = mine - x0, theirs - x0
    assert rel_err(dm.cpu().numpy(), dt.cpu().numpy()) < 1e-2
    assert cos(dm, dt) > 0.9999


@pytest.fixture(scope="module")
def setup(engine):
    import blocks

    g = torch.Generator().manual_seed(42)
    T, I = 512, 1024
    L = T + I
    txt_w, img_w = blocks.random_stream(g, DEV), blocks.random_stream(g, DEV)
    sw = blocks.random_single(g, DEV)

    def act(m, dt=torch.bfloat16):
        return torch.randn((m, blocks.HIDDEN), generator=g).to(dt).to(DEV)

    acts = dict(txt_mod1=act(T), img_mod1=act(I), txt_mod2=act(T), img_mod2=act(I), txt=act(T, torch.float32),
                img=act(I, torch.float32), x_mod=act(L), x=act(L, torch.float32))
    gates = [torch.randn(blocks.HIDDEN, generator=g).to(DEV) for _ in range(5)]
    ang = torch.rand((L, blocks.DHEAD // 2), generator=g) * 6.283
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous().to(DEV)
    mask = torch.zeros(L)
    mask[T - 400:T] = float("-inf")
    return dict(T=T, I=I, L=L, txt_w=txt_w, img_w=img_w, sw=sw, acts=acts, gates=gates, pe=pe, mask=mask.to(DEV),
                scratch=blocks.Scratch(T, I, DEV))


def test_double_block_vs_reference(engine, setup):
    import blocks

    ref = attn_ref()
    s = setup
    a, gt = s["acts"], s["gates"]
    txt, img = a["txt"].clone(), a["img"].clone()
    blocks.double_block(s["txt_w"], s["img_w"], a["txt_mod1"], a["img_mod1"], a["txt_mod2"], a["img_mod2"], txt, img,
                        gt[0], gt[1], gt[2], gt[3], s["pe"], s["mask"], s["scratch"])
    rtxt, rimg = a["txt"].clone(), a["img"].clone()
    ptrs = []
    for w in (s["img_w"], s["txt_w"]):
        ptrs += [w.qkv_w.data_ptr(), w.qkv_b.data_ptr(), w.q_norm.data_ptr(), w.k_norm.data_ptr(),
                 w.proj_w.data_ptr(), w.proj_b.data_ptr(), w.mlp0_w.data_ptr(), w.mlp0_b.data_ptr(),
                 w.mlp2_w.data_ptr(), w.mlp2_b.data_ptr()]
    ptrs += [a["img_mod1"].data_ptr(), a["txt_mod1"].data_ptr(), a["img_mod2"].data_ptr(), a["txt_mod2"].data_ptr(),
             rimg.data_ptr(), rtxt.data_ptr(), gt[1].data_ptr(), gt[0].data_ptr(), gt[3].data_ptr(),
             gt[2].data_ptr(), s["pe"].data_ptr(), s["mask"].data_ptr()]
    assert ref.double_block(ptrs, s["T"], s["I"]) == 0
    torch.cuda.synchronize()
    check_delta(txt, rtxt, a["txt"])
    check_delta(img, rimg, a["img"])


def test_single_block_vs_reference(engine, setup):
    import blocks

    ref = attn_ref()
    s = setup
    a, sw = s["acts"], s["sw"]
    x = a["x"].clone()
    blocks.single_block(sw, a["x_mod"], x, s["gates"][4], s["pe"], s["mask"], s["scratch"])
    rx = a["x"].clone()
    ptrs = [sw.linear1_w.data_ptr(), sw.linear1_b.data_ptr(), sw.q_norm.data_ptr(), sw.k_norm.data_ptr(),
            sw.linear2_w.data_ptr(), sw.linear2_b.data_ptr(), a["x_mod"].data_ptr(), rx.data_ptr(),
            s["gates"][4].data_ptr(), s["pe"].data_ptr(), s["mask"].data_ptr()]
    assert ref.single_block(ptrs, s["L"]) == 0
    torch.cuda.synchronize()
    check_delta(x, rx, a["x"])


def test_block_pair_in_cuda_graph_matches_eager(engine, setup):
    """The bench replays the block pair as a CUDA graph; replay must equal eager execution."""
    import blocks

    s = setup
    a, gt = s["acts"], s["gates"]
    state = {k: a[k].clone() for k in ("txt", "img", "x")}

    def step(st):
        blocks.double_block(s["txt_w"], s["img_w"], a["txt_mod1"], a["img_mod1"], a["txt_mod2"], a["img_mod2"],
                            st["txt"], st["img"], gt[0], gt[1], gt[2], gt[3], s["pe"], s["mask"], s["scratch"])
        blocks.single_block(s["sw"], a["x_mod"], st["x"], gt[4], s["pe"], s["mask"], s["scratch"])

    eager = {k: a[k].clone() for k in ("txt", "img", "x")}
    step(eager)
    step(state)  # warm-up (workspaces sized) before capture
    for k in state:
        state[k].copy_(a[k])
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            step(state)
    for k in state:
        state[k].copy_(a[k])
    graph.replay()
    torch.cuda.synchronize()
    for k in state:
        assert torch.equal(state[k], eager[k]), k


def test_forward_pass_is_the_blocks_in_sequence(engine):
    """blocks.forward_pass over a short pass (2 double + 2 single blocks, txt/img as row views
    of the single blocks' stream, every block modulating its inputs on the device) gives the
    same bits as calling modulate_to_bf16 and the block functions one by one, and stays finite."""
    import blocks

    T, I = 128, 256
    L = T + I
    g = torch.Generator(device=DEV).manual_seed(5)
    pw = blocks.random_pass(g, DEV, n_double=2, n_single=2)
    pw.mods.copy_(torch.randn(tuple(pw.mods.shape), generator=g, device=DEV) * 0.1)
    ang = torch.rand((L, blocks.DHEAD // 2), generator=g, device=DEV) * 6.2831853
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    mask = torch.zeros(L, device=DEV)
    mask[T - 40:T] = float("-inf")
    x0 = torch.randn((L, blocks.HIDDEN), generator=g, device=DEV)

    x = x0.clone()
    blocks.forward_pass(pw, x, pe, mask, blocks.PassScratch(T, I, DEV), T)

    y = x0.clone()
    s = blocks.PassScratch(T, I, DEV)
    txt, img = y[:T], y[T:]
    for i, (tw, iw) in enumerate(pw.double):
        mt, mi = blocks.double_mods(pw.mods, i, len(pw.double), len(pw.single))
        m1t, m1i = engine.modulate_to_bf16(txt, mt[0], mt[1]), engine.modulate_to_bf16(img, mi[0], mi[1])
        blocks.double_block_attention(tw, iw, m1t, m1i, txt, img, mt[2], mi[2], pe, mask, s)
        m2t, m2i = engine.modulate_to_bf16(txt, mt[3], mt[4]), engine.modulate_to_bf16(img, mi[3], mi[4])
        blocks.double_block_mlp(tw, iw, m2t, m2i, txt, img, mt[5], mi[5], s)
    for i, sw in enumerate(pw.single):
        m = blocks.single_mods(pw.mods, i)
        blocks.single_block(sw, engine.modulate_to_bf16(y, m[0], m[1]), y, m[2], pe, mask, s)
    torch.cuda.synchronize()
    assert torch.isfinite(x).all()
    assert torch.equal(x, y)
    assert not torch.equal(x, x0)
    assert blocks.pass_flops(T, I, 2, 2) > 0


def test_cfg_pass_equals_each_half_alone(engine):
    """forward_pass over two guidance halves stacked half-major (each with its own key mask:
    the conditional prompt and an almost empty unconditional one) against the same pass on each
    half alone.  With one GEMM variant forced (2-CTA tiles, no split-K) every tile runs the same
    instructions on the same data in both, so the results are bit-identical; with the
    variants the cost model picks (the CFG launches have twice the tiles, and may get another
    variant) they agree to bf16 rounding of the activations, as check_delta states."""
    import blocks

    T, I = 128, 256
    L = T + I
    g = torch.Generator(device=DEV).manual_seed(9)
    pw = blocks.random_pass(g, DEV, n_double=2, n_single=2)
    pw.mods.copy_(torch.randn(tuple(pw.mods.shape), generator=g, device=DEV) * 0.1)
    ang = torch.rand((L, blocks.DHEAD // 2), generator=g, device=DEV) * 6.2831853
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    masks = torch.zeros((2, L), device=DEV)
    masks[0, T - 40:T] = float("-inf")
    masks[1, 1:T] = float("-inf")
    x0 = torch.randn((2 * L, blocks.HIDDEN), generator=g, device=DEV)
    for variant in (2, -1):
        engine.set_gemm_variant(variant, 0)
        try:
            x = x0.clone()
            blocks.forward_pass(pw, x, pe, masks, blocks.PassScratch(T, I, DEV, halves=2), T)
            ys = []
            for b in range(2):
                y = x0[b * L:(b + 1) * L].clone()
                blocks.forward_pass(pw, y, pe, masks[b], blocks.PassScratch(T, I, DEV), T)
                ys.append(y)
            torch.cuda.synchronize()
        finally:
            engine.set_gemm_variant(-1, 0)
        assert torch.isfinite(x).all()
        for b in range(2):
            if variant == 2:
                assert torch.equal(x[b * L:(b + 1) * L], ys[b]), f"half {b}"
            else:
                check_delta(x[b * L:(b + 1) * L], ys[b], x0[b * L:(b + 1) * L])
    assert not torch.equal(x[:L], x[L:])


def test_fp8_block_pair_close_to_bf16(engine, setup):
    """Config 5's transformer block pair (E4M3 weights per channel, per-token E4M3 activations,
    the bf16 path's epilogues) against the bf16 block pair on the same weights and inputs:
    the difference is E4M3 rounding of both operands of every linear (2.65% relative per
    element on Gaussian operands), so the residual-stream update agrees to max|d|/max|ref|
    <= 0.1 and cosine >= 0.998."""
    import blocks

    s = setup
    a, gt = s["acts"], s["gates"]
    T, I, L = s["T"], s["I"], s["L"]
    tw8, iw8 = blocks.quantize_stream(s["txt_w"]), blocks.quantize_stream(s["img_w"])
    sw8 = blocks.quantize_single(s["sw"])
    s8 = blocks.ScratchFP8(T, I, DEV)
    q8 = {k: blocks.Q8(*engine.quantize_e4m3(a[k])) for k in ("txt_mod1", "img_mod1", "txt_mod2", "img_mod2",
                                                              "x_mod")}
    txt, img, x = a["txt"].clone(), a["img"].clone(), a["x"].clone()
    blocks.double_block_attention_fp8(tw8, iw8, q8["txt_mod1"], q8["img_mod1"], txt, img, gt[0], gt[1], s["pe"],
                                      s["mask"], s8)
    blocks.double_block_mlp_fp8(tw8, iw8, q8["txt_mod2"], q8["img_mod2"], txt, img, gt[2], gt[3], s8)
    blocks.single_block_fp8(sw8, q8["x_mod"], x, gt[4], s["pe"], s["mask"], s8)
    rtxt, rimg, rx = a["txt"].clone(), a["img"].clone(), a["x"].clone()
    blocks.double_block(s["txt_w"], s["img_w"], a["txt_mod1"], a["img_mod1"], a["txt_mod2"], a["img_mod2"], rtxt,
                        rimg, gt[0], gt[1], gt[2], gt[3], s["pe"], s["mask"], s["scratch"])
    blocks.single_block(s["sw"], a["x_mod"], rx, gt[4], s["pe"], s["mask"], s["scratch"])
    torch.cuda.synchronize()
    engine.check_device_error()
    for mine, ref, x0 in ((txt, rtxt, a["txt"]), (img, rimg, a["img"]), (x, rx, a["x"])):
        dm, dr = (mine - x0).double(), (ref - x0).double()
        err = float((dm - dr).abs().max() / dr.abs().max())
        c = cos(dm, dr)
        print(f"fp8 vs bf16: max rel {err:.4f} cos {c:.6f}")
        assert err <= 0.1 and c >= 0.998


def test_fp8_cfg_pass_equals_each_half_alone(engine):
    """forward_pass_fp8 over two stacked guidance halves is bit-identical to each half alone
    with the GEMM variant fixed (the quantisations are per row, so they see the same rows)."""
    import blocks

    T, I = 128, 256
    L = T + I
    g = torch.Generator(device=DEV).manual_seed(13)
    pw = blocks.random_pass(g, DEV, n_double=2, n_single=2)
    pw.mods.copy_(torch.randn(tuple(pw.mods.shape), generator=g, device=DEV) * 0.1)
    pw8 = blocks.quantize_pass(pw)
    ang = torch.rand((L, blocks.DHEAD // 2), generator=g, device=DEV) * 6.2831853
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    masks = torch.zeros((2, L), device=DEV)
    masks[0, T - 40:T] = float("-inf")
    masks[1, 1:T] = float("-inf")
    x0 = torch.randn((2 * L, blocks.HIDDEN), generator=g, device=DEV)
    engine.set_gemm_variant(2, 0)
    try:
        x = x0.clone()
        blocks.forward_pass_fp8(pw8, x, pe, masks, blocks.ScratchFP8(T, I, DEV, halves=2), T)
        ys = []
        for b in range(2):
            y = x0[b * L:(b + 1) * L].clone()
            blocks.forward_pass_fp8(pw8, y, pe, masks[b], blocks.ScratchFP8(T, I, DEV), T)
            ys.append(y)
        torch.cuda.synchronize()
    finally:
        engine.set_gemm_variant(-1, 0)
    assert torch.isfinite(x).all()
    for b in range(2):
        assert torch.equal(x[b * L:(b + 1) * L], ys[b]), f"half {b}"


def test_short_pass_chained_vs_reference(engine, ref):
    """The north star's full-forward criterion (output cosine >= 0.999) on a chained pass of 2
    double + 2 single blocks at 512^2 (T=512, I=1024): the engine's forward_pass against the
    reference's own code run the same way: its modulate_to_bf16 on the current residual
    streams before each half of each block (kernels.cu:552-599), its double block's attention
    and MLP halves (chroma.cuh:808-964) and its single block (chroma.cuh:1101-1157), every
    block on its own random weights and modulation vectors.  Compared: the update of the F32
    stream over the whole pass, cosine >= 0.999 (the north star's bar) and max|d|/max|ref| <=
    5e-3 (bf16 operands and activations on both sides, rounded at different points and
    compounding over four blocks; measured 2.0e-3, cosine 0.999999)."""
    import blocks

    attn = attn_ref()
    T, I = 512, 1024
    L, H = T + I, blocks.HIDDEN
    g = torch.Generator(device=DEV).manual_seed(21)
    pw = blocks.random_pass(g, DEV, n_double=2, n_single=2)
    pw.mods.copy_(torch.randn(tuple(pw.mods.shape), generator=g, device=DEV) * 0.1)
    ang = torch.rand((L, blocks.DHEAD // 2), generator=g, device=DEV) * 6.2831853
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    mask = torch.zeros(L, device=DEV)
    mask[T - 400:T] = float("-inf")
    x0 = torch.randn((L, H), generator=g, device=DEV)

    x = x0.clone()
    blocks.forward_pass(pw, x, pe, mask, blocks.PassScratch(T, I, DEV), T)

    xr = x0.clone()
    txt, img = xr[:T], xr[T:]
    m1t, m2t = (torch.empty((T, H), dtype=torch.bfloat16, device=DEV) for _ in range(2))
    m1i, m2i = (torch.empty((I, H), dtype=torch.bfloat16, device=DEV) for _ in range(2))
    xm = torch.empty((L, H), dtype=torch.bfloat16, device=DEV)

    def modulate(src, shift, scale, out):
        assert ref.modulate_to_bf16(src.data_ptr(), shift.data_ptr(), scale.data_ptr(), out.data_ptr(),
                                    src.shape[0], H, 1e-6) == 0

    def wptrs(w):
        return [w.qkv_w.data_ptr(), w.qkv_b.data_ptr(), w.q_norm.data_ptr(), w.k_norm.data_ptr(),
                w.proj_w.data_ptr(), w.proj_b.data_ptr(), w.mlp0_w.data_ptr(), w.mlp0_b.data_ptr(),
                w.mlp2_w.data_ptr(), w.mlp2_b.data_ptr()]

    for i, (tw, iw) in enumerate(pw.double):
        mt, mi = blocks.double_mods(pw.mods, i, len(pw.double), len(pw.single))
        ptrs = wptrs(iw) + wptrs(tw) + [m1i.data_ptr(), m1t.data_ptr(), m2i.data_ptr(), m2t.data_ptr(),
                                        img.data_ptr(), txt.data_ptr(), mi[2].data_ptr(), mt[2].data_ptr(),
                                        mi[5].data_ptr(), mt[5].data_ptr(), pe.data_ptr(), mask.data_ptr()]
        modulate(txt, mt[0], mt[1], m1t)
        modulate(img, mi[0], mi[1], m1i)
        assert attn.double_block_attn(ptrs, T, I) == 0
        modulate(txt, mt[3], mt[4], m2t)
        modulate(img, mi[3], mi[4], m2i)
        assert attn.double_block_mlp(ptrs, T, I) == 0
    for j, sw in enumerate(pw.single):
        m = blocks.single_mods(pw.mods, j)
        modulate(xr, m[0], m[1], xm)
        assert attn.single_block([sw.linear1_w.data_ptr(), sw.linear1_b.data_ptr(), sw.q_norm.data_ptr(),
                                  sw.k_norm.data_ptr(), sw.linear2_w.data_ptr(), sw.linear2_b.data_ptr(),
                                  xm.data_ptr(), xr.data_ptr(), m[2].data_ptr(), pe.data_ptr(),
                                  mask.data_ptr()], L) == 0
    torch.cuda.synchronize()
    dm, dr = (x - x0).double(), (xr - x0).double()
    err = float((dm - dr).abs().max() / dr.abs().max())
    c = cos(dm, dr)
    print(f"chained 2+2 blocks: cosine {c:.6f}, max rel {err:.4f}")
    assert torch.isfinite(x).all() and c >= 0.999 and err <= 5e-3


def test_fp8_full_pass_close_to_bf16(engine):
    """Config 5's FP8 transformer over a whole pass (Chroma's 19 double + 38 single blocks at
    512^2, both guidance halves, E4M3 weights per channel and per-token E4M3 activations)
    against the bf16 pass on the same random weights, modulation vectors and inputs.  Every
    linear of every block rounds both operands to E4M3 (3.7% RMS relative error per K=3072
    product on Gaussian operands), and the residual streams carry it through 57 blocks: the
    update x_out - x_in agrees to cosine >= 0.995 (the measured value is printed)."""
    import blocks

    T, I = 512, 1024
    L = T + I
    g = torch.Generator(device=DEV).manual_seed(21)
    pw = blocks.random_pass(g, DEV)
    pw.mods.copy_(torch.randn(tuple(pw.mods.shape), generator=g, device=DEV) * 0.1)
    pw8 = blocks.quantize_pass(pw)
    ang = torch.rand((L, blocks.DHEAD // 2), generator=g, device=DEV) * 6.2831853
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    masks = torch.zeros((2, L), device=DEV)
    masks[0, 112:T] = float("-inf")
    masks[1, 2:T] = float("-inf")
    x0 = torch.randn((2 * L, blocks.HIDDEN), generator=g, device=DEV)
    x16, x8 = x0.clone(), x0.clone()
    blocks.forward_pass(pw, x16, pe, masks, blocks.PassScratch(T, I, DEV, halves=2), T)
    blocks.forward_pass_fp8(pw8, x8, pe, masks, blocks.ScratchFP8(T, I, DEV, halves=2), T)
    torch.cuda.synchronize()
    engine.check_device_error()
    d16, d8 = (x16 - x0).double(), (x8 - x0).double()
    c = float((d16.flatten() @ d8.flatten()) / (d16.norm() * d8.norm()))
    err = float((d8 - d16).abs().max() / d16.abs().max())
    print(f"fp8 vs bf16 57-block pass: cosine {c:.6f}, max|d|/max|ref| {err:.4f}")
    assert torch.isfinite(x8).all()
    assert c >= 0.995
