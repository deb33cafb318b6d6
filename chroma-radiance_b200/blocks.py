"""The GEMM + attention path of one Chroma double-stream and one single-stream block on the
engine, with the fusions the engine offers.

Mirrors the BF16 branch of the reference's block code, from the modulated bf16 inputs to the
updated residual streams; LayerNorm/modulation and the modulation vector are inputs here:

  double_block_forward (chroma.cuh:808-964), per stream s in {txt, img}:
      qkv_s = x_mod1_s . Wqkv_s^T + b            reference: 3 linear() calls, F32 out
      qk_norm + RoPE + attention over [txt; img]  reference: rms_norm x2, cuDNN SDPA, F32 out
      x_s  += gate1_s * (attn_s . Wproj_s^T + b)  reference: linear_gated_residual
      h_s   = gelu(x_mod2_s . Wmlp0_s^T + b)      reference: linear() F32 + gelu_to_bf16
      x_s  += gate2_s * (h_s . Wmlp2_s^T + b)     reference: linear() F32 + gated_residual
  single_block_forward (chroma.cuh:1101-1157):
      qkv   = x_mod . W1[0:9216]^T + b            reference: 3 linear() calls, F32 out
      mlp   = gelu(x_mod . W1[9216:]^T + b)       reference: linear() F32 + gelu_cuda
      attn  = attention(qk_norm(qkv))             reference: rms_norm x2 + cuDNN SDPA
      x    += gate * ([attn, mlp] . W2^T + b)     reference: concat_last_dim_to_bf16,
                                                  linear() F32, gated_residual
Engine fusions: the txt and img GEMMs of each double-block layer share one launch; the GELU
and the gated residual are GEMM epilogues; qk_norm and RoPE are fused into the qkv GEMM's
epilogue; the attention writes bf16 straight into the proj input / the concat buffer, and
the MLP half of linear1 writes GELU'd bf16 into the other concat columns.

Classifier-free guidance (forward_cfg, chroma.cuh:1499-1584) runs the blocks on a
conditional and an unconditional half that share every weight and modulation vector.  The
reference stacks M per stream ([txt_c; txt_u], [img_c; img_u]) in the double blocks and
re-assembles [txt_c, img_c | txt_u, img_u] for the single blocks (chroma.cuh:1546-1558),
gathering each half's [txt; img] rows around every attention (chroma.cuh:851-876).  Here the
F32 stream stays in the single blocks' layout throughout, half-major: rows [b*L, b*L + T) are
half b's txt tokens and [b*L + T, (b+1)*L) its img tokens.  Every double-block layer then
computes its four row blocks (txt_c, txt_u with the txt weights; img_c, img_u with the img
weights) in one launch, each half's attention reads its [txt; img] rows in place, and the
single block's linear1 covers both halves as one problem whose RoPE row is the token's row
modulo L.  The block functions take a guidance batch as lists of per-half row views (a plain
tensor is one half).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

import b2g

HIDDEN, HEADS, DHEAD, MLP = 3072, 24, 128, 12288


@dataclass
class StreamWeights:
    qkv_w: torch.Tensor   # bf16 [9216, 3072]
    qkv_b: torch.Tensor   # f32 [9216]
    q_norm: torch.Tensor  # f32 [128]
    k_norm: torch.Tensor
    proj_w: torch.Tensor  # bf16 [3072, 3072]
    proj_b: torch.Tensor
    mlp0_w: torch.Tensor  # bf16 [12288, 3072]
    mlp0_b: torch.Tensor
    mlp2_w: torch.Tensor  # bf16 [3072, 12288]
    mlp2_b: torch.Tensor


@dataclass
class SingleWeights:
    linear1_w: torch.Tensor  # bf16 [21504, 3072]
    linear1_b: torch.Tensor  # f32 [21504]
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    linear2_w: torch.Tensor  # bf16 [3072, 15360]
    linear2_b: torch.Tensor  # f32 [3072]


def _randn(gen: torch.Generator, shape, scale=1.0, shift=0.0):
    """N(shift, scale^2) drawn on the generator's own device."""
    return torch.randn(shape, generator=gen, device=gen.device) * scale + shift


def random_stream(gen: torch.Generator, dev) -> StreamWeights:
    def w(n, k):
        return _randn(gen, (n, k), 0.02).to(torch.bfloat16).to(dev)

    def b(n):
        return _randn(gen, n, 0.02).to(dev)

    def nrm():
        return _randn(gen, DHEAD, 0.1, 1.0).to(dev)

    return StreamWeights(w(3 * HIDDEN, HIDDEN), b(3 * HIDDEN), nrm(), nrm(), w(HIDDEN, HIDDEN), b(HIDDEN),
                         w(MLP, HIDDEN), b(MLP), w(HIDDEN, MLP), b(HIDDEN))


def random_single(gen: torch.Generator, dev) -> SingleWeights:
    return SingleWeights(_randn(gen, (3 * HIDDEN + MLP, HIDDEN), 0.02).to(torch.bfloat16).to(dev),
                         _randn(gen, 3 * HIDDEN + MLP, 0.02).to(dev),
                         _randn(gen, DHEAD, 0.1, 1.0).to(dev),
                         _randn(gen, DHEAD, 0.1, 1.0).to(dev),
                         _randn(gen, (HIDDEN, HIDDEN + MLP), 0.02).to(torch.bfloat16).to(dev),
                         _randn(gen, HIDDEN, 0.02).to(dev))


class Scratch:
    """Activation buffers of one block pair for `halves` guidance halves (rows half-major),
    allocated once (no allocation inside a step)."""

    def __init__(self, T: int, I: int, dev, halves: int = 1):
        L = T + I
        B = halves
        self.qkv = torch.empty((B * L, 3 * HIDDEN), dtype=torch.bfloat16, device=dev)  # normed, rotated
        self.attn = torch.empty((B * L, HIDDEN), dtype=torch.bfloat16, device=dev)
        self.h_img = torch.empty((B * I, MLP), dtype=torch.bfloat16, device=dev)
        self.h_txt = torch.empty((B * T, MLP), dtype=torch.bfloat16, device=dev)
        self.cat = torch.empty((B * L, HIDDEN + MLP), dtype=torch.bfloat16, device=dev)


def _halves(t) -> list:
    """Per-half row views: a list/tuple as given, a plain tensor as one half."""
    return list(t) if isinstance(t, (list, tuple)) else [t]


def _masks(mask, B: int) -> list:
    """Key bias per half: None, one [L] tensor shared by all halves, a [B, L] tensor or a list."""
    if mask is None:
        return [None] * B
    if isinstance(mask, (list, tuple)):
        assert len(mask) == B, "one key mask per guidance half"
        return list(mask)
    if mask.dim() == 2:
        assert mask.shape[0] == B, "one key mask row per guidance half"
        return [mask[b] for b in range(B)]
    return [mask] * B


def double_block(txt_w: StreamWeights, img_w: StreamWeights, txt_mod1, img_mod1, txt_mod2, img_mod2, txt, img,
                 txt_gate1, img_gate1, txt_gate2, img_gate2, pe, mask, s: Scratch, mark=None) -> None:
    """Updates txt [T, 3072] and img [I, 3072] (F32 residual streams) in place.

    `mark(label)`, when given, is called after each operation (labels and FLOPs in
    block_pair_ops order) so a caller can record events between the launches."""
    double_block_attention(txt_w, img_w, txt_mod1, img_mod1, txt, img, txt_gate1, img_gate1, pe, mask, s, mark)
    double_block_mlp(txt_w, img_w, txt_mod2, img_mod2, txt, img, txt_gate2, img_gate2, s, mark)


def double_block_attention(txt_w: StreamWeights, img_w: StreamWeights, txt_mod1, img_mod1, txt, img, txt_gate1,
                           img_gate1, pe, mask, s: Scratch, mark=None) -> None:
    """The attention half of a double block (chroma.cuh:808-905): qkv, attention, proj.

    txt_mod1, img_mod1, txt, img: row views [T, 3072] / [I, 3072], or lists of them, one per
    guidance half (the scratch then holds half b's rows at [b*L, (b+1)*L))."""
    mark = mark or _no_mark
    txt_m, img_m, txts, imgs = _halves(txt_mod1), _halves(img_mod1), _halves(txt), _halves(img)
    B, T = len(txts), txts[0].shape[0]
    L = T + imgs[0].shape[0]
    # Each layer's GEMMs over all row blocks share one launch (b2g_gemm_group): together their
    # tiles fill the SMs where the txt GEMM alone (M=512) would leave most of them idle.  The
    # qkv projection applies qk_norm and RoPE in its epilogue (txt rows take pe rows [0, T),
    # img rows [T, L): each half's attention sequence is its txt then its img tokens) and
    # writes the attention's bf16 operands.
    b2g.gemm_qkv_rope([dict(x=txt_m[b], w=txt_w.qkv_w, bias=txt_w.qkv_b, out=s.qkv[b * L:b * L + T], pe=pe[:T],
                            q_norm=txt_w.q_norm, k_norm=txt_w.k_norm) for b in range(B)] +
                      [dict(x=img_m[b], w=img_w.qkv_w, bias=img_w.qkv_b, out=s.qkv[b * L + T:(b + 1) * L],
                            pe=pe[T:L], q_norm=img_w.q_norm, k_norm=img_w.k_norm) for b in range(B)], HEADS)
    mark("double.qkv")
    for b, mb in enumerate(_masks(mask, B)):
        rows = s.qkv[b * L:(b + 1) * L]
        b2g.attention_bf16(rows[:, :HIDDEN], rows[:, HIDDEN:2 * HIDDEN], rows[:, 2 * HIDDEN:], HEADS, DHEAD,
                           attn_mask=mb, out=s.attn[b * L:(b + 1) * L])
    mark("double.attention")
    b2g.gemm_group([dict(x=s.attn[b * L:b * L + T], w=txt_w.proj_w, bias=txt_w.proj_b, out=txts[b],
                         epilogue="gated_residual", gate=txt_gate1) for b in range(B)] +
                   [dict(x=s.attn[b * L + T:(b + 1) * L], w=img_w.proj_w, bias=img_w.proj_b, out=imgs[b],
                         epilogue="gated_residual", gate=img_gate1) for b in range(B)])
    mark("double.proj")


def double_block_mlp(txt_w: StreamWeights, img_w: StreamWeights, txt_mod2, img_mod2, txt, img, txt_gate2,
                     img_gate2, s: Scratch, mark=None) -> None:
    """The MLP half of a double block (chroma.cuh:906-964): mlp0 + GELU, mlp2 + gated residual.
    Arguments as in double_block_attention."""
    mark = mark or _no_mark
    txt_m, img_m, txts, imgs = _halves(txt_mod2), _halves(img_mod2), _halves(txt), _halves(img)
    B, T, I = len(txts), txts[0].shape[0], imgs[0].shape[0]
    h_txt = [s.h_txt[b * T:(b + 1) * T] for b in range(B)]
    h_img = [s.h_img[b * I:(b + 1) * I] for b in range(B)]
    b2g.gemm_group([dict(x=txt_m[b], w=txt_w.mlp0_w, bias=txt_w.mlp0_b, out=h_txt[b], epilogue="gelu")
                    for b in range(B)] +
                   [dict(x=img_m[b], w=img_w.mlp0_w, bias=img_w.mlp0_b, out=h_img[b], epilogue="gelu")
                    for b in range(B)])
    mark("double.mlp0")
    b2g.gemm_group([dict(x=h_txt[b], w=txt_w.mlp2_w, bias=txt_w.mlp2_b, out=txts[b], epilogue="gated_residual",
                         gate=txt_gate2) for b in range(B)] +
                   [dict(x=h_img[b], w=img_w.mlp2_w, bias=img_w.mlp2_b, out=imgs[b], epilogue="gated_residual",
                         gate=img_gate2) for b in range(B)])
    mark("double.mlp2")


def single_block(w: SingleWeights, x_mod, x, gate, pe, mask, s: Scratch, mark=None) -> None:
    """Updates x [B*L, 3072] (F32 residual stream, B guidance halves of L = pe rows tokens,
    half-major) in place.  `mark` as in double_block."""
    mark = mark or _no_mark
    L = pe.shape[0]
    B = x.shape[0] // L
    assert B * L == x.shape[0], "x must hold whole guidance halves of pe.shape[0] rows"
    # linear1 in one launch over all halves (its weight rows are [q | k | v | mlp]): the qkv
    # columns get qk_norm + RoPE (row r rotated by pe row r % L) into s.qkv, the MLP columns
    # bias + GELU straight into the linear2 concat buffer.
    b2g.gemm_qkv_rope([dict(x=x_mod, w=w.linear1_w, bias=w.linear1_b, out=s.qkv[:B * L], pe=pe, pe_period=L,
                            q_norm=w.q_norm, k_norm=w.k_norm, gelu_out=s.cat[:B * L, HIDDEN:])], HEADS)
    mark("single.linear1")
    for b, mb in enumerate(_masks(mask, B)):
        rows = s.qkv[b * L:(b + 1) * L]
        b2g.attention_bf16(rows[:, :HIDDEN], rows[:, HIDDEN:2 * HIDDEN], rows[:, 2 * HIDDEN:], HEADS, DHEAD,
                           attn_mask=mb, out=s.cat[b * L:(b + 1) * L, :HIDDEN])
    mark("single.attention")
    b2g.gemm(s.cat[:B * L], w.linear2_w, w.linear2_b, out=x, epilogue="gated_residual", gate=gate)
    mark("single.linear2")


def _no_mark(label: str) -> None:
    pass


# ---------------------------------------------------------------------------- transformer pass
DOUBLE_BLOCKS, SINGLE_BLOCKS = 19, 38  # Chroma's layout (chroma.cuh:1499-1584)


@dataclass
class PassWeights:
    """Weights of every block of one transformer pass, and the modulation vectors the
    approximator would produce for it: per double block and stream [6, 3072] F32 (shift1,
    scale1, gate1, shift2, scale2, gate2), per single block [3, 3072] (shift, scale, gate)."""
    double: list          # [(txt StreamWeights, img StreamWeights)]
    single: list          # [SingleWeights]
    mods: torch.Tensor    # [DOUBLE_BLOCKS * 2 * 6 + SINGLE_BLOCKS * 3, 3072] F32


def random_pass(gen: torch.Generator, dev, n_double: int = DOUBLE_BLOCKS, n_single: int = SINGLE_BLOCKS) -> PassWeights:
    """Random-init weights of a whole pass (about 17 GB of bf16 for Chroma's 19 + 38 blocks)."""
    double = [(random_stream(gen, dev), random_stream(gen, dev)) for _ in range(n_double)]
    single = [random_single(gen, dev) for _ in range(n_single)]
    return PassWeights(double, single, mods=torch.zeros((n_double * 12 + n_single * 3, HIDDEN), device=dev))


class PassScratch(Scratch):
    """Scratch of a pass: the block buffers plus the modulated activations."""

    def __init__(self, T: int, I: int, dev, halves: int = 1):
        super().__init__(T, I, dev, halves)
        L = T + I
        self.mod = torch.empty((halves * L, HIDDEN), dtype=torch.bfloat16, device=dev)


def forward_pass(pw: PassWeights, x, pe, mask, s: PassScratch, T: int) -> None:
    """The transformer blocks of one denoising step (forward, chroma.cuh:1345-1493, or with
    guidance halves forward_cfg's block loop, chroma.cuh:1540-1563; without the embedders,
    approximator, final layer and cfg_blend): the double blocks on the txt and img rows of the
    F32 stream x [B*L, 3072] (B = x rows / pe rows guidance halves, half-major: half b's txt
    rows at [b*L, b*L + T), its img rows after them), then the single blocks on x, every block
    modulating its inputs on the device (modulate_to_bf16, kernels.cu:552-599) as the
    reference's blocks do.  x is updated in place; txt and img are row views of it, so the
    double-to-single concatenation costs nothing.  mask: one [L] key bias for every half, or
    one per half ([B, L] or a list)."""
    L = pe.shape[0]
    B = x.shape[0] // L
    assert B * L == x.shape[0] and 0 < T < L, "x must hold whole guidance halves of pe.shape[0] rows"
    txts = [x[b * L:b * L + T] for b in range(B)]
    imgs = [x[b * L + T:(b + 1) * L] for b in range(B)]
    mod_t = [s.mod[b * L:b * L + T] for b in range(B)]
    mod_i = [s.mod[b * L + T:(b + 1) * L] for b in range(B)]
    for i, (tw, iw) in enumerate(pw.double):
        mt, mi = pw.mods[12 * i:12 * i + 6], pw.mods[12 * i + 6:12 * i + 12]
        for b in range(B):
            b2g.modulate_to_bf16(txts[b], mt[0], mt[1], out=mod_t[b])
            b2g.modulate_to_bf16(imgs[b], mi[0], mi[1], out=mod_i[b])
        double_block_attention(tw, iw, mod_t, mod_i, txts, imgs, mt[2], mi[2], pe, mask, s)
        for b in range(B):
            b2g.modulate_to_bf16(txts[b], mt[3], mt[4], out=mod_t[b])
            b2g.modulate_to_bf16(imgs[b], mi[3], mi[4], out=mod_i[b])
        double_block_mlp(tw, iw, mod_t, mod_i, txts, imgs, mt[5], mi[5], s)
    base = 12 * len(pw.double)
    for i, sw in enumerate(pw.single):
        m = pw.mods[base + 3 * i:base + 3 * i + 3]
        b2g.modulate_to_bf16(x, m[0], m[1], out=s.mod[:B * L])
        single_block(sw, s.mod[:B * L], x, m[2], pe, mask, s)


def pass_flops(T: int, I: int, n_double: int = DOUBLE_BLOCKS, n_single: int = SINGLE_BLOCKS,
               halves: int = 1) -> float:
    """GEMM + attention (unmasked) FLOPs of forward_pass; the modulations are not counted."""
    ops = block_pair_ops(T, I)
    dbl = sum(f for lab, _, f in ops if lab.startswith("double."))
    sgl = sum(f for lab, _, f in ops if lab.startswith("single."))
    return halves * (n_double * dbl + n_single * sgl)


def block_pair_ops(T: int, I: int) -> list[tuple[str, str, float]]:
    """(label, kind, FLOPs) of every operation of one double + one single block, in launch order.

    kind "gemm" is one engine GEMM launch (2*M*N*K summed over its problems); kind
    "attention" is the whole attention (QK^T + PV over 24 heads, 4*L*L*3072, unmasked)."""
    L = T + I
    H3, H = 3 * HIDDEN, HIDDEN
    att = 4.0 * L * L * HIDDEN
    return [("double.qkv", "gemm", 2.0 * L * H3 * H), ("double.attention", "attention", att),
            ("double.proj", "gemm", 2.0 * L * H * H), ("double.mlp0", "gemm", 2.0 * L * MLP * H),
            ("double.mlp2", "gemm", 2.0 * L * H * MLP),
            ("single.linear1", "gemm", 2.0 * L * (H3 + MLP) * H),
            ("single.attention", "attention", att), ("single.linear2", "gemm", 2.0 * L * H * (H + MLP))]


def block_pair_flops(T: int, I: int) -> tuple[float, float]:
    """(linear FLOPs, attention FLOPs counted unmasked) of one double + one single block."""
    ops = block_pair_ops(T, I)
    return (sum(f for _, kind, f in ops if kind == "gemm"), sum(f for _, kind, f in ops if kind == "attention"))
