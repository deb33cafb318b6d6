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
and the gated residual are GEMM epilogues; qk_norm is fused into the
attention's RoPE producer; the attention writes bf16 straight into the proj input / the
concat buffer, and the MLP half of linear1 writes GELU'd bf16 into the other concat columns.
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
    """Activation buffers of one block pair, allocated once (no allocation inside a step)."""

    def __init__(self, T: int, I: int, dev):
        L = T + I
        self.qkv = torch.empty((L, 3 * HIDDEN), dtype=torch.bfloat16, device=dev)  # normed, rotated
        self.attn = torch.empty((L, HIDDEN), dtype=torch.bfloat16, device=dev)
        self.h_img = torch.empty((I, MLP), dtype=torch.bfloat16, device=dev)
        self.h_txt = torch.empty((T, MLP), dtype=torch.bfloat16, device=dev)
        self.cat = torch.empty((L, HIDDEN + MLP), dtype=torch.bfloat16, device=dev)


def double_block(txt_w: StreamWeights, img_w: StreamWeights, txt_mod1, img_mod1, txt_mod2, img_mod2, txt, img,
                 txt_gate1, img_gate1, txt_gate2, img_gate2, pe, mask, s: Scratch, mark=None) -> None:
    """Updates txt [T, 3072] and img [I, 3072] (F32 residual streams) in place.

    `mark(label)`, when given, is called after each operation (labels and FLOPs in
    block_pair_ops order) so a caller can record events between the launches."""
    double_block_attention(txt_w, img_w, txt_mod1, img_mod1, txt, img, txt_gate1, img_gate1, pe, mask, s, mark)
    double_block_mlp(txt_w, img_w, txt_mod2, img_mod2, txt, img, txt_gate2, img_gate2, s, mark)


def double_block_attention(txt_w: StreamWeights, img_w: StreamWeights, txt_mod1, img_mod1, txt, img, txt_gate1,
                           img_gate1, pe, mask, s: Scratch, mark=None) -> None:
    """The attention half of a double block (chroma.cuh:808-905): qkv, attention, proj."""
    mark = mark or _no_mark
    T = txt.shape[0]
    # Each layer's txt and img GEMMs share one launch (b2g_gemm_group): together their tiles
    # fill the SMs where the txt GEMM alone (M=512) would leave most of them idle.  The qkv
    # projection applies qk_norm and RoPE in its epilogue (txt rows take pe rows [0, T), img
    # rows [T, L): the attention sequence is txt then img) and writes the attention's bf16
    # operands.
    b2g.gemm_qkv_rope([dict(x=txt_mod1, w=txt_w.qkv_w, bias=txt_w.qkv_b, out=s.qkv[:T], pe=pe[:T],
                            q_norm=txt_w.q_norm, k_norm=txt_w.k_norm),
                       dict(x=img_mod1, w=img_w.qkv_w, bias=img_w.qkv_b, out=s.qkv[T:], pe=pe[T:],
                            q_norm=img_w.q_norm, k_norm=img_w.k_norm)], HEADS)
    mark("double.qkv")
    q, k, v = s.qkv[:, :HIDDEN], s.qkv[:, HIDDEN:2 * HIDDEN], s.qkv[:, 2 * HIDDEN:]
    b2g.attention_bf16(q, k, v, HEADS, DHEAD, attn_mask=mask, out=s.attn)
    mark("double.attention")
    b2g.gemm_group([dict(x=s.attn[:T], w=txt_w.proj_w, bias=txt_w.proj_b, out=txt, epilogue="gated_residual",
                         gate=txt_gate1),
                    dict(x=s.attn[T:], w=img_w.proj_w, bias=img_w.proj_b, out=img, epilogue="gated_residual",
                         gate=img_gate1)])
    mark("double.proj")


def double_block_mlp(txt_w: StreamWeights, img_w: StreamWeights, txt_mod2, img_mod2, txt, img, txt_gate2,
                     img_gate2, s: Scratch, mark=None) -> None:
    """The MLP half of a double block (chroma.cuh:906-964): mlp0 + GELU, mlp2 + gated residual."""
    mark = mark or _no_mark
    b2g.gemm_group([dict(x=txt_mod2, w=txt_w.mlp0_w, bias=txt_w.mlp0_b, out=s.h_txt, epilogue="gelu"),
                    dict(x=img_mod2, w=img_w.mlp0_w, bias=img_w.mlp0_b, out=s.h_img, epilogue="gelu")])
    mark("double.mlp0")
    b2g.gemm_group([dict(x=s.h_txt, w=txt_w.mlp2_w, bias=txt_w.mlp2_b, out=txt, epilogue="gated_residual",
                         gate=txt_gate2),
                    dict(x=s.h_img, w=img_w.mlp2_w, bias=img_w.mlp2_b, out=img, epilogue="gated_residual",
                         gate=img_gate2)])
    mark("double.mlp2")


def single_block(w: SingleWeights, x_mod, x, gate, pe, mask, s: Scratch, mark=None) -> None:
    """Updates x [L, 3072] (F32 residual stream) in place.  `mark` as in double_block."""
    mark = mark or _no_mark
    # linear1 in one launch (its weight rows are [q | k | v | mlp]): the qkv columns get qk_norm
    # + RoPE into s.qkv, the MLP columns bias + GELU straight into the linear2 concat buffer.
    b2g.gemm_qkv_rope([dict(x=x_mod, w=w.linear1_w, bias=w.linear1_b, out=s.qkv, pe=pe, q_norm=w.q_norm,
                            k_norm=w.k_norm, gelu_out=s.cat[:, HIDDEN:])], HEADS)
    mark("single.linear1")
    q, k, v = s.qkv[:, :HIDDEN], s.qkv[:, HIDDEN:2 * HIDDEN], s.qkv[:, 2 * HIDDEN:]
    b2g.attention_bf16(q, k, v, HEADS, DHEAD, attn_mask=mask, out=s.cat[:, :HIDDEN])
    mark("single.attention")
    b2g.gemm(s.cat, w.linear2_w, w.linear2_b, out=x, epilogue="gated_residual", gate=gate)
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

    def __init__(self, T: int, I: int, dev):
        super().__init__(T, I, dev)
        L = T + I
        self.mod = torch.empty((L, HIDDEN), dtype=torch.bfloat16, device=dev)


def forward_pass(pw: PassWeights, x, pe, mask, s: PassScratch, T: int) -> None:
    """The transformer blocks of one denoising step (forward, chroma.cuh:1345-1493, without the
    embedders, approximator and final layer): the double blocks on the txt rows x[:T] and img
    rows x[T:] of the F32 stream x [L, 3072], then the single blocks on x, every block
    modulating its inputs on the device (modulate_to_bf16, kernels.cu:552-599) as the
    reference's blocks do.  x is updated in place; txt and img are row views of it, so the
    double-to-single concatenation costs nothing."""
    txt, img = x[:T], x[T:]
    for i, (tw, iw) in enumerate(pw.double):
        mt, mi = pw.mods[12 * i:12 * i + 6], pw.mods[12 * i + 6:12 * i + 12]
        b2g.modulate_to_bf16(txt, mt[0], mt[1], out=s.mod[:T])
        b2g.modulate_to_bf16(img, mi[0], mi[1], out=s.mod[T:])
        double_block_attention(tw, iw, s.mod[:T], s.mod[T:], txt, img, mt[2], mi[2], pe, mask, s)
        b2g.modulate_to_bf16(txt, mt[3], mt[4], out=s.mod[:T])
        b2g.modulate_to_bf16(img, mi[3], mi[4], out=s.mod[T:])
        double_block_mlp(tw, iw, s.mod[:T], s.mod[T:], txt, img, mt[5], mi[5], s)
    base = 12 * len(pw.double)
    for i, sw in enumerate(pw.single):
        m = pw.mods[base + 3 * i:base + 3 * i + 3]
        b2g.modulate_to_bf16(x, m[0], m[1], out=s.mod)
        single_block(sw, s.mod, x, m[2], pe, mask, s)


def pass_flops(T: int, I: int, n_double: int = DOUBLE_BLOCKS, n_single: int = SINGLE_BLOCKS) -> float:
    """GEMM + attention (unmasked) FLOPs of forward_pass; the modulations are not counted."""
    ops = block_pair_ops(T, I)
    dbl = sum(f for lab, _, f in ops if lab.startswith("double."))
    sgl = sum(f for lab, _, f in ops if lab.startswith("single."))
    return n_double * dbl + n_single * sgl


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
