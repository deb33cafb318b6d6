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
        self.h = torch.empty((B * L, MLP), dtype=torch.bfloat16, device=dev)  # txt rows of all halves, then img
        self.h_txt = self.h[:B * T]
        self.h_img = self.h[B * T:]
        self.cat = torch.empty((B * L, HIDDEN + MLP), dtype=torch.bfloat16, device=dev)


def _halves(t) -> list:
    """Per-half row views: a list/tuple as given, a plain tensor as one half."""
    return list(t) if isinstance(t, (list, tuple)) else [t]


def _rope_table(pe, s):
    """pe in its compact (cos, sin) form when it has the rotation form (every RoPE table does):
    the qkv epilogue then reads half the bytes.  Made once per table and kept on the scratch,
    so a captured graph reuses the same tensor."""
    if getattr(s, "_pe_src", None) is not pe:
        s._pe_src = pe
        s._pe_c = b2g.compact_rope_table(pe)
    return s._pe_c if s._pe_c is not None else pe


def _attention(qkv, mask, B: int, L: int, out) -> None:
    """The attention of every guidance half over the half-major [q | k | v] rows of qkv into
    the same rows of out: one launch for all halves (attention_bf16_batched) when the key
    biases are one [L] tensor or a contiguous [B, L] tensor, else one launch per half."""
    R = B * L
    q, k, v = qkv[:R, :HIDDEN], qkv[:R, HIDDEN:2 * HIDDEN], qkv[:R, 2 * HIDDEN:]
    if B == 1:
        b2g.attention_bf16(q, k, v, HEADS, DHEAD, attn_mask=_masks(mask, 1)[0], out=out[:R])
        return
    if mask is None or (torch.is_tensor(mask) and mask.is_contiguous() and
                        (mask.dim() == 1 or tuple(mask.shape) == (B, L))):
        b2g.attention_bf16_batched(q, k, v, HEADS, DHEAD, B, attn_mask=mask, out=out[:R])
        return
    for b, mb in enumerate(_masks(mask, B)):
        rows = slice(b * L, (b + 1) * L)
        b2g.attention_bf16(q[rows], k[rows], v[rows], HEADS, DHEAD, attn_mask=mb, out=out[rows])


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
    pe = _rope_table(pe, s)
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
    _attention(s.qkv, mask, B, L, s.attn)
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
    pe = _rope_table(pe, s)
    # linear1 in one launch over all halves (its weight rows are [q | k | v | mlp]): the qkv
    # columns get qk_norm + RoPE (row r rotated by pe row r % L) into s.qkv, the MLP columns
    # bias + GELU straight into the linear2 concat buffer.
    b2g.gemm_qkv_rope([dict(x=x_mod, w=w.linear1_w, bias=w.linear1_b, out=s.qkv[:B * L], pe=pe, pe_period=L,
                            q_norm=w.q_norm, k_norm=w.k_norm, gelu_out=s.cat[:B * L, HIDDEN:])], HEADS)
    mark("single.linear1")
    _attention(s.qkv, mask, B, L, s.cat[:, :HIDDEN])
    mark("single.attention")
    b2g.gemm(s.cat[:B * L], w.linear2_w, w.linear2_b, out=x, epilogue="gated_residual", gate=gate)
    mark("single.linear2")


def _no_mark(label: str) -> None:
    pass


# ---------------------------------------------------------------------------- transformer pass
DOUBLE_BLOCKS, SINGLE_BLOCKS = 19, 38  # Chroma's layout (chroma.cuh:1499-1584)


def single_mods(mods: torch.Tensor, i: int) -> torch.Tensor:
    """Rows (shift, scale, gate) of single block i in the approximator's output: 3i
    (chroma.cuh:980-984)."""
    return mods[3 * i:3 * i + 3]


def double_mods(mods: torch.Tensor, i: int, n_double: int, n_single: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Rows (shift1, scale1, gate1, shift2, scale2, gate2) of double block i, txt then img, in the
    approximator's output: img at 6i + 3*n_single, txt at 6i + 6*n_double + 3*n_single
    (chroma.cuh:535-553)."""
    img = 6 * i + 3 * n_single
    txt = 6 * i + 6 * n_double + 3 * n_single
    return mods[txt:txt + 6], mods[img:img + 6]


@dataclass
class PassWeights:
    """Weights of every block of one transformer pass, and the modulation vectors the
    approximator produces for it, in its own row order (single_mods, double_mods): per double
    block and stream 6 rows (shift1, scale1, gate1, shift2, scale2, gate2), per single block 3
    (shift, scale, gate)."""
    double: list          # [(txt StreamWeights, img StreamWeights)]
    single: list          # [SingleWeights]
    mods: torch.Tensor    # [SINGLE_BLOCKS * 3 + DOUBLE_BLOCKS * 12 (+ unused rows), 3072] F32


def random_pass(gen: torch.Generator, dev, n_double: int = DOUBLE_BLOCKS, n_single: int = SINGLE_BLOCKS) -> PassWeights:
    """Random-init weights of a whole pass (about 17 GB of bf16 for Chroma's 19 + 38 blocks)."""
    double = [(random_stream(gen, dev), random_stream(gen, dev)) for _ in range(n_double)]
    single = [random_single(gen, dev) for _ in range(n_single)]
    return PassWeights(double, single, mods=torch.zeros((n_single * 3 + n_double * 12, HIDDEN), device=dev))


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
    reference's blocks do (a double block's txt and img rows of all halves in one launch,
    modulate_streams).  x is updated in place; txt and img are row views of it, so the
    double-to-single concatenation costs nothing.  mask: one [L] key bias for every half, or
    one per half ([B, L] or a list)."""
    L = pe.shape[0]
    B = x.shape[0] // L
    assert B * L == x.shape[0] and 0 < T < L, "x must hold whole guidance halves of pe.shape[0] rows"
    txts = [x[b * L:b * L + T] for b in range(B)]
    imgs = [x[b * L + T:(b + 1) * L] for b in range(B)]
    mod_t = [s.mod[b * L:b * L + T] for b in range(B)]
    mod_i = [s.mod[b * L + T:(b + 1) * L] for b in range(B)]
    nd, ns = len(pw.double), len(pw.single)
    for i, (tw, iw) in enumerate(pw.double):
        mt, mi = double_mods(pw.mods, i, nd, ns)
        # both streams of every half in one launch (each row as modulate_to_bf16 writes it)
        b2g.modulate_streams(x, mt[0], mt[1], mi[0], mi[1], L, T, out=s.mod[:B * L])
        double_block_attention(tw, iw, mod_t, mod_i, txts, imgs, mt[2], mi[2], pe, mask, s)
        b2g.modulate_streams(x, mt[3], mt[4], mi[3], mi[4], L, T, out=s.mod[:B * L])
        double_block_mlp(tw, iw, mod_t, mod_i, txts, imgs, mt[5], mi[5], s)
    for i, sw in enumerate(pw.single):
        m = single_mods(pw.mods, i)
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


# ---------------------------------------------------------------------------- FP8 variant
# BASELINE config 5's transformer: every linear on E4M3 weights with one fp32 scale per output
# channel (absmax / 448, made once at load) and E4M3 activations with one scale per token.
# The reference's quantised path is INT8 (linear_prequant / quantize_act, kernels.cu:1988-2125,
# 2504-2644) and has no FP8 form; the producers here follow its structure: the modulation
# writes the quantised A operand of qkv / mlp0 / linear1 directly (modulate_to_e4m3), and the
# bf16 attention output, MLP hidden state and single-block concat buffer are quantised per
# token before proj / mlp2 / linear2 (one launch each).  Epilogues are those of the bf16 path.


@dataclass
class QLinear:
    """E4M3 weight codes [N, K] (uint8) with one fp32 scale per output channel [N]."""
    q: torch.Tensor
    s: torch.Tensor


@dataclass
class Q8:
    """Per-token E4M3 activations: codes [M, K] (uint8) and one fp32 scale per row [M]."""
    q: torch.Tensor
    s: torch.Tensor

    def rows(self, a: int, b: int) -> "Q8":
        return Q8(self.q[a:b], self.s[a:b])


@dataclass
class StreamWeightsFP8:
    qkv: QLinear
    qkv_b: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    proj: QLinear
    proj_b: torch.Tensor
    mlp0: QLinear
    mlp0_b: torch.Tensor
    mlp2: QLinear
    mlp2_b: torch.Tensor


@dataclass
class SingleWeightsFP8:
    linear1: QLinear
    linear1_b: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    linear2: QLinear
    linear2_b: torch.Tensor


def quantize_weight(w: torch.Tensor) -> QLinear:
    """The load-time FP8 transform of one linear's weight (per output channel)."""
    return QLinear(*b2g.quantize_e4m3(w))


def quantize_stream(w: StreamWeights) -> StreamWeightsFP8:
    return StreamWeightsFP8(quantize_weight(w.qkv_w), w.qkv_b, w.q_norm, w.k_norm, quantize_weight(w.proj_w),
                            w.proj_b, quantize_weight(w.mlp0_w), w.mlp0_b, quantize_weight(w.mlp2_w), w.mlp2_b)


def quantize_single(w: SingleWeights) -> SingleWeightsFP8:
    return SingleWeightsFP8(quantize_weight(w.linear1_w), w.linear1_b, w.q_norm, w.k_norm,
                            quantize_weight(w.linear2_w), w.linear2_b)


def _q8(rows: int, cols: int, dev) -> Q8:
    return Q8(torch.empty((rows, cols), dtype=torch.uint8, device=dev), torch.empty(rows, device=dev))


class ScratchFP8(Scratch):
    """The bf16 scratch plus the E4M3 forms of the quantised activations."""

    def __init__(self, T: int, I: int, dev, halves: int = 1):
        super().__init__(T, I, dev, halves)
        R = halves * (T + I)
        self.mod8 = _q8(R, HIDDEN, dev)          # modulated block inputs
        self.attn8 = _q8(R, HIDDEN, dev)         # double-block attention output (proj input)
        self.h8 = _q8(R, MLP, dev)               # GELU'd MLP hidden state (mlp2 input)
        self.cat8 = _q8(R, HIDDEN + MLP, dev)    # single-block [attn | mlp] (linear2 input)


def double_block_attention_fp8(txt_w: StreamWeightsFP8, img_w: StreamWeightsFP8, txt_mod1, img_mod1, txt, img,
                               txt_gate1, img_gate1, pe, mask, s: ScratchFP8, mark=None) -> None:
    """double_block_attention on E4M3 weights: txt_mod1 / img_mod1 are Q8 (or lists of Q8, one
    per guidance half) from modulate_to_e4m3; the rest as in double_block_attention."""
    mark = mark or _no_mark
    txt_m, img_m, txts, imgs = _halves(txt_mod1), _halves(img_mod1), _halves(txt), _halves(img)
    B, T = len(txts), txts[0].shape[0]
    L = T + imgs[0].shape[0]
    pe = _rope_table(pe, s)
    b2g.gemm_qkv_rope([dict(x=txt_m[b].q, x_scale=txt_m[b].s, w=txt_w.qkv.q, w_scale=txt_w.qkv.s, bias=txt_w.qkv_b,
                            out=s.qkv[b * L:b * L + T], pe=pe[:T], q_norm=txt_w.q_norm, k_norm=txt_w.k_norm)
                       for b in range(B)] +
                      [dict(x=img_m[b].q, x_scale=img_m[b].s, w=img_w.qkv.q, w_scale=img_w.qkv.s, bias=img_w.qkv_b,
                            out=s.qkv[b * L + T:(b + 1) * L], pe=pe[T:L], q_norm=img_w.q_norm,
                            k_norm=img_w.k_norm) for b in range(B)], HEADS)
    mark("double.qkv")
    _attention(s.qkv, mask, B, L, s.attn)
    mark("double.attention")
    b2g.quantize_e4m3(s.attn[:B * L], out=s.attn8.q[:B * L], scales=s.attn8.s[:B * L])
    mark("double.quantize_attn")
    a8 = s.attn8
    b2g.gemm_fp8_group([dict(x=a8.q[b * L:b * L + T], x_scale=a8.s[b * L:b * L + T], w=txt_w.proj.q,
                             w_scale=txt_w.proj.s, bias=txt_w.proj_b, out=txts[b], epilogue="gated_residual",
                             gate=txt_gate1) for b in range(B)] +
                       [dict(x=a8.q[b * L + T:(b + 1) * L], x_scale=a8.s[b * L + T:(b + 1) * L], w=img_w.proj.q,
                             w_scale=img_w.proj.s, bias=img_w.proj_b, out=imgs[b], epilogue="gated_residual",
                             gate=img_gate1) for b in range(B)])
    mark("double.proj")


def double_block_mlp_fp8(txt_w: StreamWeightsFP8, img_w: StreamWeightsFP8, txt_mod2, img_mod2, txt, img,
                         txt_gate2, img_gate2, s: ScratchFP8, mark=None) -> None:
    """double_block_mlp on E4M3 weights (modulated inputs as Q8, one per half or a list)."""
    mark = mark or _no_mark
    txt_m, img_m, txts, imgs = _halves(txt_mod2), _halves(img_mod2), _halves(txt), _halves(img)
    B, T, I = len(txts), txts[0].shape[0], imgs[0].shape[0]
    # h rows: every half's txt rows, then every half's img rows (one quantisation launch)
    ht = [(b * T, (b + 1) * T) for b in range(B)]
    hi = [(B * T + b * I, B * T + (b + 1) * I) for b in range(B)]
    b2g.gemm_fp8_group([dict(x=txt_m[b].q, x_scale=txt_m[b].s, w=txt_w.mlp0.q, w_scale=txt_w.mlp0.s,
                             bias=txt_w.mlp0_b, out=s.h[r0:r1], epilogue="gelu") for b, (r0, r1) in enumerate(ht)] +
                       [dict(x=img_m[b].q, x_scale=img_m[b].s, w=img_w.mlp0.q, w_scale=img_w.mlp0.s,
                             bias=img_w.mlp0_b, out=s.h[r0:r1], epilogue="gelu") for b, (r0, r1) in enumerate(hi)])
    mark("double.mlp0")
    R = B * (T + I)
    b2g.quantize_e4m3(s.h[:R], out=s.h8.q[:R], scales=s.h8.s[:R])
    mark("double.quantize_h")
    h8 = s.h8
    b2g.gemm_fp8_group([dict(x=h8.q[r0:r1], x_scale=h8.s[r0:r1], w=txt_w.mlp2.q, w_scale=txt_w.mlp2.s,
                             bias=txt_w.mlp2_b, out=txts[b], epilogue="gated_residual", gate=txt_gate2)
                        for b, (r0, r1) in enumerate(ht)] +
                       [dict(x=h8.q[r0:r1], x_scale=h8.s[r0:r1], w=img_w.mlp2.q, w_scale=img_w.mlp2.s,
                             bias=img_w.mlp2_b, out=imgs[b], epilogue="gated_residual", gate=img_gate2)
                        for b, (r0, r1) in enumerate(hi)])
    mark("double.mlp2")


def single_block_fp8(w: SingleWeightsFP8, x_mod: Q8, x, gate, pe, mask, s: ScratchFP8, mark=None) -> None:
    """single_block on E4M3 weights; x_mod is the Q8 of all B*L rows (modulate_to_e4m3)."""
    mark = mark or _no_mark
    L = pe.shape[0]
    B = x.shape[0] // L
    assert B * L == x.shape[0], "x must hold whole guidance halves of pe.shape[0] rows"
    pe = _rope_table(pe, s)
    R = B * L
    b2g.gemm_qkv_rope([dict(x=x_mod.q, x_scale=x_mod.s, w=w.linear1.q, w_scale=w.linear1.s, bias=w.linear1_b,
                            out=s.qkv[:R], pe=pe, pe_period=L, q_norm=w.q_norm, k_norm=w.k_norm,
                            gelu_out=s.cat[:R, HIDDEN:])], HEADS)
    mark("single.linear1")
    _attention(s.qkv, mask, B, L, s.cat[:, :HIDDEN])
    mark("single.attention")
    b2g.quantize_e4m3(s.cat[:R], out=s.cat8.q[:R], scales=s.cat8.s[:R])
    mark("single.quantize_cat")
    b2g.gemm_fp8_group([dict(x=s.cat8.q[:R], x_scale=s.cat8.s[:R], w=w.linear2.q, w_scale=w.linear2.s,
                             bias=w.linear2_b, out=x, epilogue="gated_residual", gate=gate)])
    mark("single.linear2")


def block_pair_ops_fp8(T: int, I: int) -> list[tuple[str, str, float]]:
    """block_pair_ops with the FP8 path's per-token quantisations (kind "quantize", 0 FLOPs)."""
    out = []
    for lab, kind, f in block_pair_ops(T, I):
        out.append((lab, kind, f))
        if lab == "double.attention":
            out.append(("double.quantize_attn", "quantize", 0.0))
        elif lab == "double.mlp0":
            out.append(("double.quantize_h", "quantize", 0.0))
        elif lab == "single.attention":
            out.append(("single.quantize_cat", "quantize", 0.0))
    return out


@dataclass
class PassWeightsFP8:
    """PassWeights with every linear in E4M3 (quantize_pass)."""
    double: list          # [(txt StreamWeightsFP8, img StreamWeightsFP8)]
    single: list          # [SingleWeightsFP8]
    mods: torch.Tensor


def quantize_pass(pw: PassWeights) -> PassWeightsFP8:
    """The load-time FP8 transform of a whole pass (8.6 GB of codes for Chroma's 57 blocks)."""
    return PassWeightsFP8([(quantize_stream(t), quantize_stream(i)) for t, i in pw.double],
                          [quantize_single(w) for w in pw.single], pw.mods)


def forward_pass_fp8(pw: PassWeightsFP8, x, pe, mask, s: ScratchFP8, T: int) -> None:
    """forward_pass on E4M3 weights: every block's modulation writes the E4M3 A operand with
    per-token scales (modulate_to_e4m3); layout, guidance halves and masks as forward_pass."""
    L = pe.shape[0]
    B = x.shape[0] // L
    assert B * L == x.shape[0] and 0 < T < L, "x must hold whole guidance halves of pe.shape[0] rows"
    txts = [x[b * L:b * L + T] for b in range(B)]
    imgs = [x[b * L + T:(b + 1) * L] for b in range(B)]
    mod_t = [s.mod8.rows(b * L, b * L + T) for b in range(B)]
    mod_i = [s.mod8.rows(b * L + T, (b + 1) * L) for b in range(B)]

    def modulate(src, shift, scale, dst: Q8):
        b2g.modulate_to_e4m3(src, shift, scale, out=dst.q, scales=dst.s)

    x8 = s.mod8.rows(0, B * L)
    nd, ns = len(pw.double), len(pw.single)
    for i, (tw, iw) in enumerate(pw.double):
        mt, mi = double_mods(pw.mods, i, nd, ns)
        b2g.modulate_streams(x, mt[0], mt[1], mi[0], mi[1], L, T, out=x8.q, scales=x8.s, fp8=True)
        double_block_attention_fp8(tw, iw, mod_t, mod_i, txts, imgs, mt[2], mi[2], pe, mask, s)
        b2g.modulate_streams(x, mt[3], mt[4], mi[3], mi[4], L, T, out=x8.q, scales=x8.s, fp8=True)
        double_block_mlp_fp8(tw, iw, mod_t, mod_i, txts, imgs, mt[5], mi[5], s)
    for i, sw in enumerate(pw.single):
        m = single_mods(pw.mods, i)
        modulate(x, m[0], m[1], x8)
        single_block_fp8(sw, x8, x, m[2], pe, mask, s)
