"""The whole Chroma Radiance denoising step on the engine: ChromaRadiance.forward_cfg mirrors the
reference's ChromaRadiance::forward_cfg (chroma.cuh:1499-1584) with the same weights (by the
checkpoint names its load() reads, chroma.cuh:375-462) and the same inputs:

  1. img_in (conv2d_img_in, chroma.cuh:1311-1327): im2col + bf16 cast in one kernel, then one
     GEMM launch writing both guidance halves' image rows.
  2. txt_in (chroma.cuh:1526-1527): both contexts cast to bf16, one grouped GEMM launch.
  3. compute_modulation (chroma.cuh:467-505, ChromaApproximator::forward :188-212): the
     timestep vector, then 12 skinny (M = 344) GEMMs; RMSNorm writes the next GEMM's bf16
     operand, SiLU is the in_layer's epilogue and the residual add the out_layer's (a gated
     residual with a gate of ones).
  4. 19 double + 38 single blocks (blocks.forward_pass), both halves in one half-major stream.
  5. nerf_decode for both halves at once (chroma.cuh:1163-1306): the embedder input in one
     kernel, then per GLU block one param_generator GEMM over both halves' patches and one
     fused tcgen05 kernel (b2g.nerf_glu_block) for the weight preparation, RMSNorm, the three
     TF32 products, SiLU * mul and the residual add, intermediates kept on chip.
  6. the final norm + 3x3 conv of both halves and cfg_blend (chroma.cuh:1225-1250, 1581).

Everything runs on the current stream and allocates nothing after ForwardScratch is made, so a
whole step can be captured in one CUDA graph; the timestep is read from device memory.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

import b2g
import blocks

HIDDEN, MLP, DHEAD = blocks.HIDDEN, blocks.MLP, blocks.DHEAD
PATCH = 16
TXT_TOKENS, CTX_DIM = 512, 4096
MOD_ROWS, APPROX_DIM, APPROX_LAYERS = 344, 5120, 5
NERF_HID, NERF_MLP, NERF_DEPTH, NERF_FEAT = 64, 256, 4, 67
NERF_PARAMS = 3 * NERF_HID * NERF_MLP
EMB_K = 72                 # the NeRF embedder's K = 67 padded to 16-byte bf16 rows


def weight_specs() -> dict[str, tuple[tuple[int, ...], torch.dtype]]:
    """Every tensor ChromaRadiance::load reads (chroma.cuh:375-462): name -> (shape, dtype).
    Linear weights are bf16 (load_weight keeps the file's dtype), biases, norm scales and the
    final conv F32 (load_tensor(..., F32))."""
    bf, f = torch.bfloat16, torch.float32
    s = {"img_in_patch.weight": ((HIDDEN, 3, PATCH, PATCH), bf), "img_in_patch.bias": ((HIDDEN,), f),
         "txt_in.weight": ((HIDDEN, CTX_DIM), bf), "txt_in.bias": ((HIDDEN,), f),
         "nerf_image_embedder.embedder.0.weight": ((NERF_HID, NERF_FEAT), bf),
         "nerf_image_embedder.embedder.0.bias": ((NERF_HID,), f),
         "nerf_final_layer_conv.norm.scale": ((NERF_HID,), f),
         "nerf_final_layer_conv.conv.weight": ((3, NERF_HID, 3, 3), f),
         "nerf_final_layer_conv.conv.bias": ((3,), f)}
    ap = "distilled_guidance_layer."
    s.update({ap + "in_proj.weight": ((APPROX_DIM, 64), bf), ap + "in_proj.bias": ((APPROX_DIM,), f),
              ap + "out_proj.weight": ((HIDDEN, APPROX_DIM), bf), ap + "out_proj.bias": ((HIDDEN,), f)})
    for i in range(APPROX_LAYERS):
        lp = f"{ap}layers.{i}."
        s.update({f"{ap}norms.{i}.scale": ((APPROX_DIM,), f),
                  lp + "in_layer.weight": ((APPROX_DIM, APPROX_DIM), bf), lp + "in_layer.bias": ((APPROX_DIM,), f),
                  lp + "out_layer.weight": ((APPROX_DIM, APPROX_DIM), bf), lp + "out_layer.bias": ((APPROX_DIM,), f)})
    for i in range(blocks.DOUBLE_BLOCKS):
        for st in ("img", "txt"):
            p = f"double_blocks.{i}.{st}"
            s.update({p + "_attn.qkv.weight": ((3 * HIDDEN, HIDDEN), bf), p + "_attn.qkv.bias": ((3 * HIDDEN,), f),
                      p + "_attn.norm.query_norm.scale": ((DHEAD,), f),
                      p + "_attn.norm.key_norm.scale": ((DHEAD,), f),
                      p + "_attn.proj.weight": ((HIDDEN, HIDDEN), bf), p + "_attn.proj.bias": ((HIDDEN,), f),
                      p + "_mlp.0.weight": ((MLP, HIDDEN), bf), p + "_mlp.0.bias": ((MLP,), f),
                      p + "_mlp.2.weight": ((HIDDEN, MLP), bf), p + "_mlp.2.bias": ((HIDDEN,), f)})
    for i in range(blocks.SINGLE_BLOCKS):
        p = f"single_blocks.{i}."
        s.update({p + "linear1.weight": ((3 * HIDDEN + MLP, HIDDEN), bf), p + "linear1.bias": ((3 * HIDDEN + MLP,), f),
                  p + "linear2.weight": ((HIDDEN, HIDDEN + MLP), bf), p + "linear2.bias": ((HIDDEN,), f),
                  p + "norm.query_norm.scale": ((DHEAD,), f), p + "norm.key_norm.scale": ((DHEAD,), f)})
    for i in range(NERF_DEPTH):
        p = f"nerf_blocks.{i}."
        s.update({p + "param_generator.weight": ((NERF_PARAMS, HIDDEN), bf),
                  p + "param_generator.bias": ((NERF_PARAMS,), f), p + "norm.scale": ((NERF_HID,), f)})
    return s


def random_weights(gen: torch.Generator, dev) -> dict[str, torch.Tensor]:
    """Seeded random init (about 19.6 GB): linear weights and the final conv ~ N(0, 0.02), biases
    ~ N(0, 0.02), RMSNorm scales ~ 1 + N(0, 0.1)."""
    out = {}
    for name, (shape, dt) in weight_specs().items():
        t = torch.randn(shape, generator=gen, device=dev)
        if name.endswith("scale"):
            t.mul_(0.1).add_(1.0)
        else:
            t.mul_(0.02)
        out[name] = t.to(dt)
    return out


def rope_table(H: int, W: int, txt_tokens: int = TXT_TOKENS, theta: int = 10000,
               axes: tuple[int, ...] = (16, 56, 56)) -> np.ndarray:
    """RoPE::gen_pe (rope.cuh:84-124): [txt_tokens + (H/16)(W/16), 64 * 4] rows (cos, -sin,
    sin, cos) of the 3-axis (index, row, col) positions, text tokens all at 0."""
    hp, wp = (H + PATCH // 2) // PATCH, (W + PATCH // 2) // PATCH
    ids = np.zeros((txt_tokens + hp * wp, 3), dtype=np.float32)
    ids[txt_tokens:, 1] = np.repeat(np.arange(hp, dtype=np.float32), wp)
    ids[txt_tokens:, 2] = np.tile(np.arange(wp, dtype=np.float32), hp)
    cols = []
    for a, dim in enumerate(axes):
        half = dim // 2
        end = np.float32((np.float32(dim) - np.float32(2)) / np.float32(dim))  # linspace(0, (dim-2)/dim, half)
        scale = np.array([end * np.float32(i) / np.float32(half - 1) for i in range(half)], dtype=np.float32)
        omega = (np.float32(1) / np.power(np.float32(theta), scale)).astype(np.float32)
        ang = (ids[:, a:a + 1] * omega[None, :]).astype(np.float32)
        c, s = np.cos(ang), np.sin(ang)
        cols.append(np.stack([c, -s, s, c], -1).reshape(ids.shape[0], half * 4))
    return np.concatenate(cols, 1).astype(np.float32)


def dct_features(patch: int = PATCH, freqs: int = 8) -> np.ndarray:
    """compute_dct_features (main.cu:22-65): [patch^2, freqs^2] cos(px fx pi) cos(py fy pi) /
    (1 + fx fy), positions i / (patch - 1)."""
    pos = np.arange(patch, dtype=np.float32) / np.float32(patch - 1)
    px, py = np.tile(pos, patch), np.repeat(pos, patch)
    f = np.arange(freqs, dtype=np.float32)
    cx = np.cos(px[:, None] * f[None, :] * np.float32(np.pi))
    cy = np.cos(py[:, None] * f[None, :] * np.float32(np.pi))
    coef = 1.0 / (1.0 + f[:, None] * f[None, :])
    return (cx[:, :, None] * cy[:, None, :] * coef[None]).reshape(patch * patch, freqs * freqs).astype(np.float32)


def key_masks(real_tokens: list[int], H: int, W: int, txt_tokens: int = TXT_TOKENS) -> np.ndarray:
    """One key bias row per guidance half (main.cu:413-430): text tokens past real + 1 are -inf."""
    L = txt_tokens + (H // PATCH) * (W // PATCH)
    m = np.zeros((len(real_tokens), L), dtype=np.float32)
    for b, r in enumerate(real_tokens):
        m[b, min(r + 1, txt_tokens):txt_tokens] = -np.inf
    return m


@dataclass
class ApproxLayer:
    norm: torch.Tensor
    in_w: torch.Tensor
    in_b: torch.Tensor
    out_w: torch.Tensor
    out_b: torch.Tensor


@dataclass
class NerfBlock:
    param_w: torch.Tensor   # [49152, 3072] bf16
    param_b: torch.Tensor
    norm: torch.Tensor      # [64]


class ForwardScratch:
    """Every buffer of one forward_cfg at H x W with both guidance halves, allocated once."""

    def __init__(self, H: int, W: int, dev, txt_tokens: int = TXT_TOKENS):
        T = txt_tokens
        P = (H // PATCH) * (W // PATCH)
        L = T + P
        self.H, self.W, self.T, self.P, self.L = H, W, T, P, L
        f, bf = torch.float32, torch.bfloat16
        self.timestep = torch.zeros(1, dtype=f, device=dev)
        self.x = torch.empty((2 * L, HIDDEN), dtype=f, device=dev)          # half-major residual stream
        self.patches = torch.empty((P, 3 * PATCH * PATCH), dtype=bf, device=dev)
        self.ctx = torch.empty((2, T, CTX_DIM), dtype=bf, device=dev)
        self.vec = torch.empty((MOD_ROWS, 64), dtype=f, device=dev)
        self.ax = torch.empty((MOD_ROWS, APPROX_DIM), dtype=f, device=dev)
        self.an = torch.empty((MOD_ROWS, APPROX_DIM), dtype=bf, device=dev)
        self.ah = torch.empty((MOD_ROWS, APPROX_DIM), dtype=bf, device=dev)
        self.mod = torch.empty((MOD_ROWS, HIDDEN), dtype=f, device=dev)
        self.blocks = blocks.PassScratch(T, P, dev, halves=2)
        self.img16 = torch.empty((2 * P, HIDDEN), dtype=bf, device=dev)    # both halves' image rows
        self.emb_in = torch.empty((P * 256, EMB_K), dtype=bf, device=dev)
        self.nx = torch.empty((2, P * 256, NERF_HID), dtype=f, device=dev)  # decoder state per half
        self.params = torch.empty((2 * P, NERF_PARAMS), dtype=f, device=dev)
        self.velocity = torch.empty((1, 3, H, W), dtype=f, device=dev)


class ChromaRadiance:
    """The reference's ChromaRadiance (chroma.cuh:340-1584) on the engine's kernels.

    `weights`: name -> device tensor in weight_specs()'s shapes and dtypes (any contiguous
    shape with that many elements is accepted, e.g. the flat buffers of another
    implementation); the model keeps views, not copies, except for two load-time transforms:
    the NeRF embedder's weight padded to EMB_K columns and a gate vector of ones."""

    def __init__(self, weights: dict[str, torch.Tensor], dev):
        specs = weight_specs()

        def g(name):
            return weights[name].view(specs[name][0])

        self.dev = dev
        self.img_in_w = g("img_in_patch.weight").view(HIDDEN, 3 * PATCH * PATCH)
        self.img_in_b = g("img_in_patch.bias")
        self.txt_in_w, self.txt_in_b = g("txt_in.weight"), g("txt_in.bias")
        emb = g("nerf_image_embedder.embedder.0.weight")
        self.emb_w = torch.zeros((NERF_HID, EMB_K), dtype=torch.bfloat16, device=dev)
        self.emb_w[:, :NERF_FEAT] = emb
        self.emb_b = g("nerf_image_embedder.embedder.0.bias")
        self.final_norm = g("nerf_final_layer_conv.norm.scale")
        self.conv_w, self.conv_b = g("nerf_final_layer_conv.conv.weight"), g("nerf_final_layer_conv.conv.bias")
        ap = "distilled_guidance_layer."
        self.in_proj_w, self.in_proj_b = g(ap + "in_proj.weight"), g(ap + "in_proj.bias")
        self.out_proj_w, self.out_proj_b = g(ap + "out_proj.weight"), g(ap + "out_proj.bias")
        self.approx = [ApproxLayer(g(f"{ap}norms.{i}.scale"), g(f"{ap}layers.{i}.in_layer.weight"),
                                   g(f"{ap}layers.{i}.in_layer.bias"), g(f"{ap}layers.{i}.out_layer.weight"),
                                   g(f"{ap}layers.{i}.out_layer.bias")) for i in range(APPROX_LAYERS)]
        self.ones = torch.ones(APPROX_DIM, device=dev)

        def stream(p):
            return blocks.StreamWeights(g(p + "_attn.qkv.weight"), g(p + "_attn.qkv.bias"),
                                        g(p + "_attn.norm.query_norm.scale"), g(p + "_attn.norm.key_norm.scale"),
                                        g(p + "_attn.proj.weight"), g(p + "_attn.proj.bias"), g(p + "_mlp.0.weight"),
                                        g(p + "_mlp.0.bias"), g(p + "_mlp.2.weight"), g(p + "_mlp.2.bias"))

        double = [(stream(f"double_blocks.{i}.txt"), stream(f"double_blocks.{i}.img"))
                  for i in range(blocks.DOUBLE_BLOCKS)]
        single = [blocks.SingleWeights(g(f"single_blocks.{i}.linear1.weight"), g(f"single_blocks.{i}.linear1.bias"),
                                       g(f"single_blocks.{i}.norm.query_norm.scale"),
                                       g(f"single_blocks.{i}.norm.key_norm.scale"),
                                       g(f"single_blocks.{i}.linear2.weight"), g(f"single_blocks.{i}.linear2.bias"))
                  for i in range(blocks.SINGLE_BLOCKS)]
        self.blocks = blocks.PassWeights(double, single, mods=None)
        self.nerf = [NerfBlock(g(f"nerf_blocks.{i}.param_generator.weight"), g(f"nerf_blocks.{i}.param_generator.bias"),
                               g(f"nerf_blocks.{i}.norm.scale")) for i in range(NERF_DEPTH)]

    # ------------------------------------------------------------------ pieces of the step
    def compute_modulation(self, s: ForwardScratch, mark=None) -> torch.Tensor:
        """ChromaApproximator on the timestep in s.timestep (guidance 0, as forward_cfg calls it)
        into s.mod [344, 3072].  `mark(label)`, when given, is called after each GEMM (with the
        RMSNorm and timestep embedding before it counted in)."""
        mk = mark or (lambda label: None)
        b2g.timestep_vec(s.timestep, 0.0, s.vec)
        b2g.gemm(s.vec, self.in_proj_w, self.in_proj_b, out=s.ax)
        mk("in_proj")
        for i, layer in enumerate(self.approx):
            b2g.rms_norm(s.ax, layer.norm, s.an)
            b2g.gemm(s.an, layer.in_w, layer.in_b, out=s.ah, epilogue="silu")
            mk(f"layer{i}.in")
            b2g.gemm(s.ah, layer.out_w, layer.out_b, out=s.ax, epilogue="gated_residual", gate=self.ones)
            mk(f"layer{i}.out")
        b2g.gemm(s.ax, self.out_proj_w, self.out_proj_b, out=s.mod)
        mk("out_proj")
        return s.mod

    def embed(self, s: ForwardScratch, x_img: torch.Tensor, ctx_cond: torch.Tensor, ctx_uncond: torch.Tensor) -> None:
        """img_in and txt_in into the half-major stream s.x: half b's text rows [bL, bL + T),
        its image rows after them (both halves start from the same image tokens)."""
        T, L = s.T, s.L
        b2g.patchify_bf16(x_img, PATCH, s.patches)
        b2g.gemm_group([dict(x=s.patches, w=self.img_in_w, bias=self.img_in_b, out=s.x[b * L + T:(b + 1) * L])
                        for b in range(2)])
        b2g.convert_f32(ctx_cond, s.ctx[0])
        b2g.convert_f32(ctx_uncond, s.ctx[1])
        b2g.gemm_group([dict(x=s.ctx[b], w=self.txt_in_w, bias=self.txt_in_b, out=s.x[b * L:b * L + T])
                        for b in range(2)])

    def nerf_decode(self, s: ForwardScratch, x_img: torch.Tensor, dct: torch.Tensor) -> None:
        """nerf_decode of both halves' transformer image rows (chroma.cuh:1163-1306) into the
        decoder state s.nx [2, P*256, 64]."""
        T, L, P = s.T, s.L, s.P
        b2g.nerf_input_bf16(x_img, dct, s.emb_in)
        b2g.gemm_group([dict(x=s.emb_in, w=self.emb_w, bias=self.emb_b, out=s.nx[b]) for b in range(2)])
        for b in range(2):
            b2g.convert_f32(s.x[b * L + T:(b + 1) * L], s.img16[b * P:(b + 1) * P])
        for blk in self.nerf:
            b2g.gemm(s.img16, blk.param_w, blk.param_b, out=s.params)
            b2g.nerf_glu_block(s.params, blk.norm, s.nx)

    def forward_cfg(self, s: ForwardScratch, x_img: torch.Tensor, ctx_cond: torch.Tensor, ctx_uncond: torch.Tensor,
                    pe: torch.Tensor, dct: torch.Tensor, masks: torch.Tensor, cfg_scale: float) -> torch.Tensor:
        """One denoising step's velocity [1, 3, H, W] (in s.velocity) at the timestep in
        s.timestep: x_img F32 [1, 3, H, W], ctx_* F32 [T, 4096] (the T5 outputs), pe F32 [L, 256]
        (rope_table), dct F32 [256, 64], masks F32 [2, L] (conditional, unconditional)."""
        self.embed(s, x_img, ctx_cond, ctx_uncond)
        self.blocks.mods = self.compute_modulation(s)
        blocks.forward_pass(self.blocks, s.x, pe, masks, s.blocks, s.T)
        self.nerf_decode(s, x_img, dct)
        b2g.nerf_final(s.nx[0], s.nx[1], self.final_norm, self.conv_w, self.conv_b, cfg_scale, s.H, s.W,
                       s.velocity.view(3, s.H, s.W))
        return s.velocity


def step_flops(H: int, W: int, txt_tokens: int = TXT_TOKENS) -> dict:
    """Algorithmic FLOPs of one forward_cfg (both guidance halves), by part."""
    P = (H // PATCH) * (W // PATCH)
    embed = 2.0 * P * HIDDEN * 3 * PATCH * PATCH + 2.0 * txt_tokens * HIDDEN * CTX_DIM * 2  # img_in once
    approx = 2.0 * MOD_ROWS * (APPROX_DIM * 64 + 2 * APPROX_LAYERS * APPROX_DIM * APPROX_DIM + HIDDEN * APPROX_DIM)
    blocks_f = blocks.pass_flops(txt_tokens, P, halves=2)
    nerf = 2 * (2.0 * P * 256 * NERF_HID * NERF_FEAT + NERF_DEPTH * (2.0 * P * NERF_PARAMS * HIDDEN +
                                                                      3 * 2.0 * P * 256 * NERF_MLP * NERF_HID))
    return {"embed": embed, "approximator": approx, "blocks": blocks_f, "nerf": nerf,
            "total": embed + approx + blocks_f + nerf}
