"""Classifier-free guidance layout of blocks.py on CPU (no GPU): the engine calls are replaced
by an fp32 torch stand-in with the same signatures, and a pass over two guidance halves
stacked half-major ([txt_c, img_c | txt_u, img_u], each half with its own key mask) must equal
the same pass run on each half alone.  This checks the row views, the per-half attention and
masks and the single block's RoPE row period that forward_cfg's block loop
(chroma.cuh:1540-1563) needs.  Tolerance: max|d|/max|x| <= 1e-5 (the stand-in is fp32 and
rounds the bf16 activations at the same points in both runs; matrix products over different
row counts may round differently in the last bits)."""
from __future__ import annotations

import pytest
import torch

import b2g as engine_b2g
import blocks


class FakeEngine:
    """fp32 CPU stand-in for the b2g calls blocks.py makes."""

    B2GError = engine_b2g.B2GError

    def __init__(self):
        self.calls = []

    def gemm(self, x, w, bias=None, out=None, epilogue="none", gate=None, out_dtype=None):
        self.calls.append(("gemm", 1))
        return self._gemm(x, w, bias, out, epilogue, gate)

    @staticmethod
    def _gemm(x, w, bias, out, epilogue, gate):
        y = x.float() @ w.float().t()
        if bias is not None:
            y = y + bias
        if epilogue == "gelu":
            y = 0.5 * y * (1 + torch.tanh(0.7978845608 * (y + 0.044715 * y ** 3)))
        if epilogue == "gated_residual":
            out += gate * y
        else:
            out.copy_(y.to(out.dtype))
        return out

    def gemm_group(self, problems):
        assert 1 <= len(problems) <= 4
        self.calls.append(("gemm_group", len(problems)))
        return [self._gemm(p["x"], p["w"], p.get("bias"), p.get("out"), p.get("epilogue", "none"), p.get("gate"))
                for p in problems]

    @staticmethod
    def _deq(t, sc):
        if t.dtype != torch.uint8:
            return t.float()
        return t.view(torch.float8_e4m3fn).float() * sc[:, None]

    def quantize_e4m3(self, x, out=None, scales=None):
        self.calls.append(("quantize", 1))
        xf = x.float()
        amax = xf.abs().amax(1)
        sc = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
        q = (xf / sc[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
        out = out if out is not None else torch.empty_like(q)
        scales = scales if scales is not None else torch.empty_like(sc)
        out.copy_(q)
        scales.copy_(sc)
        return out, scales

    def modulate_to_e4m3(self, x, shift, scale, out=None, scales=None, eps=1e-6):
        self.calls.append(("modulate", 1))
        xf = x.float()
        mu = xf.mean(-1, keepdim=True)
        var = ((xf - mu) ** 2).mean(-1, keepdim=True)
        calls = len(self.calls)
        r = self.quantize_e4m3((xf - mu) * torch.rsqrt(var + eps) * (1 + scale) + shift, out, scales)
        del self.calls[calls:]
        return r

    def gemm_fp8_group(self, problems):
        assert 1 <= len(problems) <= 4
        self.calls.append(("gemm_fp8_group", len(problems)))
        return [self._gemm(self._deq(p["x"], p["x_scale"]), self._deq(p["w"], p["w_scale"]), p.get("bias"),
                           p.get("out"), p.get("epilogue", "none"), p.get("gate")) for p in problems]

    def gemm_qkv_rope(self, problems, n_head, eps=1e-6):
        assert 1 <= len(problems) <= 4
        self.calls.append(("gemm_qkv_rope", len(problems)))
        for pr in problems:
            y = self._deq(pr["x"], pr.get("x_scale")) @ self._deq(pr["w"], pr.get("w_scale")).t() + pr["bias"]
            M = y.shape[0]
            qkv = 3 * n_head * blocks.DHEAD
            if pr.get("gelu_out") is not None:
                t = y[:, qkv:]
                pr["gelu_out"].copy_((0.5 * t * (1 + torch.tanh(0.7978845608 * (t + 0.044715 * t ** 3)))).to(
                    torch.bfloat16))
                y = y[:, :qkv]
            period = pr.get("pe_period") or M
            rows = torch.arange(M) % period
            pe = pr["pe"]
            if pe.dim() == 3 and pe.shape[-1] == 2:   # compact (cos, sin) form
                pe = torch.stack([pe[..., 0], -pe[..., 1], pe[..., 1], pe[..., 0]], -1)
            p = pe.reshape(-1, blocks.DHEAD // 2, 4)[rows].reshape(M, 1, blocks.DHEAD // 2, 4)
            q, k, v = y.reshape(M, 3, n_head, blocks.DHEAD).unbind(1)

            def norm_rope(a, scale):
                a = a * torch.rsqrt((a * a).mean(-1, keepdim=True) + eps) * scale
                e, o = a[..., 0::2], a[..., 1::2]
                return torch.stack([e * p[..., 0] + o * p[..., 1], e * p[..., 2] + o * p[..., 3]], -1).reshape(
                    M, n_head, blocks.DHEAD)

            out = torch.stack([norm_rope(q, pr["q_norm"]), norm_rope(k, pr["k_norm"]), v], 1).reshape(M, -1)
            pr["out"].copy_(out.to(torch.bfloat16))

    def attention_bf16(self, q, k, v, n_head, d_head, attn_mask=None, out=None):
        self.calls.append(("attention_bf16", 1))
        return self._attend(q, k, v, n_head, d_head, attn_mask, out)

    @staticmethod
    def _attend(q, k, v, n_head, d_head, attn_mask, out):
        L = q.shape[0]
        qq, kk, vv = (t.float().reshape(L, n_head, d_head) for t in (q, k, v))
        s = torch.einsum("lhd,mhd->hlm", qq, kk) / d_head ** 0.5
        if attn_mask is not None:
            s = s + attn_mask[None, None, :]
        o = torch.einsum("hlm,mhd->lhd", torch.softmax(s, -1), vv).reshape(L, n_head * d_head)
        out.copy_(o.to(out.dtype))
        return out

    compact_rope_table = staticmethod(engine_b2g.compact_rope_table)

    def attention_bf16_batched(self, q, k, v, n_head, d_head, batch, attn_mask=None, out=None):
        self.calls.append(("attention_bf16_batched", batch))
        L = q.shape[0] // batch
        for b in range(batch):
            r = slice(b * L, (b + 1) * L)
            m = None if attn_mask is None else (attn_mask[b] if attn_mask.dim() == 2 else attn_mask)
            self._attend(q[r], k[r], v[r], n_head, d_head, m, out[r])
        return out

    def modulate_streams(self, x, txt_shift, txt_scale, img_shift, img_scale, seq, txt_rows, out=None,
                         scales=None, fp8=False, eps=1e-6):
        self.calls.append(("modulate", 1))
        img = ((torch.arange(x.shape[0]) % seq) >= txt_rows)[:, None]
        shift = torch.where(img, img_shift, txt_shift)
        scale = torch.where(img, img_scale, txt_scale)
        xf = x.float()
        mu = xf.mean(-1, keepdim=True)
        var = ((xf - mu) ** 2).mean(-1, keepdim=True)
        y = (xf - mu) * torch.rsqrt(var + eps) * (1 + scale) + shift
        if fp8:
            calls = len(self.calls)
            r = self.quantize_e4m3(y, out, scales)
            del self.calls[calls:]
            return r
        out.copy_(y.to(torch.bfloat16))
        return out

    def modulate_to_bf16(self, x, shift, scale, out=None, eps=1e-6):
        self.calls.append(("modulate", 1))
        xf = x.float()
        mu = xf.mean(-1, keepdim=True)
        var = ((xf - mu) ** 2).mean(-1, keepdim=True)
        out.copy_(((xf - mu) * torch.rsqrt(var + eps) * (1 + scale) + shift).to(torch.bfloat16))
        return out


T, I = 8, 16
L = T + I


@pytest.fixture(scope="module")
def pass_inputs():
    g = torch.Generator().manual_seed(11)
    pw = blocks.random_pass(g, "cpu", n_double=1, n_single=1)
    pw.mods.copy_(torch.randn(tuple(pw.mods.shape), generator=g) * 0.1)
    ang = torch.rand((L, blocks.DHEAD // 2), generator=g) * 6.2831853
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    masks = torch.zeros((2, L))
    masks[0, T - 3:T] = float("-inf")
    masks[1, 1:T] = float("-inf")      # the unconditional half: an (almost) empty prompt
    x0 = torch.randn((2 * L, blocks.HIDDEN), generator=g)
    return pw, pe, masks, x0


def test_cfg_pass_equals_each_half_alone(pass_inputs, monkeypatch):
    pw, pe, masks, x0 = pass_inputs
    fake = FakeEngine()
    monkeypatch.setattr(blocks, "b2g", fake)
    x = x0.clone()
    blocks.forward_pass(pw, x, pe, masks, blocks.PassScratch(T, I, "cpu", halves=2), T)
    # one launch per double-block GEMM layer over the four row blocks, one linear1 over both
    # halves
    assert ("gemm_qkv_rope", 4) in fake.calls and ("gemm_group", 4) in fake.calls
    assert ("gemm_qkv_rope", 1) in fake.calls
    # both halves' attention in one launch per block (the masks are one [2, L] tensor)
    assert [c for c in fake.calls if c[0].startswith("attention")] == [("attention_bf16_batched", 2)] * 2
    for b in range(2):
        y = x0[b * L:(b + 1) * L].clone()
        blocks.forward_pass(pw, y, pe, masks[b], blocks.PassScratch(T, I, "cpu"), T)
        d = (x[b * L:(b + 1) * L] - y).abs().max() / y.abs().max()
        assert d <= 1e-5, f"half {b}: {d:.3e}"
    assert not torch.equal(x[:L], x[L:])
    assert torch.isfinite(x).all()


def test_single_block_rope_period_and_per_half_masks(pass_inputs, monkeypatch):
    """single_block on two stacked halves rotates each half's rows by pe rows 0..L-1 and masks
    each half with its own key bias."""
    pw, pe, masks, x0 = pass_inputs
    monkeypatch.setattr(blocks, "b2g", FakeEngine())
    sw = pw.single[0]
    g = torch.Generator().manual_seed(2)
    x_mod = torch.randn((2 * L, blocks.HIDDEN), generator=g).to(torch.bfloat16)
    gate = torch.randn(blocks.HIDDEN, generator=g)
    x = x0.clone()
    blocks.single_block(sw, x_mod, x, gate, pe, masks, blocks.Scratch(T, I, "cpu", halves=2))
    for b in range(2):
        y = x0[b * L:(b + 1) * L].clone()
        blocks.single_block(sw, x_mod[b * L:(b + 1) * L], y, gate, pe, masks[b], blocks.Scratch(T, I, "cpu"))
        assert (x[b * L:(b + 1) * L] - y).abs().max() / y.abs().max() <= 1e-5


def test_masks_per_half_are_checked():
    with pytest.raises(AssertionError):
        blocks._masks(torch.zeros((3, L)), 2)
    assert blocks._masks(None, 2) == [None, None]
    m = torch.zeros(L)
    assert all(t is m for t in blocks._masks(m, 2))


def test_cfg_flops_double():
    assert blocks.pass_flops(T, I, 1, 1, halves=2) == 2 * blocks.pass_flops(T, I, 1, 1)


def test_fp8_cfg_pass_equals_each_half_alone(pass_inputs, monkeypatch):
    """The FP8 pass (E4M3 weights, per-token E4M3 activations) over two stacked guidance
    halves equals each half alone, and launches the FP8 layers as the bf16 pass does."""
    pw, pe, masks, x0 = pass_inputs
    fake = FakeEngine()
    monkeypatch.setattr(blocks, "b2g", fake)
    pw8 = blocks.quantize_pass(pw)
    x = x0.clone()
    blocks.forward_pass_fp8(pw8, x, pe, masks, blocks.ScratchFP8(T, I, "cpu", halves=2), T)
    assert ("gemm_qkv_rope", 4) in fake.calls and ("gemm_fp8_group", 4) in fake.calls
    # the 10 weights (4 per stream, 2 single), then one attention output, one MLP hidden state
    # and one concat buffer per pass over both halves
    assert sum(1 for c in fake.calls if c[0] == "quantize") == 10 + 3
    for b in range(2):
        y = x0[b * L:(b + 1) * L].clone()
        blocks.forward_pass_fp8(pw8, y, pe, masks[b], blocks.ScratchFP8(T, I, "cpu"), T)
        d = (x[b * L:(b + 1) * L] - y).abs().max() / y.abs().max()
        assert d <= 1e-5, f"half {b}: {d:.3e}"
    # close to the bf16 pass (E4M3 rounding of weights and activations)
    z = x0.clone()
    blocks.forward_pass(pw, z, pe, masks, blocks.PassScratch(T, I, "cpu", halves=2), T)
    dz, dx = (z - x0).double(), (x - x0).double()
    assert (dz - dx).abs().max() / dz.abs().max() < 0.2
    assert float((dz * dx).sum() / (dz.norm() * dx.norm())) > 0.99


def test_per_half_mask_list_falls_back_to_one_launch_per_half(pass_inputs, monkeypatch):
    """Key biases given as a list (not one [B, L] tensor) run one attention launch per half,
    with the same result."""
    pw, pe, masks, x0 = pass_inputs
    fake = FakeEngine()
    monkeypatch.setattr(blocks, "b2g", fake)
    x, y = x0.clone(), x0.clone()
    blocks.forward_pass(pw, x, pe, masks, blocks.PassScratch(T, I, "cpu", halves=2), T)
    blocks.forward_pass(pw, y, pe, [masks[0], masks[1]], blocks.PassScratch(T, I, "cpu", halves=2), T)
    assert ("attention_bf16", 1) in fake.calls
    assert torch.allclose(x, y, rtol=0, atol=1e-5 * float(y.abs().max()))


def test_compact_rope_table():
    """compact_rope_table keeps (cos, sin) of a rotation-form table and refuses other tables."""
    ang = torch.rand((5, 64), generator=torch.Generator().manual_seed(4)) * 6.28
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    c = engine_b2g.compact_rope_table(pe)
    assert c.shape == (5, 64, 2) and c.is_contiguous()
    assert torch.equal(c[..., 0], ang.cos()) and torch.equal(c[..., 1], ang.sin())
    general = pe.clone()
    general[2, 7, 1] += 0.5
    assert engine_b2g.compact_rope_table(general) is None
