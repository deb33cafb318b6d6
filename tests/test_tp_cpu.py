"""Tensor-parallel block pair on CPU `gloo` ranks (no GPU): the sharding of tp.py (column
splits, K-split views, the packed linear2 slice, where the all-reduces and the bias/gate
step sit) must reproduce the unsharded computation.  The engine's kernels are replaced by an
fp32 torch stand-in with the same signatures and the same bf16 rounding points; world size 2
and 4 are compared against world size 1 of the same code (tolerance: max|d|/max|ref| of the
residual-stream update <= 1e-2, cosine >= 0.9999; the partials are rounded to bf16 before
the reduce, as on the GPUs)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import blocks
import tp

D = tp.Dims(hidden=256, heads=4, dhead=64, mlp=512)
T, I = 16, 24


class TorchOps:
    """fp32 CPU stand-in for tp.EngineOps (all-reduce over the gloo group when `reduce`)."""

    def __init__(self, reduce: bool):
        self.reduce = reduce

    def gemm_group(self, problems):
        return [self.gemm(**p) for p in problems]

    def gemm(self, x, w, bias=None, out=None, epilogue="none", gate=None, out_dtype=None):
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

    def qkv_rope(self, problems, n_head, eps=1e-6):
        for pr in problems:
            y = pr["x"].float() @ pr["w"].float().t() + pr["bias"]
            M = y.shape[0]
            dh = D.dhead
            if pr.get("gelu_out") is not None:   # linear1's MLP columns: bias + GELU
                t = y[:, 3 * n_head * dh:]
                pr["gelu_out"].copy_((0.5 * t * (1 + torch.tanh(0.7978845608 * (t + 0.044715 * t ** 3)))).to(
                    pr["gelu_out"].dtype))
                y = y[:, :3 * n_head * dh]
            q, k, v = y.reshape(M, 3, n_head, dh).unbind(1)
            pe = pr["pe"]
            if pe.shape[-1] == 2:                # compact (cos, sin) table
                c, sn = pe[..., 0], pe[..., 1]
                pe = torch.stack([c, -sn, sn, c], -1)
            p = pe.reshape(M, 1, dh // 2, 4)

            def norm_rope(x, scale):
                if scale is not None:
                    x = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * scale
                e, o = x[..., 0::2], x[..., 1::2]
                return torch.stack([e * p[..., 0] + o * p[..., 1], e * p[..., 2] + o * p[..., 3]], -1).reshape(
                    M, n_head, dh)

            y = torch.stack([norm_rope(q, pr["q_norm"]), norm_rope(k, pr["k_norm"]), v], 1).reshape(M, -1)
            pr["out"].copy_(y.to(pr["out"].dtype))

    def attention_bf16(self, q, k, v, n_head, d_head, attn_mask=None, out=None):
        L = q.shape[0]
        qq, kk, vv = (t.float().reshape(L, n_head, d_head) for t in (q, k, v))
        s = torch.einsum("lhd,mhd->hlm", qq, kk) / d_head ** 0.5
        if attn_mask is not None:
            s = s + attn_mask[None, None, :]
        o = torch.einsum("hlm,mhd->lhd", torch.softmax(s, -1), vv).reshape(L, n_head * d_head)
        out.copy_(o.to(out.dtype))
        return out

    def bias_gated_residual(self, y, bias, gate, residual):
        residual += gate * (y.float() + (bias if bias is not None else 0))

    def all_reduce(self, t):
        if self.reduce:
            f = t.float()
            dist.all_reduce(f)
            t.copy_(f.to(t.dtype))


def make_inputs():
    g = torch.Generator().manual_seed(3)

    def w(n, k):
        return (torch.randn((n, k), generator=g) * 0.05).to(torch.bfloat16)

    def b(n):
        return torch.randn(n, generator=g) * 0.05

    def nrm():
        return 1 + 0.1 * torch.randn(D.dhead, generator=g)

    H, M = D.hidden, D.mlp

    def stream():
        return blocks.StreamWeights(w(3 * H, H), b(3 * H), nrm(), nrm(), w(H, H), b(H), w(M, H), b(M), w(H, M), b(H))

    txt_w, img_w = stream(), stream()
    sw = blocks.SingleWeights(w(3 * H + M, H), b(3 * H + M), nrm(), nrm(), w(H, H + M), b(H))
    L = T + I
    act = {k: torch.randn((n, H), generator=g).to(torch.bfloat16) for k, n in
           (("txt_mod1", T), ("img_mod1", I), ("txt_mod2", T), ("img_mod2", I), ("x_mod", L))}
    res = {k: torch.randn((n, H), generator=g) for k, n in (("txt", T), ("img", I), ("x", L))}
    gates = [torch.randn(H, generator=g) for _ in range(5)]
    ang = torch.rand((L, D.dhead // 2), generator=g) * 6.28
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    mask = torch.zeros(L)
    mask[3:9] = float("-inf")
    return txt_w, img_w, sw, act, res, gates, pe, mask


def run_tp(rank, world):
    txt_w, img_w, sw, act, res, g, pe, mask = make_inputs()
    ops = TorchOps(reduce=world > 1)
    tw, iw = tp.shard_stream(txt_w, rank, world, D), tp.shard_stream(img_w, rank, world, D)
    s1 = tp.shard_single(sw, rank, world, D)
    scratch = tp.TPScratch(T, I, world, "cpu", D)
    out = {k: v.clone() for k, v in res.items()}
    tp.tp_double_block(ops, tw, iw, act["txt_mod1"], act["img_mod1"], act["txt_mod2"], act["img_mod2"], out["txt"],
                       out["img"], g[0], g[1], g[2], g[3], pe, mask, scratch)
    tp.tp_single_block(ops, s1, act["x_mod"], out["x"], g[4], pe, mask, scratch)
    return out, res


def _worker(rank, world, port, errs):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got, res = run_tp(rank, world)
        ref, _ = run_tp(0, 1)
        for k in got:
            # every rank holds the full (replicated) residual streams after the all-reduces
            d1, d0 = (got[k] - res[k]).double().flatten(), (ref[k] - res[k]).double().flatten()
            err = (d1 - d0).abs().max() / d0.abs().max()
            cos = (d1 @ d0) / (d1.norm() * d0.norm())
            if not (err <= 1e-2 and cos >= 0.9999):
                errs.put(f"rank {rank} {k}: err {err:.3e} cos {cos:.6f}")
    except Exception as e:  # surfaces in the parent
        errs.put(f"rank {rank}: {e!r}")
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_tp_block_pair_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    errs = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, free_port(), errs), nprocs=world, start_method="spawn", join=True)
    msgs = []
    while not errs.empty():
        msgs.append(errs.get())
    assert not msgs, msgs


def test_shard_layout():
    txt_w, img_w, sw, *_ = make_inputs()
    world = 2
    parts = [tp.shard_single(sw, r, world, D) for r in range(world)]
    H, hd = D.hidden, D.heads // world * D.dhead
    # the packed linear2 slices cover every input column of linear2 exactly once
    cols = torch.cat([torch.cat([p.linear2_w[:, :hd], p.linear2_w[:, hd:]], 1) for p in parts], 1)
    perm = torch.cat([torch.cat([torch.arange(r * hd, (r + 1) * hd),
                                 H + torch.arange(r * D.mlp // world, (r + 1) * D.mlp // world)]) for r in range(world)])
    assert torch.equal(cols, sw.linear2_w[:, perm])
    s0 = tp.shard_stream(txt_w, 0, world, D)
    assert s0.proj_w.stride(0) == H and s0.proj_w.data_ptr() == txt_w.proj_w.data_ptr()  # a view, no copy
    with pytest.raises(ValueError):
        tp.shard_stream(txt_w, 0, 3, D)   # 3 does not divide 4 heads
