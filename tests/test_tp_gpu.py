"""Tensor-parallel block pair on B200s.  With one GPU: the TP code at world size 1 (no
all-reduce) against the unsharded engine path.  With two or more visible GPUs: torchrun over
all of them (NCCL) through tests/tp_gpu_worker.py, each rank checked against the unsharded
path (update max|d|/max|ref| <= 1e-2, cosine >= 0.9999)."""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
HERE = Path(__file__).resolve().parent


def test_tp_world1_matches_blocks(engine):
    import blocks
    import tp

    T, I = 512, 1024
    L = T + I
    g = torch.Generator(device=DEV).manual_seed(5)
    txt_w, img_w = blocks.random_stream(g, DEV), blocks.random_stream(g, DEV)
    sw = blocks.random_single(g, DEV)
    H = blocks.HIDDEN
    act = {k: torch.randn((n, H), generator=g, device=DEV).to(torch.bfloat16) for k, n in
           (("txt_mod1", T), ("img_mod1", I), ("txt_mod2", T), ("img_mod2", I), ("x_mod", L))}
    res = {k: torch.randn((n, H), generator=g, device=DEV) for k, n in (("txt", T), ("img", I), ("x", L))}
    gates = [torch.randn(H, generator=g, device=DEV) for _ in range(5)]
    ang = torch.rand((L, blocks.DHEAD // 2), generator=g, device=DEV) * 6.28
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    mask = torch.zeros(L, device=DEV)
    mask[100:512] = float("-inf")
    ref = {k: v.clone() for k, v in res.items()}
    s1 = blocks.Scratch(T, I, DEV)
    blocks.double_block(txt_w, img_w, act["txt_mod1"], act["img_mod1"], act["txt_mod2"], act["img_mod2"], ref["txt"],
                        ref["img"], gates[0], gates[1], gates[2], gates[3], pe, mask, s1)
    blocks.single_block(sw, act["x_mod"], ref["x"], gates[4], pe, mask, s1)
    got = {k: v.clone() for k, v in res.items()}
    ops = tp.EngineOps()
    s = tp.TPScratch(T, I, 1, DEV)
    tp.tp_double_block(ops, tp.shard_stream(txt_w, 0, 1), tp.shard_stream(img_w, 0, 1), act["txt_mod1"],
                       act["img_mod1"], act["txt_mod2"], act["img_mod2"], got["txt"], got["img"], gates[0], gates[1],
                       gates[2], gates[3], pe, mask, s)
    tp.tp_single_block(ops, tp.shard_single(sw, 0, 1), act["x_mod"], got["x"], gates[4], pe, mask, s)
    torch.cuda.synchronize()
    for k in got:
        d1, d0 = (got[k] - res[k]).double().flatten(), (ref[k] - res[k]).double().flatten()
        assert ((d1 - d0).abs().max() / d0.abs().max()).item() <= 1e-2, k
        assert ((d1 @ d0) / (d1.norm() * d0.norm())).item() >= 0.9999, k


@pytest.mark.parametrize("M,dtype,with_bias", [(300, torch.bfloat16, True), (301, torch.bfloat16, False),
                                                (7, torch.float32, True), (4608, torch.bfloat16, True)])
def test_bias_gated_residual_kernel(engine, M, dtype, with_bias):
    """residual += gate * (y + bias) after a tensor-parallel all-reduce (gated_residual,
    kernels.cu:942-968), rows not a multiple of the kernel's 4-row groups included."""
    g = torch.Generator(device=DEV).manual_seed(9)
    y = torch.randn((M, 3072), generator=g, device=DEV).to(dtype)
    b = torch.randn(3072, generator=g, device=DEV) if with_bias else None
    gate = torch.randn(3072, generator=g, device=DEV)
    r = torch.randn((M, 3072), generator=g, device=DEV)
    want = r + gate * (y.float() + (b if with_bias else 0.0))
    engine.bias_gated_residual(y, b, gate, r)
    torch.cuda.synchronize()
    assert torch.allclose(r, want, rtol=1e-6, atol=1e-5)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_tp_multi_gpu_matches_unsharded():
    n = min(torch.cuda.device_count(), 8)
    n = 8 if n >= 8 else (4 if n >= 4 else 2)
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={port}", str(HERE / "tp_gpu_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
