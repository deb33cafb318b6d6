"""Generates the golden vectors in this directory by running the REFERENCE ITSELF.

    python tests/golden/make_golden.py [out_dir]      # on a machine with a B200

The reference's own GEMM path (cublas_ops.cuh + kernels.cu, compiled from its sources by
oracle/Makefile into oracle/_ref/libref_cublaslt.so) is called on small seeded inputs; the
inputs and its outputs are saved as .npz.  tests/test_oracle_golden.py then pins the C
oracle (oracle/oracle.c) to these files on any machine, without a GPU.

Inputs are numpy-seeded (PCG64, seed per case); bf16/fp16 tensors are stored as their raw
uint16 bit patterns.  torch is used only to hold device buffers.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO / "oracle"))
from oracle import BF16, CUDA_R_16BF, CUDA_R_16F, CUDA_R_32F, F16, F32, AttnRef, Oracle, Ref  # noqa: E402

DEV = torch.device("cuda:0")
ORC = Oracle()  # only for float -> bf16/fp16 bit conversion of the seeded inputs


def dev(a: np.ndarray) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(DEV)
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t: torch.Tensor, dtype) -> np.ndarray:
    a = t.cpu().numpy()
    return a.view(np.uint16) if dtype == np.uint16 else a.astype(dtype)


def bits(a: np.ndarray, dt: int) -> np.ndarray:
    if dt == BF16:
        return ORC.to_bf16_bits(a)
    if dt == F16:
        return ORC.to_f16_bits(a)
    return np.ascontiguousarray(a, dtype=np.float32)


CUDA_T = {F32: CUDA_R_32F, F16: CUDA_R_16F, BF16: CUDA_R_16BF}


def main(out_dir: Path) -> None:
    ref = Ref()
    out_dir.mkdir(parents=True, exist_ok=True)
    saved = []

    def save(name, **arrays):
        np.savez_compressed(out_dir / f"{name}.npz", **arrays)
        saved.append(name)

    # linear_lt with one operand dtype (cublas_ops.cuh:214)
    for name, (M, K, N, dt, has_bias, seed) in {
        "linear_lt_bf16_bias": (37, 200, 72, BF16, True, 1),
        "linear_lt_bf16_nobias": (128, 256, 256, BF16, False, 2),
        "linear_lt_fp16": (19, 136, 40, F16, False, 3),
        "linear_lt_f32_k67": (16, 67, 24, F32, True, 4),
    }.items():
        rng = np.random.default_rng(seed)
        x = bits(rng.standard_normal((M, K), dtype=np.float32), dt)
        w = bits((rng.standard_normal((N, K), dtype=np.float32) * 0.02), dt)
        bias = (rng.standard_normal(N, dtype=np.float32) * 0.02) if has_bias else None
        xo, wo = dev(x), dev(w)
        bo = dev(bias) if has_bias else None
        out = torch.zeros((M, N), dtype=torch.float32, device=DEV)
        ref.linear_lt(M, K, N, xo.data_ptr(), CUDA_T[dt], wo.data_ptr(), CUDA_T[dt],
                      bo.data_ptr() if has_bias else None, out.data_ptr())
        ref.sync()
        arrays = dict(x=x, w=w, out=host(out, np.float32), dtype=np.int32(dt))
        if has_bias:
            arrays["bias"] = bias
        save(name, **arrays)

    # linear() with F32 activations and 16-bit weights: the reference casts x first (:484-495)
    for name, (M, K, N, wdt, seed) in {
        "linear_f32x_bf16w": (33, 96, 48, BF16, 5),
        "linear_f32x_fp16w": (9, 64, 32, F16, 6),
    }.items():
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((M, K), dtype=np.float32)
        w = bits(rng.standard_normal((N, K), dtype=np.float32) * 0.02, wdt)
        bias = rng.standard_normal(N, dtype=np.float32) * 0.02
        xo, wo, bo = dev(x), dev(w), dev(bias)
        out = torch.zeros((M, N), dtype=torch.float32, device=DEV)
        ref.linear(xo.data_ptr(), F32, wo.data_ptr(), wdt, bo.data_ptr(), out.data_ptr(), M, K, N)
        ref.sync()
        save(name, x=x, w=w, bias=bias, out=host(out, np.float32), wdtype=np.int32(wdt))

    # linear_gated_residual (cublas_ops.cuh:684), bf16 activations and weights
    rng = np.random.default_rng(7)
    M, K, N = 20, 64, 40
    x = bits(rng.standard_normal((M, K), dtype=np.float32), BF16)
    w = bits(rng.standard_normal((N, K), dtype=np.float32) * 0.02, BF16)
    bias = rng.standard_normal(N, dtype=np.float32) * 0.02
    resid = rng.standard_normal((M, N), dtype=np.float32)
    gate = rng.standard_normal(N, dtype=np.float32)
    ro, xo, wo, bo, go_ = dev(resid), dev(x), dev(w), dev(bias), dev(gate)
    ref.linear_gated_residual(xo.data_ptr(), BF16, wo.data_ptr(), BF16, bo.data_ptr(), ro.data_ptr(), go_.data_ptr(),
                              M, K, N)
    ref.sync()
    save("linear_gated_residual_bf16", x=x, w=w, bias=bias, resid=resid, gate=gate, out=host(ro, np.float32))

    # GELU (kernels.cu:266-310)
    rng = np.random.default_rng(8)
    g = np.concatenate([np.linspace(-8, 8, 1001, dtype=np.float32), rng.standard_normal(1000, dtype=np.float32) * 3])
    go = dev(g)
    o32 = torch.zeros_like(go)
    o16 = torch.zeros(g.shape, dtype=torch.int16, device=DEV)
    ref.gelu(go.data_ptr(), o32.data_ptr(), g.size)
    ref.gelu_to_bf16(go.data_ptr(), o16.data_ptr(), g.size)
    ref.sync()
    save("gelu", x=g, out=host(o32, np.float32), out_bf16=host(o16, np.uint16))

    # gated_residual (kernels.cu:942-968)
    rng = np.random.default_rng(9)
    M, C = 7, 48
    gx = rng.standard_normal((M, C), dtype=np.float32)
    gy = rng.standard_normal((M, C), dtype=np.float32)
    gg = rng.standard_normal(C, dtype=np.float32)
    oo = torch.zeros((M, C), dtype=torch.float32, device=DEV)
    gxo, gyo, ggo = dev(gx), dev(gy), dev(gg)
    ref.gated_residual(gxo.data_ptr(), gyo.data_ptr(), ggo.data_ptr(), oo.data_ptr(), M, C)
    ref.sync()
    save("gated_residual", x=gx, y=gy, gate=gg, out=host(oo, np.float32))

    # batched_matmul_Bt (cublas_ops.cuh:558), F32 with FAST_16BF
    rng = np.random.default_rng(10)
    B_, M, K, N = 3, 16, 64, 24
    A = rng.standard_normal((B_, M, K), dtype=np.float32)
    Bm = rng.standard_normal((B_, N, K), dtype=np.float32)
    Co = torch.zeros((B_, M, N), dtype=torch.float32, device=DEV)
    Ao, Bo = dev(A), dev(Bm)
    ref.batched_matmul_Bt(Ao.data_ptr(), Bo.data_ptr(), Co.data_ptr(), B_, M, K, N)
    ref.sync()
    save("batched_matmul_Bt", A=A, B=Bm, out=host(Co, np.float32))

    # modulate_to_bf16 (kernels.cu:552-599) and rms_norm (kernels.cu:174-207)
    rng = np.random.default_rng(11)
    M, C = 5, 96
    mx = rng.standard_normal((M, C), dtype=np.float32) * 2 + 0.5
    sh = rng.standard_normal(C, dtype=np.float32) * 0.1
    sc = rng.standard_normal(C, dtype=np.float32) * 0.1
    mo = torch.zeros((M, C), dtype=torch.int16, device=DEV)
    mxo, sho, sco = dev(mx), dev(sh), dev(sc)
    ref.modulate_to_bf16(mxo.data_ptr(), sho.data_ptr(), sco.data_ptr(), mo.data_ptr(), M, C, 1e-6)
    rows, C2 = 6, 128
    rx = rng.standard_normal((rows, C2), dtype=np.float32)
    rs = rng.standard_normal(C2, dtype=np.float32) * 0.5 + 1.0
    ro2 = torch.zeros((rows, C2), dtype=torch.float32, device=DEV)
    rxo, rso = dev(rx), dev(rs)
    ref.rms_norm(rxo.data_ptr(), rso.data_ptr(), ro2.data_ptr(), rows, C2, 1e-6)
    ref.sync()
    save("modulate_to_bf16", x=mx, shift=sh, scale=sc, out_bf16=host(mo, np.uint16))
    save("rms_norm", x=rx, scale=rs, out=host(ro2, np.float32))

    # attention_with_rope (attention.cuh:23 -> cuDNN SDPA), with a 0/-inf key mask
    attn = AttnRef()
    rng = np.random.default_rng(12)
    L, H, D = 128, 2, 128
    aq, ak, av = (rng.standard_normal((L, H, D), dtype=np.float32) for _ in range(3))
    ang = rng.uniform(0, 2 * np.pi, (L, D // 2)).astype(np.float32)
    pe = np.stack([np.cos(ang), -np.sin(ang), np.sin(ang), np.cos(ang)], -1).astype(np.float32)
    mask = np.zeros(L, np.float32)
    mask[40:64] = -np.inf
    dq, dk, dv, dpe, dm = dev(aq), dev(ak), dev(av), dev(pe), dev(mask)
    ao = torch.zeros((L, H * D), dtype=torch.float32, device=DEV)
    attn.attention_with_rope(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dpe.data_ptr(), H, D, L, dm.data_ptr(),
                             ao.data_ptr())
    torch.cuda.synchronize()
    save("attention_rope", q=aq, k=ak, v=av, pe=pe, mask=mask, out=host(ao, np.float32))

    (out_dir / "MANIFEST.txt").write_text(
        "Golden vectors from the reference's own kernels (oracle/_ref/libref_cublaslt.so, cuBLASLt "
        f"{ref.cublaslt_version()}) on {torch.cuda.get_device_name(0)}.\n"
        "Generated by tests/golden/make_golden.py.\n" + "\n".join(saved) + "\n")
    print("wrote", len(saved), "fixtures to", out_dir)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent)
