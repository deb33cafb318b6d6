"""GPU parity of the engine's GEMM path against the C oracle, the reference's own cuBLASLt
build, and a plain fp32 product, through the C ABI.

Tolerance (north star): per GEMM, max|got - ref| / max|ref| <= 2e-3 for bf16 operands.  F32
outputs are held to 1e-4 (fp32 accumulation order only).  A bf16 or fp16 *output* adds one
rounding whose size no GEMM can avoid: half an ulp of the value, up to 2^-8 of max|ref| for
bf16 when the largest value sits just above a power of two.  Those outputs are therefore
checked element by element for correct rounding: |got - ref| <= ulp(ref)/2 + 1e-5 max|ref|
(the second term is fp32 accumulation-order noise).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL_F32_OUT = 1e-4


def seeded(shape, seed, scale=1.0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype).to(DEV)


def fp32_ref(x, w, bias=None):
    y = x.double() @ w.double().t()
    if bias is not None:
        y = y + bias.double()
    return y


def assert_rounded(got16: torch.Tensor, ref: torch.Tensor):
    """got16 (bf16/fp16) is ref correctly rounded, up to fp32 accumulation noise."""
    mant = 7 if got16.dtype == torch.bfloat16 else 10
    g = got16.double().cpu()
    r = ref.double().cpu()
    mag = r.abs().clamp_min(torch.finfo(torch.float32).tiny)
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - mant)
    bound = 0.5 * ulp + 1e-5 * r.abs().max()
    excess = ((g - r).abs() - bound).max().item()
    assert excess <= 0, f"rounding error exceeds half an ulp by {excess:.3e}"


def check(out, ref):
    if out.dtype == torch.float32:
        assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= TOL_F32_OUT
    else:
        assert_rounded(out, ref)


def gelu_t(y):
    return 0.5 * y * (1 + torch.tanh(0.7978845608 * (y + 0.044715 * y ** 3)))


SHAPES = [
    # M, N, K
    (128, 256, 64),        # one tile, one k-block
    (256, 512, 1024),
    (100, 200, 72),        # ragged M, N and K
    (1, 8, 8),             # smallest
    (7, 1000, 136),
    (300, 130, 3000),      # K tail, N < 256 tile
    (1536, 3072, 3072),    # single-block Q/K/V at 512^2
    (512, 9216, 3072),     # double-block txt qkv
    (1024, 3072, 12288),   # double-block img mlp2
    (1536, 3072, 15360),   # single-block linear2
    (344, 5120, 5120),     # approximator (skinny M)
]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_bias_vs_fp64(engine, M, N, K, out_dtype):
    x = seeded((M, K), M + N + K)
    w = seeded((N, K), M * N + 1, 0.02)
    bias = seeded((N,), 7, 0.02, torch.float32)
    out = engine.gemm(x, w, bias, out_dtype=out_dtype)
    torch.cuda.synchronize()
    check(out, fp32_ref(x, w, bias))


@pytest.mark.parametrize("variant", [0, 1, 2])
@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (300, 700, 520), (1536, 3072, 3072), (100, 200, 72),
                                   (513, 300, 3000), (777, 1300, 200)])
def test_every_kernel_variant(engine, variant, M, N, K):
    """Each tensor-core kernel (1-CTA 128/256-wide, 2-CTA 256x256 pair) forced on ragged
    shapes, with bias and GELU epilogues and F32 / bf16 outputs."""
    x = seeded((M, K), 3 * M + K)
    w = seeded((N, K), 5 * N + K, 0.02)
    bias = seeded((N,), 9, 0.02, torch.float32)
    try:
        engine.set_gemm_variant(variant, 1)
        out = engine.gemm(x, w, bias, out_dtype=torch.float32)
        out16 = engine.gemm(x, w, bias, out_dtype=torch.bfloat16, epilogue="gelu")
        torch.cuda.synchronize()
    finally:
        engine.set_gemm_variant(-1, 0)
    ref = fp32_ref(x, w, bias)
    check(out, ref)
    check(out16, gelu_t(ref))


@pytest.mark.parametrize("splits", [-2, -5, -8])
@pytest.mark.parametrize("variant,M,N,K", [(2, 512, 10240, 1024), (0, 1024, 2560, 512), (1, 1024, 5120, 640)])
def test_split_last_wave(engine, variant, splits, M, N, K):
    """Whole tiles for the full waves and the last, partial wave's tiles split (80 pair tiles
    on 74 SM pairs, 160 tiles on 148 SMs): every epilogue kind, twice in a row."""
    x = seeded((M, K), 5 * M + K)
    w = seeded((N, K), 3 * N + K, 0.02)
    bias = seeded((N,), 23, 0.02, torch.float32)
    gate = seeded((N,), 24, 1.0, torch.float32)
    r0 = seeded((M, N), 25, 1.0, torch.float32)
    ref = fp32_ref(x, w, bias)
    try:
        engine.set_gemm_variant(variant, splits)
        for _ in range(2):
            out = engine.gemm(x, w, bias, out_dtype=torch.float32)
            g16 = engine.gemm(x, w, bias, out_dtype=torch.bfloat16, epilogue="gelu")
            res = r0.clone()
            engine.gemm(x, w, bias, out=res, epilogue="gated_residual", gate=gate)
            torch.cuda.synchronize()
            check(out, ref)
            check(g16, gelu_t(ref))
            assert rel_err(res.cpu().numpy(), (r0.double() + gate.double() * ref).cpu().numpy()) <= TOL_F32_OUT
    finally:
        engine.set_gemm_variant(-1, 0)
    engine.check_device_error()


@pytest.mark.parametrize("variant", [0, 1, 2])
@pytest.mark.parametrize("splits", [2, 3, 5])
@pytest.mark.parametrize("M,N,K", [(512, 3072, 3072), (300, 700, 2000), (1024, 3072, 12288)])
def test_split_k(engine, variant, splits, M, N, K):
    """Split-K partial sums (workspace + last-arriver reduction) for every kernel variant and
    epilogue kind, twice in a row (the arrival counters must re-arm themselves)."""
    x = seeded((M, K), 7 * M + K)
    w = seeded((N, K), 11 * N + K, 0.02)
    bias = seeded((N,), 13, 0.02, torch.float32)
    gate = seeded((N,), 14, 1.0, torch.float32)
    r0 = seeded((M, N), 15, 1.0, torch.float32)
    ref = fp32_ref(x, w, bias)
    try:
        engine.set_gemm_variant(variant, splits)
        for _ in range(2):
            out = engine.gemm(x, w, bias, out_dtype=torch.float32)
            g16 = engine.gemm(x, w, bias, out_dtype=torch.bfloat16, epilogue="gelu")
            res = r0.clone()
            engine.gemm(x, w, bias, out=res, epilogue="gated_residual", gate=gate)
            torch.cuda.synchronize()
            check(out, ref)
            check(g16, gelu_t(ref))
            assert rel_err(res.cpu().numpy(), (r0.double() + gate.double() * ref).cpu().numpy()) <= TOL_F32_OUT
    finally:
        engine.set_gemm_variant(-1, 0)
    engine.check_device_error()


def test_split_k_is_deterministic(engine):
    x = seeded((512, 3072), 201)
    w = seeded((3072, 3072), 202, 0.02)
    try:
        engine.set_gemm_variant(1, 4)
        a = engine.gemm(x, w, out_dtype=torch.float32)
        b = engine.gemm(x, w, out_dtype=torch.float32)
        torch.cuda.synchronize()
    finally:
        engine.set_gemm_variant(-1, 0)
    assert torch.equal(a, b)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (512, 10240, 4096), (512, 4096, 10240), (19, 40, 136)])
def test_gemm_t5_shapes_fp16_and_bf16(engine, dt, M, N, K):
    x = seeded((M, K), 11, 1.0, dt)
    w = seeded((N, K), 12, 0.02, dt)
    out = engine.gemm(x, w, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), fp32_ref(x, w).cpu().numpy()) <= TOL_F32_OUT


@pytest.mark.parametrize("M,N,K", [(512, 12288, 3072), (100, 300, 64), (1536, 12288, 3072)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gemm_gelu_epilogue(engine, M, N, K, out_dtype):
    x = seeded((M, K), 21)
    w = seeded((N, K), 22, 0.02)
    bias = seeded((N,), 23, 0.02, torch.float32)
    out = engine.gemm(x, w, bias, out_dtype=out_dtype, epilogue="gelu")
    torch.cuda.synchronize()
    check(out, gelu_t(fp32_ref(x, w, bias)))


@pytest.mark.parametrize("M,N,K", [(1024, 3072, 12288), (1536, 3072, 15360), (33, 70, 96)])
def test_gemm_gated_residual_epilogue(engine, M, N, K):
    x = seeded((M, K), 31)
    w = seeded((N, K), 32, 0.02)
    bias = seeded((N,), 33, 0.02, torch.float32)
    resid = seeded((M, N), 34, 1.0, torch.float32)
    gate = seeded((N,), 35, 1.0, torch.float32)
    want = resid.double() + gate.double() * fp32_ref(x, w, bias)
    engine.gemm(x, w, bias, out=resid, epilogue="gated_residual", gate=gate)
    torch.cuda.synchronize()
    assert rel_err(resid.cpu().numpy(), want.cpu().numpy()) <= TOL_F32_OUT


def test_gemm_vs_c_oracle(engine, oracle):
    """Same seeded bf16 inputs through the engine and the fp32 C oracle."""
    M, N, K = 200, 384, 520
    x = seeded((M, K), 41)
    w = seeded((N, K), 42, 0.02)
    bias = seeded((N,), 43, 0.02, torch.float32)
    out = engine.gemm(x, w, bias, out_dtype=torch.float32)
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
    wb = w.cpu().view(torch.int16).numpy().view(np.uint16)
    want = oracle.linear(xb, 2, wb, 2, bias.cpu().numpy())
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), want) <= TOL_F32_OUT


@pytest.mark.parametrize("M,K,N", [(1536, 3072, 21504), (512, 3072, 9216), (37, 200, 72)])
def test_linear_lt_vs_reference_cublaslt(engine, ref, M, K, N):
    """b2g_linear_lt and the reference's linear_lt (cuBLASLt) on identical device buffers."""
    x = seeded((M, K), 51)
    w = seeded((N, K), 52, 0.02)
    bias = seeded((N,), 53, 0.02, torch.float32)
    mine = torch.empty((M, N), device=DEV)
    theirs = torch.empty((M, N), device=DEV)
    engine.linear_lt(M, K, N, x, engine.CUDA_R_16BF, w, engine.CUDA_R_16BF, bias, mine)
    ref.linear_lt(M, K, N, x.data_ptr(), 14, w.data_ptr(), 14, bias.data_ptr(), theirs.data_ptr())
    torch.cuda.synchronize()
    assert rel_err(mine.cpu().numpy(), theirs.cpu().numpy()) <= 2e-3
    assert rel_err(mine.cpu().numpy(), theirs.cpu().numpy()) <= TOL_F32_OUT


def test_config1_bf16_out_vs_reference(engine, ref):
    """BASELINE config 1 (linear1 GEMM+bias, seed 0): the engine's F32 output within the
    north-star 2e-3 of the reference's, and its bf16 output the reference's correctly rounded."""
    M, K, N = 1536, 3072, 21504
    g = torch.Generator().manual_seed(0)
    x = torch.randn((M, K), generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn((N, K), generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    bias = (torch.randn((N,), generator=g) * 0.02).to(torch.bfloat16).float().to(DEV)
    mine = engine.gemm(x, w, bias, out_dtype=torch.bfloat16)
    theirs = torch.empty((M, N), device=DEV)
    ref.linear_lt(M, K, N, x.data_ptr(), 14, w.data_ptr(), 14, bias.data_ptr(), theirs.data_ptr())
    mine32 = engine.gemm(x, w, bias, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert rel_err(mine32.cpu().numpy(), theirs.cpu().numpy()) <= 2e-3
    assert_rounded(mine, theirs)


@pytest.mark.parametrize("wdt", [torch.bfloat16, torch.float16])
def test_linear_f32_activation_cast_matches_reference(engine, ref, wdt):
    """linear() with F32 x and 16-bit W casts x first, in both implementations."""
    M, K, N = 512, 4096, 1024
    x = seeded((M, K), 61, 1.0, torch.float32)
    w = seeded((N, K), 62, 0.02, wdt)
    bias = seeded((N,), 63, 0.02, torch.float32)
    mine = torch.empty((M, N), device=DEV)
    theirs = torch.empty((M, N), device=DEV)
    engine.linear(x, w, bias, mine)
    wcode = 2 if wdt == torch.bfloat16 else 1
    ref.linear(x.data_ptr(), 0, w.data_ptr(), wcode, bias.data_ptr(), theirs.data_ptr(), M, K, N)
    torch.cuda.synchronize()
    assert rel_err(mine.cpu().numpy(), theirs.cpu().numpy()) <= TOL_F32_OUT


def test_linear_f32_f32_exact_path(engine, ref):
    M, K, N = 64, 67, 96  # K=67 like the NeRF embedder: no TMA, exact fp32 CUDA-core path
    x = seeded((M, K), 71, 1.0, torch.float32)
    w = seeded((N, K), 72, 0.1, torch.float32)
    bias = seeded((N,), 73, 0.02, torch.float32)
    mine = torch.empty((M, N), device=DEV)
    theirs = torch.empty((M, N), device=DEV)
    engine.linear(x, w, bias, mine)
    ref.linear(x.data_ptr(), 0, w.data_ptr(), 0, bias.data_ptr(), theirs.data_ptr(), M, K, N)
    torch.cuda.synchronize()
    assert rel_err(mine.cpu().numpy(), theirs.cpu().numpy()) <= 1e-5


def test_linear_gated_residual_vs_reference(engine, ref):
    M, K, N = 1024, 3072, 3072
    x = seeded((M, K), 81, 1.0, torch.float32)   # attention output is F32 in the reference
    w = seeded((N, K), 82, 0.02)
    bias = seeded((N,), 83, 0.02, torch.float32)
    gate = seeded((N,), 84, 1.0, torch.float32)
    r0 = seeded((M, N), 85, 1.0, torch.float32)
    mine, theirs = r0.clone(), r0.clone()
    engine.linear_gated_residual(x, w, bias, mine, gate, M, N)
    ref.linear_gated_residual(x.data_ptr(), 0, w.data_ptr(), 2, bias.data_ptr(), theirs.data_ptr(),
                              gate.data_ptr(), M, K, N)
    torch.cuda.synchronize()
    assert rel_err(mine.cpu().numpy(), theirs.cpu().numpy()) <= TOL_F32_OUT


BATCHED = [(64, 256, 64, 256), (5, 256, 256, 64), (3, 16, 64, 24), (2, 50, 70, 30)]


@pytest.mark.parametrize("batch,M,K,N", BATCHED)
def test_batched_matmul_bt_vs_oracle(engine, oracle, batch, M, K, N):
    A = seeded((batch, M, K), 91, 1.0, torch.float32)
    B = seeded((batch, N, K), 92, 1.0, torch.float32)
    mine = torch.empty((batch, M, N), device=DEV)
    engine.batched_matmul_Bt(A, B, mine)
    want = oracle.batched_matmul_bt(A.cpu().numpy(), B.cpu().numpy())  # TF32 operand rounding
    torch.cuda.synchronize()
    got = mine.cpu().numpy()
    for b in range(batch):
        assert rel_err(got[b], want[b]) <= TOL_F32_OUT, f"batch {b}"


@pytest.mark.parametrize("batch,M,K,N", BATCHED)
def test_batched_matmul_bt_vs_reference(engine, ref, oracle, batch, M, K, N):
    A = seeded((batch, M, K), 91, 1.0, torch.float32)
    B = seeded((batch, N, K), 92, 1.0, torch.float32)
    mine = torch.empty((batch, M, N), device=DEV)
    theirs = torch.zeros((batch, M, N), device=DEV)
    engine.batched_matmul_Bt(A, B, mine)
    ref.batched_matmul_Bt(A.data_ptr(), B.data_ptr(), theirs.data_ptr(), batch, M, K, N)
    torch.cuda.synchronize()
    want = oracle.batched_matmul_bt(A.cpu().numpy(), B.cpu().numpy())
    t = theirs.cpu().numpy()
    per_batch_ref = [rel_err(t[b], want[b]) for b in range(batch)]
    assert rel_err(mine.cpu().numpy(), t) <= TOL_F32_OUT, f"reference vs oracle per batch: {per_batch_ref}"


GROUPS = [
    # (M0, M1, N, K): the double block's txt/img layer pairs at 512^2, then ragged shapes
    (512, 1024, 9216, 3072), (512, 1024, 3072, 3072), (512, 1024, 3072, 12288), (100, 300, 700, 136),
    (1, 77, 64, 8),
]


@pytest.mark.parametrize("variant", [-1, 0, 1, 2])
@pytest.mark.parametrize("M0,M1,N,K", GROUPS)
@pytest.mark.parametrize("epilogue,out_dtype", [("none", torch.float32), ("gelu", torch.bfloat16),
                                                ("gated_residual", torch.float32)])
def test_gemm_group_one_launch(engine, variant, M0, M1, N, K, epilogue, out_dtype):
    """Two problems with their own rows, weights, biases and gates in one launch."""
    if variant in (1, 2) and N <= 128:
        pytest.skip("256-wide tiles need N > 128")
    engine.set_gemm_variant(variant, 0)
    try:
        probs, refs = [], []
        for i, M in enumerate((M0, M1)):
            x = seeded((M, K), 7 * M + i)
            w = seeded((N, K), 11 * M + i, 0.02)
            b = seeded((N,), 13 * M + i, 0.02, torch.float32)
            gate = seeded((N,), 17 * M + i, 1.0, torch.float32) if epilogue == "gated_residual" else None
            out = (seeded((M, N), 19 * M + i, 1.0, torch.float32) if gate is not None
                   else torch.empty((M, N), dtype=out_dtype, device=DEV))
            y = fp32_ref(x, w, b)
            if epilogue == "gelu":
                y = gelu_t(y)
            elif gate is not None:
                y = out.double() + gate.double() * y
            refs.append(y)
            probs.append(dict(x=x, w=w, bias=b, out=out, epilogue=epilogue, gate=gate))
        n0 = engine.launch_count()
        engine.gemm_group(probs)
        torch.cuda.synchronize()
        assert engine.launch_count() - n0 == 1
        for pr, y in zip(probs, refs):
            check(pr["out"], y)
    finally:
        engine.set_gemm_variant(-1, 0)
    engine.check_device_error()


FOUR = [
    # (Ms, N, K): the double block's layers with guidance halves at 512^2 ([txt_c, txt_u, img_c,
    # img_u] row blocks), then ragged rows and K
    ((512, 512, 1024, 1024), 3072, 3072), ((3, 130, 257, 64), 640, 200),
]


@pytest.mark.parametrize("variant", [-1, 0, 1, 2])
@pytest.mark.parametrize("Ms,N,K", FOUR)
@pytest.mark.parametrize("epilogue,out_dtype", [("none", torch.float32), ("gelu", torch.bfloat16),
                                                ("gated_residual", torch.float32)])
def test_gemm_group_four_problems_one_launch(engine, variant, Ms, N, K, epilogue, out_dtype):
    """Four problems (problems 0/1 and 2/3 share a weight, as the guidance halves of one stream
    do) in one launch; every variant; the outputs are row views of one buffer."""
    engine.set_gemm_variant(variant, 0)
    try:
        ws = [seeded((N, K), 31 * K + j, 0.02) for j in range(2)]
        bs = [seeded((N,), 37 * K + j, 0.02, torch.float32) for j in range(2)]
        gate = seeded((N,), 41, 1.0, torch.float32) if epilogue == "gated_residual" else None
        rows = sum(Ms)
        buf = (seeded((rows, N), 43, 1.0, torch.float32) if gate is not None
               else torch.zeros((rows, N), dtype=out_dtype, device=DEV))
        probs, refs, r0 = [], [], 0
        for i, M in enumerate(Ms):
            x = seeded((M, K), 47 * M + i)
            out = buf[r0:r0 + M]
            y = fp32_ref(x, ws[i // 2], bs[i // 2])
            if epilogue == "gelu":
                y = gelu_t(y)
            elif gate is not None:
                y = out.double() + gate.double() * y
            refs.append(y)
            probs.append(dict(x=x, w=ws[i // 2], bias=bs[i // 2], out=out, epilogue=epilogue, gate=gate))
            r0 += M
        n0 = engine.launch_count()
        engine.gemm_group(probs)
        torch.cuda.synchronize()
        assert engine.launch_count() - n0 == 1
        for pr, y in zip(probs, refs):
            check(pr["out"], y)
    finally:
        engine.set_gemm_variant(-1, 0)
    engine.check_device_error()


def test_gemm_group_five_problems_run_one_by_one(engine):
    xs = [seeded((64 + 8 * i, 256), 60 + i) for i in range(5)]
    w = seeded((384, 256), 70, 0.02)
    n0 = engine.launch_count()
    outs = engine.gemm_group([dict(x=x, w=w) for x in xs])
    torch.cuda.synchronize()
    assert engine.launch_count() - n0 == 5
    for x, o in zip(xs, outs):
        check(o, fp32_ref(x, w))


def test_gemm_group_shares_the_activation_cast(engine):
    """Problems on one F32 input against fp16 weights (the T5 layer's q, k, v) cast it once and
    run as one launch; with different epilogues (wi_0 GELU, wi_1 none) the cast is still shared.
    Results equal each problem run alone (same fp16 operands)."""
    x = seeded((200, 512), 1, 1.0, torch.float32)
    ws = [seeded((384, 512), 2 + i, 0.02, torch.float16) for i in range(3)]
    alone = [engine.gemm(x, w) for w in ws]
    n0 = engine.launch_count()
    grouped = engine.gemm_group([dict(x=x, w=w) for w in ws])
    torch.cuda.synchronize()
    assert engine.launch_count() - n0 == 2            # one cast + one GEMM launch
    for a, b in zip(alone, grouped):
        assert rel_err(b.cpu().numpy(), a.cpu().numpy()) <= 1e-6
    n0 = engine.launch_count()
    g2 = engine.gemm_group([dict(x=x, w=ws[0], epilogue="gelu"), dict(x=x, w=ws[1])])
    torch.cuda.synchronize()
    assert engine.launch_count() - n0 == 3            # one cast + two GEMM launches
    assert rel_err(g2[1].cpu().numpy(), alone[1].cpu().numpy()) <= 1e-6
    check(g2[0], gelu_t(fp32_ref(x.to(torch.float16), ws[0])))


def test_gemm_group_split_k(engine):
    engine.set_gemm_variant(2, 3)
    try:
        xs = [seeded((M, 3072), M) for M in (512, 1024)]
        ws = [seeded((3072, 3072), M + 1, 0.02) for M in (512, 1024)]
        outs = engine.gemm_group([dict(x=x, w=w) for x, w in zip(xs, ws)])
        torch.cuda.synchronize()
        for x, w, o in zip(xs, ws, outs):
            check(o, fp32_ref(x, w))
    finally:
        engine.set_gemm_variant(-1, 0)


def test_gemm_group_mismatched_problems_run_one_by_one(engine):
    x0, w0 = seeded((64, 256), 1), seeded((128, 256), 2, 0.02)
    x1, w1 = seeded((96, 256), 3), seeded((192, 256), 4, 0.02)      # different N: no shared launch
    n0 = engine.launch_count()
    o0, o1 = engine.gemm_group([dict(x=x0, w=w0), dict(x=x1, w=w1, out_dtype=torch.bfloat16)])
    torch.cuda.synchronize()
    assert engine.launch_count() - n0 == 2
    check(o0, fp32_ref(x0, w0))
    check(o1, fp32_ref(x1, w1))


def test_strided_views_like_txt_img_rows(engine):
    """Operands and outputs that are row-offset views of larger buffers (the reference's
    txt/img views) with row strides larger than K / N."""
    big_x = seeded((1536, 3200), 101)
    x = big_x[512:, 64:64 + 3072]            # row stride 3200, base offset 128 B
    w = seeded((3072, 3072), 102, 0.02)
    big_out = torch.zeros((1536, 3328), device=DEV)
    out = big_out[512:, 128:128 + 3072]
    engine.gemm(x, w, None, out=out)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), fp32_ref(x, w).cpu().numpy()) <= TOL_F32_OUT
    assert float(big_out[:512].abs().max()) == 0.0          # nothing written outside the view
    assert float(big_out[512:, :128].abs().max()) == 0.0
    assert float(big_out[512:, 128 + 3072:].abs().max()) == 0.0


def test_unaligned_stride_uses_exact_fallback(engine):
    x = seeded((50, 67), 111)            # K=67: row stride not a multiple of 8 elements
    w = seeded((40, 67), 112, 0.1)
    out = engine.gemm(x, w, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), fp32_ref(x, w).cpu().numpy()) <= 1e-5


def test_empty_and_degenerate_sizes(engine):
    w = seeded((16, 64), 121)
    x0 = torch.empty((0, 64), dtype=torch.bfloat16, device=DEV)
    assert engine.gemm(x0, w).shape == (0, 16)
    # K = 0: the product is empty, the output is the bias
    xk = torch.empty((4, 0), dtype=torch.bfloat16, device=DEV)
    wk = torch.empty((8, 0), dtype=torch.bfloat16, device=DEV)
    bias = torch.arange(8, dtype=torch.float32, device=DEV)
    out = engine.gemm(xk, wk, bias)
    torch.cuda.synchronize()
    assert torch.equal(out, bias.expand(4, 8))


def test_errors_are_raised_not_silenced(engine):
    x = seeded((8, 64), 131)
    w = seeded((8, 32), 132)
    with pytest.raises(engine.B2GError):
        engine.gemm(x, w)                              # K mismatch
    with pytest.raises(engine.B2GError):
        engine.gemm(x, seeded((8, 64), 1, 1.0, torch.float16))   # mixed 16-bit operand types


def test_native_kernels_ran_and_no_device_timeouts(engine):
    n0 = engine.launch_count()
    x = seeded((256, 256), 141)
    engine.gemm(x, x)
    assert engine.launch_count() > n0
    engine.check_device_error()


def rope_table(L, D, seed):
    g = np.random.default_rng(seed)
    ang = g.uniform(0, 2 * np.pi, (L, D // 2))
    return np.stack([np.cos(ang), -np.sin(ang), np.sin(ang), np.cos(ang)], -1).astype(np.float32)


@pytest.mark.parametrize("L,H,D,masked", [(64, 2, 64, 8), (200, 3, 128, 0), (136, 2, 128, 40)])
def test_attention_vs_oracle(engine, oracle, L, H, D, masked):
    g = torch.Generator().manual_seed(L + H)
    Q, K, V = (torch.randn((L, H, D), generator=g) for _ in range(3))
    pe = rope_table(L, D, L)
    mask = np.zeros(L, np.float32)
    if masked:
        mask[L // 3:L // 3 + masked] = -np.inf
    out = engine.attention_with_rope(Q.to(DEV), K.to(DEV), V.to(DEV), torch.from_numpy(pe).to(DEV), H, D,
                                     torch.from_numpy(mask).to(DEV) if masked else None)
    want = oracle.attention_rope(Q.numpy(), K.numpy(), V.numpy(), pe, mask if masked else None)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, want) < 1e-2


@pytest.mark.parametrize("L,H,D,split,out_bf16", [(96, 2, 64, 40, False), (200, 3, 128, -1, True),
                                                   (136, 2, 128, 64, True)])
def test_attention_qknorm_rope_vs_oracle(engine, oracle, L, H, D, split, out_bf16):
    """Fused qk RMSNorm (two scale sets split at row `split`, as the double block's txt/img
    streams) + RoPE + attention, reading q/k/v as column views of one [L, 3*H*D] F32 buffer and
    writing into a column view of a wider output, against oracle rms_norm + attention_rope."""
    g = torch.Generator().manual_seed(L * 7 + H)
    HD = H * D
    qkv = torch.randn((L, 3 * HD), generator=g)
    norms = [1.0 + 0.1 * torch.randn(D, generator=g) for _ in range(4)]
    pe = rope_table(L, D, L + 1)
    mask = np.zeros(L, np.float32)
    mask[L // 4:L // 4 + 9] = -np.inf
    dq = qkv.to(DEV)
    out_w = torch.zeros((L, HD + 40), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=DEV)
    engine.attention_qknorm_rope(dq[:, :HD], dq[:, HD:2 * HD], dq[:, 2 * HD:], torch.from_numpy(pe).to(DEV), H, D,
                                 q_norm=norms[0].to(DEV), k_norm=norms[1].to(DEV), q_norm2=norms[2].to(DEV),
                                 k_norm2=norms[3].to(DEV), norm_split=split, attn_mask=torch.from_numpy(mask).to(DEV),
                                 out=out_w[:, 8:8 + HD], out_dtype=out_w.dtype)
    torch.cuda.synchronize()

    def normed(x, s1, s2):
        rows = x.reshape(L * H, D).numpy()
        a = oracle.rms_norm(rows, s1.numpy()).reshape(L, H, D)
        if split >= 0:
            b = oracle.rms_norm(rows, s2.numpy()).reshape(L, H, D)
            a[split:] = b[split:]
        return a

    q = normed(qkv[:, :HD], norms[0], norms[2])
    k = normed(qkv[:, HD:2 * HD], norms[1], norms[3])
    v = qkv[:, 2 * HD:].reshape(L, H, D).numpy()
    want = oracle.attention_rope(q, k, v, pe, mask)
    got_w = out_w.float().cpu().numpy()
    assert np.all(got_w[:, :8] == 0) and np.all(got_w[:, 8 + HD:] == 0)   # nothing written outside the view
    got = got_w[:, 8:8 + HD]
    assert np.isfinite(got).all()
    assert rel_err(got, want) < 1e-2


@pytest.mark.parametrize("L,H,D", [(136, 2, 128), (320, 3, 64)])
def test_attention_general_key_bias(engine, oracle, L, H, D):
    """A key bias with arbitrary finite values (not only the 0/-inf padding mask) and some
    -inf keys: the kernel's general-bias path against the oracle's additive bias."""
    g = torch.Generator().manual_seed(L + D)
    Q, K, V = (torch.randn((L, H, D), generator=g) for _ in range(3))
    pe = rope_table(L, D, 2 * L)
    bias = (torch.randn(L, generator=g) * 2.0).numpy().astype(np.float32)
    bias[7:19] = -np.inf
    out = engine.attention_with_rope(Q.to(DEV), K.to(DEV), V.to(DEV), torch.from_numpy(pe).to(DEV), H, D,
                                     torch.from_numpy(bias).to(DEV))
    want = oracle.attention_rope(Q.numpy(), K.numpy(), V.numpy(), pe, bias)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, want) < 1e-2


def attn_ref_or_skip():
    from oracle import ATTN_REF_PATH, AttnRef

    if not ATTN_REF_PATH.exists():
        pytest.skip("reference attention library not built")
    return AttnRef()


@pytest.mark.parametrize("L,text_masked", [(1536, 400), (512, 0)])
def test_attention_vs_reference_cudnn(engine, L, text_masked):
    """Config 2: 24 heads x 128 at S=1536 with a 0/-inf key mask on 400 of the 512 text
    tokens, against the reference's cuDNN SDPA path on identical buffers."""
    ref = attn_ref_or_skip()
    H, D = 24, 128
    g = torch.Generator().manual_seed(7)
    Q, K, V = (torch.randn((L, H, D), generator=g).to(DEV) for _ in range(3))
    pe = torch.from_numpy(rope_table(L, D, 3)).to(DEV)
    mask = torch.zeros(L, device=DEV)
    if text_masked:
        mask[512 - text_masked:512] = float("-inf")
    mine = engine.attention_with_rope(Q, K, V, pe, H, D, mask)
    theirs = torch.empty((L, H * D), device=DEV)
    ref.attention_with_rope(Q.data_ptr(), K.data_ptr(), V.data_ptr(), pe.data_ptr(), H, D, L, mask.data_ptr(),
                            theirs.data_ptr())
    torch.cuda.synchronize()
    a, b = mine.double().cpu().numpy().ravel(), theirs.double().cpu().numpy().ravel()
    assert rel_err(a, b) < 1e-2
    assert a @ b / np.sqrt((a @ a) * (b @ b)) > 0.9999


@pytest.mark.parametrize("T,I", [(512, 1024), (512, 4096)])
def test_attention_bf16_vs_reference_sdpa(engine, T, I):
    """The block path's attention (bf16 q, k, v column views of the qkv buffer, bf16 out)
    against the reference's cudnn_sdpa_forward (cudnn_attention.cuh:408-443) on the same bf16
    values in its [24, L, 128] layout, at L = 1536 and 4608 with -inf on 400 of 512 text keys:
    the pair the bench's attention leg times."""
    ref = attn_ref_or_skip()
    H, D, L = 24, 128, T + I
    g = torch.Generator(device=DEV).manual_seed(11)
    qkv = torch.randn((L, 3, H, D), generator=g, device=DEV).to(torch.bfloat16)
    mask = torch.zeros(L, device=DEV)
    mask[T - 400:T] = float("-inf")
    flat = qkv.view(L, 3 * H * D)
    mine = engine.attention_bf16(flat[:, :H * D], flat[:, H * D:2 * H * D], flat[:, 2 * H * D:], H, D,
                                 attn_mask=mask, out_dtype=torch.bfloat16)
    q, k, v = (qkv[:, j].permute(1, 0, 2).contiguous() for j in range(3))
    o = torch.empty((H, L, D), dtype=torch.bfloat16, device=DEV)
    assert ref.sdpa_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), mask.data_ptr(), o.data_ptr(), H, L, D) == 0
    torch.cuda.synchronize()
    theirs = o.permute(1, 0, 2).reshape(L, H * D)
    a, b = mine.double().cpu().numpy().ravel(), theirs.double().cpu().numpy().ravel()
    # Both round O to bf16 (½ ulp = 2^-9 relative each); the softmax is fp32 in both.
    assert rel_err(a, b) < 1e-2
    assert a @ b / np.sqrt((a @ a) * (b @ b)) > 0.99999


@pytest.mark.parametrize("L,H,splits,batch", [(4608, 3, 0, 1), (4608, 3, 3, 1), (1536, 2, 2, 2), (640, 1, 0, 1)])
def test_attention_key_splits(engine, L, H, splits, batch):
    """Key-split attention (a launch too small to fill the GPU, e.g. a tensor-parallel rank's 3
    heads: slices of the key blocks in separate CTAs, merged by a second kernel; splits 0 =
    the automatic choice) against the one-pass kernel on the same bf16 inputs, bf16 and F32
    out, with a key mask, twice in a row."""
    D, T = 128, 512
    g = torch.Generator(device=DEV).manual_seed(17)
    qkv = torch.randn((batch * L, 3 * H * D), generator=g, device=DEV).to(torch.bfloat16)
    q, k, v = qkv[:, :H * D], qkv[:, H * D:2 * H * D], qkv[:, 2 * H * D:]
    mask = torch.zeros((batch, L), device=DEV)
    mask[:, min(T, L) - 100:min(T, L)] = float("-inf")
    mask = mask if batch > 1 else mask[0]
    run = (lambda dt: engine.attention_bf16_batched(q, k, v, H, D, batch, attn_mask=mask, out_dtype=dt)) \
        if batch > 1 else (lambda dt: engine.attention_bf16(q, k, v, H, D, attn_mask=mask, out_dtype=dt))
    # fp64 softmax(q k^T / sqrt(D) + mask) v per sequence and head
    want = torch.empty((batch * L, H * D), dtype=torch.float64, device=DEV)
    mrow = mask.view(batch, L).double()
    for z in range(batch):
        rows = slice(z * L, (z + 1) * L)
        for h in range(H):
            cols = slice(h * D, (h + 1) * D)
            sc = q[rows, cols].double() @ k[rows, cols].double().t() / np.sqrt(D) + mrow[z][None, :]
            want[rows, cols] = torch.softmax(sc, dim=-1) @ v[rows, cols].double()
    b = want.cpu().numpy().ravel()
    try:
        engine.set_attention_splits(-1)
        one_pass = run(torch.float32).double().cpu().numpy().ravel()
        engine.set_attention_splits(splits)
        for _ in range(2):
            for dt in (torch.float32, torch.bfloat16):
                got = run(dt)
                torch.cuda.synchronize()
                a = got.double().cpu().numpy().ravel()
                # P is rounded to bf16 against each slice's own running max, so the slices' sums
                # differ from the one-pass kernel's at bf16 precision; both are held to the fp64
                # result by the block-path attention tolerance.
                assert rel_err(a, b) < 1e-2
                assert a @ b / np.sqrt((a @ a) * (b @ b)) > 0.9999
                assert rel_err(a, one_pass) < 1e-2
    finally:
        engine.set_attention_splits(0)
    engine.check_device_error()


@pytest.mark.parametrize("case", ["middle_blocks", "one_key_live", "per_sequence"])
@pytest.mark.parametrize("splits", [-1, 2])
def test_attention_skips_masked_key_blocks(engine, case, splits):
    """Key blocks whose 128 keys are all -inf are skipped (no loads, MMAs or softmax): the
    result must equal softmax(q k^T / sqrt(D) + mask) v in fp64 where whole blocks, all but
    one key, or different blocks per stacked sequence are masked; one pass and key-split."""
    H, D, L = 4, 128, 1536
    batch = 2 if case == "per_sequence" else 1
    g = torch.Generator(device=DEV).manual_seed(23)
    qkv = torch.randn((batch * L, 3 * H * D), generator=g, device=DEV).to(torch.bfloat16)
    q, k, v = qkv[:, :H * D], qkv[:, H * D:2 * H * D], qkv[:, 2 * H * D:]
    mask = torch.zeros((batch, L), device=DEV)
    if case == "middle_blocks":
        mask[0, 100:1400] = float("-inf")        # blocks 1..9 dead, 0 and 10 partly live
    elif case == "one_key_live":
        mask[0, :] = float("-inf")
        mask[0, 700] = 0.0                        # one live block holding one live key
    else:
        mask[0, 256:1024] = float("-inf")
        mask[1, :512] = float("-inf")
        mask[1, 1280:] = float("-inf")
    want = torch.empty((batch * L, H * D), dtype=torch.float64, device=DEV)
    for z in range(batch):
        rows = slice(z * L, (z + 1) * L)
        for h in range(H):
            cols = slice(h * D, (h + 1) * D)
            sc = q[rows, cols].double() @ k[rows, cols].double().t() / np.sqrt(D) + mask[z].double()[None, :]
            want[rows, cols] = torch.softmax(sc, dim=-1) @ v[rows, cols].double()
    b = want.cpu().numpy().ravel()
    try:
        engine.set_attention_splits(splits)
        for dt in (torch.float32, torch.bfloat16):
            if batch > 1:
                got = engine.attention_bf16_batched(q, k, v, H, D, batch, attn_mask=mask, out_dtype=dt)
            else:
                got = engine.attention_bf16(q, k, v, H, D, attn_mask=mask[0], out_dtype=dt)
            torch.cuda.synchronize()
            a = got.double().cpu().numpy().ravel()
            assert rel_err(a, b) < 1e-2
            assert a @ b / np.sqrt((a @ a) * (b @ b)) > 0.9999
    finally:
        engine.set_attention_splits(0)
    engine.check_device_error()


def test_nerf_block_gemms_vs_reference(engine, ref):
    """One NeRF GLU block's GEMMs at 512^2 (chroma.cuh:1262-1302) at their real sizes, engine
    against the reference's own linear() and batched_matmul_Bt on the same inputs: param_gen
    (F32 s [1024, 3072] x bf16 W [49152, 3072]^T + bias), then the gate, value and fc2 batched
    products over 1024 patches."""
    g = torch.Generator(device=DEV).manual_seed(17)
    P = 1024
    s = torch.randn((P, 3072), generator=g, device=DEV)
    w = (torch.randn((49152, 3072), generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    b = torch.randn(49152, generator=g, device=DEV) * 0.02
    mine, theirs = torch.empty((P, 49152), device=DEV), torch.empty((P, 49152), device=DEV)
    engine.linear(s, w, b, mine)
    ref.linear(s.data_ptr(), 0, w.data_ptr(), 2, b.data_ptr(), theirs.data_ptr(), P, 3072, 49152)
    torch.cuda.synchronize()
    assert rel_err(mine.cpu().numpy(), theirs.cpu().numpy()) <= TOL_F32_OUT
    x = torch.randn((P, 256, 64), generator=g, device=DEV)
    wg = torch.randn((P, 256, 64), generator=g, device=DEV) * 0.125
    w2 = torch.randn((P, 64, 256), generator=g, device=DEV) * 0.0625
    for a, bb, n in ((x, wg, 256), (torch.randn((P, 256, 256), generator=g, device=DEV), w2, 64)):
        c_mine = torch.empty((P, a.shape[1], n), device=DEV)
        c_ref = torch.empty((P, a.shape[1], n), device=DEV)
        engine.batched_matmul_Bt(a, bb, c_mine)
        ref.batched_matmul_Bt(a.data_ptr(), bb.data_ptr(), c_ref.data_ptr(), P, a.shape[1], a.shape[2], n)
        torch.cuda.synchronize()
        assert rel_err(c_mine.cpu().numpy(), c_ref.cpu().numpy()) <= TOL_F32_OUT
    engine.check_device_error()
