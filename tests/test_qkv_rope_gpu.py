"""The block's attention input path: the qkv GEMM with qk_norm and RoPE in its epilogue
(b2g_gemm_qkv_rope, bf16 [q | k | v] out) and the fused attention reading that buffer
(b2g_attention_bf16), against the oracle's linear, rms_norm, rope and attention on the same
seeded inputs.

Tolerances: the epilogue's output is bf16, so each element may differ from the fp32 oracle by
half a bf16 ulp (2^-8 relative) plus fp32 rounding noise; attention as in the other attention
tests (max|d|/max|ref| < 1e-2 against the oracle, which rounds P and O to bf16 as cuDNN does).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
DH = 128


def bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def pe_table(L: int, D: int, seed: int) -> np.ndarray:
    g = np.random.default_rng(seed)
    ang = g.uniform(0, 2 * np.pi, (L, D // 2))
    return np.stack([np.cos(ang), -np.sin(ang), np.sin(ang), np.cos(ang)], -1).astype(np.float32)


def identity_pe(L: int, D: int) -> np.ndarray:
    pe = np.zeros((L, D // 2, 4), np.float32)
    pe[..., 0] = 1.0
    pe[..., 3] = 1.0
    return pe


def qkv_oracle(oracle, x, w, bias, pe, H, qn, kn):
    """linear -> per-head rms_norm (when a scale is given) -> rope on q and k; v plain."""
    y = oracle.linear(bits(x), 2, bits(w), 2, bias.cpu().numpy())
    HD = H * DH

    def nr(a, s):
        a = np.ascontiguousarray(a)
        if s is not None:
            a = oracle.rms_norm(a.reshape(-1, DH), s.cpu().numpy()).reshape(a.shape)
        return oracle.rope(a, pe, H)

    return np.concatenate([nr(y[:, :HD], qn), nr(y[:, HD:2 * HD], kn), y[:, 2 * HD:]], 1)


def assert_bf16_of(got: torch.Tensor, want: np.ndarray):
    g = got.float().cpu().numpy().astype(np.float64)
    w = want.astype(np.float64)
    assert np.isfinite(g).all()
    slack = 2.0 ** -8 * np.abs(w) + 1e-5 * np.abs(w).max()
    bad = np.abs(g - w) > slack
    assert not bad.any(), f"{bad.sum()} elements off, worst {np.abs(g - w).max():.3e}"


def seeded(shape, seed, scale=1.0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


@pytest.mark.parametrize("M0,M1,H,K,norms,variant", [(40, 200, 2, 256, True, -1), (333, 0, 3, 200, False, -1),
                                                      (130, 260, 2, 320, True, 1), (64, 64, 4, 128, True, 0)])
def test_gemm_qkv_rope_vs_oracle(engine, oracle, M0, M1, H, K, norms, variant):
    """Two problems (txt rows take pe rows [0, M0), img rows [M0, M0+M1)) in one launch, their
    own norm scales; ragged M, K not a multiple of 64, H*128 not a multiple of the 256-column
    tile (a tile then spans two sections), no norm; every kernel variant (the 128-column one
    is promoted to 256 columns)."""
    N = 3 * H * DH
    L = M0 + M1
    pe = pe_table(L, DH, L + K)
    pe_d = torch.from_numpy(pe).to(DEV)
    probs, wants = [], []
    for i, (m, r0) in enumerate(((M0, 0), (M1, M0))):
        if m == 0:
            continue
        x = seeded((m, K), 10 * i + 1)
        w = seeded((N, K), 10 * i + 2, 0.05)
        b = seeded((N,), 10 * i + 3, 0.05, torch.float32)
        qn = (1 + 0.2 * seeded((DH,), 10 * i + 4, 1.0, torch.float32)) if norms else None
        kn = (1 + 0.2 * seeded((DH,), 10 * i + 5, 1.0, torch.float32)) if norms else None
        probs.append(dict(x=x.to(DEV), w=w.to(DEV), bias=b.to(DEV), pe=pe_d[r0:r0 + m],
                          q_norm=qn.to(DEV) if norms else None, k_norm=kn.to(DEV) if norms else None))
        wants.append(qkv_oracle(oracle, x, w, b, pe[r0:r0 + m], H, qn, kn))
    engine.set_gemm_variant(variant)
    try:
        outs = engine.gemm_qkv_rope(probs, H)
        torch.cuda.synchronize()
    finally:
        engine.set_gemm_variant(-1)
    for got, want in zip(outs, wants):
        assert got.dtype == torch.bfloat16 and got.shape == want.shape
        assert_bf16_of(got, want)


def test_gemm_qkv_rope_config2_shape(engine):
    """The double block's qkv layer at 512^2 (txt 512 + img 1024 rows, 24 heads, K 3072) into
    row views of one [1536, 9216] buffer, against a float64 torch restatement on the GPU."""
    T, I, H, K = 512, 1024, 24, 3072
    N = 3 * H * DH
    L = T + I
    pe = torch.from_numpy(pe_table(L, DH, 11)).to(DEV)
    buf = torch.zeros((L, N), dtype=torch.bfloat16, device=DEV)
    probs, refs = [], []
    for i, (m, r0) in enumerate(((T, 0), (I, T))):
        x = seeded((m, K), 50 + i).to(DEV)
        w = seeded((N, K), 60 + i, 0.02).to(DEV)
        b = seeded((N,), 70 + i, 0.02, torch.float32).to(DEV)
        qn = (1 + 0.2 * seeded((DH,), 80 + i, 1.0, torch.float32)).to(DEV)
        kn = (1 + 0.2 * seeded((DH,), 90 + i, 1.0, torch.float32)).to(DEV)
        probs.append(dict(x=x, w=w, bias=b, out=buf[r0:r0 + m], pe=pe[r0:r0 + m], q_norm=qn, k_norm=kn))
        y = (x.double() @ w.double().t() + b.double()).reshape(m, 3, H, DH)
        p = pe[r0:r0 + m].double().reshape(m, 1, DH // 2, 4)

        def nr(a, s):
            a = a * torch.rsqrt((a * a).mean(-1, keepdim=True) + 1e-6) * s.double()
            e, o = a[..., 0::2], a[..., 1::2]
            return torch.stack([e * p[..., 0] + o * p[..., 1], e * p[..., 2] + o * p[..., 3]], -1).reshape(m, H, DH)

        refs.append(torch.stack([nr(y[:, 0], qn), nr(y[:, 1], kn), y[:, 2]], 1).reshape(m, N))
    engine.gemm_qkv_rope(probs, H)
    torch.cuda.synchronize()
    want = torch.cat(refs).cpu().numpy()
    assert_bf16_of(buf, want)


def test_gemm_qkv_rope_rejects_bad_arguments(engine):
    x = torch.zeros((8, 64), dtype=torch.bfloat16, device=DEV)
    w = torch.zeros((3 * 2 * DH, 64), dtype=torch.bfloat16, device=DEV)
    pe = torch.zeros((8, 64, 4), device=DEV)
    with pytest.raises(engine.B2GError):
        engine.gemm_qkv_rope([dict(x=x, w=w, pe=pe)], 3)   # N != 3 * n_head * 128
    with pytest.raises(engine.B2GError):
        engine.gemm_qkv_rope([dict(x=x, w=w, pe=pe, out=torch.zeros((8, 768), device=DEV))], 2)  # F32 out


@pytest.mark.parametrize("L,H,D,mask_kind,out_bf16", [(131, 2, 128, "pad", False), (256, 3, 64, "none", True),
                                                       (300, 2, 128, "general", False), (1, 1, 64, "none", False)])
def test_attention_bf16_vs_oracle(engine, oracle, L, H, D, mask_kind, out_bf16):
    """q, k, v as column sections of one bf16 [L, 3*H*D] buffer (row stride 3*H*D); L not a
    multiple of 8 or of the 128-key block; padding mask, general bias with -inf keys, none;
    output into a column view of a wider buffer."""
    HD = H * D
    qkv = seeded((L, 3 * HD), L + D, 1.0)
    mask = np.zeros(L, np.float32)
    if mask_kind == "pad":
        mask[L // 3:L // 3 + 21] = -np.inf
    elif mask_kind == "general":
        mask = (np.random.default_rng(L).standard_normal(L) * 2.0).astype(np.float32)
        mask[5:17] = -np.inf
    dq = qkv.to(DEV)
    out_w = torch.zeros((L, HD + 16), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=DEV)
    m = torch.from_numpy(mask).to(DEV) if mask_kind != "none" else None
    engine.attention_bf16(dq[:, :HD], dq[:, HD:2 * HD], dq[:, 2 * HD:], H, D, attn_mask=m, out=out_w[:, 8:8 + HD])
    torch.cuda.synchronize()
    f = qkv.float().numpy()
    want = oracle.attention_rope(f[:, :HD].reshape(L, H, D), f[:, HD:2 * HD].reshape(L, H, D),
                                 f[:, 2 * HD:].reshape(L, H, D), identity_pe(L, D),
                                 mask if mask_kind != "none" else None)
    got_w = out_w.float().cpu().numpy()
    assert np.all(got_w[:, :8] == 0) and np.all(got_w[:, 8 + HD:] == 0)
    got = got_w[:, 8:8 + HD]
    assert np.isfinite(got).all()
    assert rel_err(got, want) < 1e-2


def test_fused_path_matches_the_separate_one(engine):
    """The block's new path (qkv GEMM with norm + RoPE epilogue, attention on bf16) against the
    engine's separate path (F32 qkv GEMM, attention_qknorm_rope prologue + the same kernel) at
    config-2 size: both round q, k, v to bf16 once, so they agree to bf16 rounding of inputs."""
    T, I, H, K = 512, 1024, 24, 3072
    HD, N, L = H * DH, 3 * H * DH, T + I
    pe = torch.from_numpy(pe_table(L, DH, 5)).to(DEV)
    mask = torch.zeros(L, device=DEV)
    mask[100:512] = float("-inf")
    xs = [seeded((m, K), 100 + i).to(DEV) for i, m in enumerate((T, I))]
    ws = [seeded((N, K), 110 + i, 0.02).to(DEV) for i in range(2)]
    bs = [seeded((N,), 120 + i, 0.02, torch.float32).to(DEV) for i in range(2)]
    ns = [(1 + 0.2 * seeded((DH,), 130 + i, 1.0, torch.float32)).to(DEV) for i in range(4)]
    buf = torch.empty((L, N), dtype=torch.bfloat16, device=DEV)
    engine.gemm_qkv_rope([dict(x=xs[0], w=ws[0], bias=bs[0], out=buf[:T], pe=pe[:T], q_norm=ns[0], k_norm=ns[1]),
                          dict(x=xs[1], w=ws[1], bias=bs[1], out=buf[T:], pe=pe[T:], q_norm=ns[2], k_norm=ns[3])], H)
    fused = engine.attention_bf16(buf[:, :HD], buf[:, HD:2 * HD], buf[:, 2 * HD:], H, DH, attn_mask=mask)
    f32 = torch.empty((L, N), device=DEV)
    engine.gemm(xs[0], ws[0], bs[0], out=f32[:T])
    engine.gemm(xs[1], ws[1], bs[1], out=f32[T:])
    sep = engine.attention_qknorm_rope(f32[:, :HD], f32[:, HD:2 * HD], f32[:, 2 * HD:], pe, H, DH, q_norm=ns[0],
                                       k_norm=ns[1], q_norm2=ns[2], k_norm2=ns[3], norm_split=T, attn_mask=mask)
    torch.cuda.synchronize()
    a, b = fused.double().cpu().numpy().ravel(), sep.double().cpu().numpy().ravel()
    assert rel_err(a, b) < 1e-2
    assert a @ b / np.sqrt((a @ a) * (b @ b)) > 0.9999


@pytest.mark.parametrize("M,H,MLPC,K", [(200, 2, 512, 256), (131, 2, 200, 192)])
def test_gemm_qkv_rope_with_gelu_tail(engine, oracle, M, H, MLPC, K):
    """The single block's linear1 in one launch: weight rows [q | k | v | mlp]; the qkv columns
    come out normed and rotated, the MLP columns as bias + tanh-GELU (bf16) in a column view of
    a wider concat buffer, nothing written outside it."""
    QKV = 3 * H * DH
    N = QKV + MLPC
    x = seeded((M, K), 5)
    w = seeded((N, K), 6, 0.05)
    b = seeded((N,), 7, 0.05, torch.float32)
    qn = 1 + 0.2 * seeded((DH,), 8, 1.0, torch.float32)
    kn = 1 + 0.2 * seeded((DH,), 9, 1.0, torch.float32)
    pe = pe_table(M, DH, 17)
    cat = torch.zeros((M, 64 + MLPC + 40), dtype=torch.bfloat16, device=DEV)
    outs = engine.gemm_qkv_rope([dict(x=x.to(DEV), w=w.to(DEV), bias=b.to(DEV), pe=torch.from_numpy(pe).to(DEV),
                                      q_norm=qn.to(DEV), k_norm=kn.to(DEV), gelu_out=cat[:, 64:64 + MLPC])], H)
    torch.cuda.synchronize()
    want_qkv = qkv_oracle(oracle, x, w[:QKV], b[:QKV], pe, H, qn, kn)
    assert outs[0].shape == (M, QKV)
    assert_bf16_of(outs[0], want_qkv)
    y = oracle.linear(bits(x), 2, bits(w[QKV:]), 2, b[QKV:].numpy())
    want_mlp = oracle.gelu(y)
    got = cat.float().cpu().numpy()
    assert np.all(got[:, :64] == 0) and np.all(got[:, 64 + MLPC:] == 0)
    assert_bf16_of(cat[:, 64:64 + MLPC], want_mlp)


@pytest.mark.parametrize("L,H,K,halves", [(200, 2, 256, 2), (131, 2, 192, 3)])
def test_gemm_qkv_rope_pe_period(engine, oracle, L, H, K, halves):
    """Guidance halves stacked in one problem (the single block's linear1 under forward_cfg):
    row r is rotated by pe row r % L, with pe holding L rows only; a GELU tail as well."""
    QKV, MLPC = 3 * H * DH, 192
    N = QKV + MLPC
    M = halves * L
    x = seeded((M, K), 21)
    w = seeded((N, K), 22, 0.05)
    b = seeded((N,), 23, 0.05, torch.float32)
    qn = 1 + 0.2 * seeded((DH,), 24, 1.0, torch.float32)
    kn = 1 + 0.2 * seeded((DH,), 25, 1.0, torch.float32)
    pe = pe_table(L, DH, 29)
    tail = torch.zeros((M, MLPC), dtype=torch.bfloat16, device=DEV)
    outs = engine.gemm_qkv_rope([dict(x=x.to(DEV), w=w.to(DEV), bias=b.to(DEV), pe=torch.from_numpy(pe).to(DEV),
                                      pe_period=L, q_norm=qn.to(DEV), k_norm=kn.to(DEV), gelu_out=tail)], H)
    torch.cuda.synchronize()
    want = qkv_oracle(oracle, x, w[:QKV], b[:QKV], np.concatenate([pe] * halves), H, qn, kn)
    assert_bf16_of(outs[0], want)
    y = oracle.linear(bits(x), 2, bits(w[QKV:]), 2, b[QKV:].numpy())
    assert_bf16_of(tail, oracle.gelu(y))


def test_gemm_qkv_rope_four_problems(engine, oracle):
    """The double block's qkv layer with guidance halves: txt_c, txt_u (txt weights, pe rows
    [0, T)), img_c, img_u (img weights, pe rows [T, L)) in one launch into the half-major
    [L_c | L_u] rows of one buffer."""
    T, I, H, K = 70, 130, 2, 192
    N, L = 3 * H * DH, T + I
    pe = pe_table(L, DH, 31)
    pe_d = torch.from_numpy(pe).to(DEV)
    buf = torch.zeros((2 * L, N), dtype=torch.bfloat16, device=DEV)
    ws = [seeded((N, K), 32 + j, 0.05) for j in range(2)]
    bs = [seeded((N,), 34 + j, 0.05, torch.float32) for j in range(2)]
    ns = [1 + 0.2 * seeded((DH,), 36 + j, 1.0, torch.float32) for j in range(4)]
    probs, wants = [], []
    for j, (m, p0) in enumerate(((T, 0), (I, T))):          # stream: txt, img
        for h in range(2):                                   # guidance half
            x = seeded((m, K), 40 + 2 * j + h)
            r0 = h * L + p0
            probs.append(dict(x=x.to(DEV), w=ws[j].to(DEV), bias=bs[j].to(DEV), out=buf[r0:r0 + m],
                              pe=pe_d[p0:p0 + m], q_norm=ns[2 * j].to(DEV), k_norm=ns[2 * j + 1].to(DEV)))
            wants.append((r0, m, qkv_oracle(oracle, x, ws[j], bs[j], pe[p0:p0 + m], H, ns[2 * j], ns[2 * j + 1])))
    n0 = engine.launch_count()
    engine.gemm_qkv_rope(probs, H)
    torch.cuda.synchronize()
    assert engine.launch_count() - n0 == 1
    for r0, m, want in wants:
        assert_bf16_of(buf[r0:r0 + m], want)


def rope_oracle_from(oracle, y, pe, H, qn, kn):
    """norm + rope on q and k of an already computed [M, 3*H*128] projection."""
    HD = H * DH

    def nr(a, sc):
        a = np.ascontiguousarray(a)
        if sc is not None:
            a = oracle.rms_norm(a.reshape(-1, DH), sc.cpu().numpy()).reshape(a.shape)
        return oracle.rope(a, pe, H)

    return np.concatenate([nr(y[:, :HD], qn), nr(y[:, HD:2 * HD], kn), y[:, 2 * HD:]], 1)


@pytest.mark.parametrize("tail,halves", [(False, 1), (True, 2)])
def test_gemm_qkv_rope_fp8_vs_oracle(engine, oracle, tail, halves):
    """The E4M3 form (config 5's qkv / linear1): per-token E4M3 x and per-channel E4M3 w, the
    accumulator scaled by both before the bias, then norm + RoPE, against the oracle's
    exact-product E4M3 GEMM on the same codes; with two problems in one launch, or one problem
    with a GELU tail over two stacked guidance halves (pe_period)."""
    H, K, L = 2, 320, 150
    QKV = 3 * H * DH
    MLPC = 256 if tail else 0
    N = QKV + MLPC
    pe = pe_table(L, DH, 41)
    pe_d = torch.from_numpy(pe).to(DEV)
    qn = (1 + 0.2 * seeded((DH,), 42, 1.0, torch.float32)).to(DEV)
    kn = (1 + 0.2 * seeded((DH,), 43, 1.0, torch.float32)).to(DEV)
    specs = [(halves * L, 0)] if tail else [(70, 0), (L - 70, 70)]
    probs, wants = [], []
    for i, (m, r0) in enumerate(specs):
        x = seeded((m, K), 50 + i, 1.0, torch.float32).to(DEV)
        w = seeded((N, K), 60 + i, 0.05).to(DEV)
        b = seeded((N,), 70 + i, 0.05, torch.float32).to(DEV)
        xq, xs = engine.quantize_e4m3(x)
        wq, ws = engine.quantize_e4m3(w)
        pr = dict(x=xq, x_scale=xs, w=wq, w_scale=ws, bias=b, q_norm=qn, k_norm=kn)
        if tail:
            pr.update(pe=pe_d, pe_period=L, gelu_out=torch.zeros((m, MLPC), dtype=torch.bfloat16, device=DEV))
            rows_pe = np.concatenate([pe] * halves)
        else:
            pr.update(pe=pe_d[r0:r0 + m])
            rows_pe = pe[r0:r0 + m]
        y = oracle.gemm_fp8(xq.cpu().numpy(), xs.cpu().numpy(), wq.cpu().numpy(), ws.cpu().numpy(), b.cpu().numpy())
        probs.append(pr)
        wants.append((rope_oracle_from(oracle, np.ascontiguousarray(y[:, :QKV]), rows_pe, H, qn, kn),
                      oracle.gelu(np.ascontiguousarray(y[:, QKV:])) if tail else None))
    n0 = engine.launch_count()
    outs = engine.gemm_qkv_rope(probs, H)
    torch.cuda.synchronize()
    assert engine.launch_count() - n0 == 1
    for pr, out, (want, want_tail) in zip(probs, outs, wants):
        assert_bf16_of(out, want)
        if tail:
            assert_bf16_of(pr["gelu_out"], want_tail)
    engine.check_device_error()


@pytest.mark.parametrize("L,batch,shared_mask,out_bf16", [(200, 2, False, True), (131, 3, True, False),
                                                           (1536, 2, False, True)])
def test_attention_bf16_batched_equals_one_call_per_sequence(engine, L, batch, shared_mask, out_bf16):
    """Sequences stacked in the rows of one [batch*L, 3*H*D] buffer (the guidance halves of
    forward_cfg, half-major) in one launch: bit-identical to one attention_bf16 call per
    sequence, including L not a multiple of the 128-key block (the last key block of a
    sequence overlaps the next one's rows, which its mask must exclude) and a bias per
    sequence or one shared bias."""
    H, D = 2, 128
    HD = H * D
    qkv = seeded((batch * L, 3 * HD), L + batch, 1.0).to(DEV)
    g = torch.Generator().manual_seed(batch)
    if shared_mask:
        mask = torch.zeros(L)
        mask[3:40] = float("-inf")
    else:
        mask = torch.randn((batch, L), generator=g) * 2.0
        mask[:, 5:17] = float("-inf")
        mask[1, 20:L // 2] = float("-inf")
    mask = mask.contiguous().to(DEV)
    dt = torch.bfloat16 if out_bf16 else torch.float32
    got = torch.zeros((batch * L, HD), dtype=dt, device=DEV)
    engine.attention_bf16_batched(qkv[:, :HD], qkv[:, HD:2 * HD], qkv[:, 2 * HD:], H, D, batch, attn_mask=mask,
                                  out=got)
    want = torch.zeros_like(got)
    for b in range(batch):
        r = slice(b * L, (b + 1) * L)
        engine.attention_bf16(qkv[r, :HD], qkv[r, HD:2 * HD], qkv[r, 2 * HD:], H, D,
                              attn_mask=mask if shared_mask else mask[b], out=want[r])
    torch.cuda.synchronize()
    assert torch.isfinite(got.float()).all()
    assert torch.equal(got, want)
    engine.check_device_error()


@pytest.mark.parametrize("fp8,tail", [(False, False), (True, False), (False, True)])
def test_gemm_qkv_rope_compact_table_equals_full(engine, fp8, tail):
    """The compact (cos, sin) RoPE table gives the same outputs as the reference's [64][4]
    table it was made from: bf16 and E4M3 operands, two problems, and one problem over two
    stacked sequences (pe_period) with a GELU tail."""
    H, K = 2, 256
    QKV = 3 * H * DH
    N = QKV + (192 if tail else 0)
    pe = torch.from_numpy(pe_table(160, DH, 51)).to(DEV)
    pe_c = engine.compact_rope_table(pe)
    assert pe_c is not None
    qn = (1 + 0.2 * seeded((DH,), 52, 1.0, torch.float32)).to(DEV)
    kn = (1 + 0.2 * seeded((DH,), 53, 1.0, torch.float32)).to(DEV)
    specs = [(320, 0, 160)] if tail else [(60, 0, 0), (100, 60, 0)]
    results = []
    for table in (pe, pe_c):
        probs = []
        for i, (m, r0, period) in enumerate(specs):
            x = seeded((m, K), 60 + i).to(DEV)
            w = seeded((N, K), 70 + i, 0.05).to(DEV)
            b = seeded((N,), 80 + i, 0.05, torch.float32).to(DEV)
            pr = dict(x=x, w=w, bias=b, q_norm=qn, k_norm=kn, pe=table if period else table[r0:r0 + m],
                      pe_period=period)
            if fp8:
                xq, xs = engine.quantize_e4m3(x)
                wq, wsc = engine.quantize_e4m3(w)
                pr.update(x=xq, x_scale=xs, w=wq, w_scale=wsc)
            if tail:
                pr["gelu_out"] = torch.zeros((m, N - QKV), dtype=torch.bfloat16, device=DEV)
            probs.append(pr)
        outs = engine.gemm_qkv_rope(probs, H)
        torch.cuda.synchronize()
        results.append([o.clone() for o in outs] + [p["gelu_out"].clone() for p in probs if "gelu_out" in p])
    for full, comp in zip(*results):
        assert torch.equal(full, comp)
    engine.check_device_error()


def test_attention_bf16_batched_rejects_bad_arguments(engine):
    """Rows that are not whole sequences, and a mask whose rows do not match the batch, are
    errors rather than silent reads past a sequence."""
    H, D = 2, 128
    qkv = torch.zeros((10, 3 * H * D), dtype=torch.bfloat16, device=DEV)
    q, k, v = qkv[:, :H * D], qkv[:, H * D:2 * H * D], qkv[:, 2 * H * D:]
    with pytest.raises(engine.B2GError):
        engine.attention_bf16_batched(q, k, v, H, D, 3)                    # 10 rows, 3 sequences
    with pytest.raises(engine.B2GError):
        engine.attention_bf16_batched(q, k, v, H, D, 2, attn_mask=torch.zeros((3, 5), device=DEV))
    out = engine.attention_bf16_batched(q, k, v, H, D, 2, attn_mask=torch.zeros((2, 5), device=DEV))
    torch.cuda.synchronize()
    assert out.shape == (10, H * D) and torch.isfinite(out).all()
