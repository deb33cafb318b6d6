"""The whole denoising step, ChromaRadiance::forward_cfg (chroma.cuh:1499-1584) at 512^2 with
classifier-free guidance: img_in conv, txt_in, the approximator, 19 double + 38 single
blocks, two NeRF decodes and cfg_blend, on seeded random-init weights (the reference's own
Tensor fields, filled by its Philox generator).

The reference (oracle/_ref/libref_model.so: its cuBLASLt, cuDNN and cuBLAS code) is the
checker.  Under test:
  * the reference's model code built through the drop-in headers (every GEMM and attention
    in libb2g.so), on bit-identical weights from its own copy of the generator;
Tolerance: the north star's full-forward bar, cosine >= 0.999 of the velocity, and
max|d|/max|ref| <= 5e-2 (bf16 operands at different rounding points through 57 blocks)."""
from __future__ import annotations

import pytest
import torch

from conftest import REPO

import harness

pytestmark = pytest.mark.gpu
STOCK = REPO / "oracle" / "_ref" / "libref_model.so"
SEED, H, W = 42, 512, 512
REAL_COND, REAL_UNCOND = 111, 1       # 112 and 2 text keys attend (one padding token each)
TIMESTEP, CFG = 0.7, 4.0


def compare(got, want) -> tuple[float, float]:
    g, w = got.double().flatten(), want.double().flatten()
    cos = float((g @ w) / (g.norm() * w.norm()))
    rel = float((g - w).abs().max() / w.abs().max())
    return cos, rel


@pytest.fixture(scope="module")
def stock():
    if not STOCK.exists():
        pytest.skip("oracle/_ref/libref_model.so not built (needs the reference sources at build time)")
    h = harness.ForwardCfgHarness(STOCK)
    h.setup(SEED, H, W, REAL_COND, REAL_UNCOND)
    h.forward(TIMESTEP, CFG)
    return h


def test_dropin_forward_cfg_matches_stock(stock):
    if not harness.DROPIN_PATH.exists():
        pytest.skip("drop-in harness not built (needs the reference sources at build time)")
    d = harness.ForwardCfgHarness(harness.DROPIN_PATH)
    d.setup(SEED, H, W, REAL_COND, REAL_UNCOND)
    for name in ("double_blocks.7.img_attn.qkv.weight", "nerf_blocks.2.param_generator.bias", "x", "pe"):
        assert torch.equal(d.tensor(name), stock.tensor(name)), name   # the same seeded inputs
    d.forward(TIMESTEP, CFG)
    torch.cuda.synchronize()
    want, got = stock.tensor("velocity"), d.tensor("velocity")
    assert torch.isfinite(got).all()
    cos, rel = compare(got, want)
    print(f"drop-in forward_cfg vs stock: cosine {cos:.6f}, max|d|/max|ref| {rel:.3e}")
    assert cos >= 0.999 and rel <= 5e-2


# ---------------------------------------------------------------------------- the engine's own model
@pytest.fixture(scope="module")
def engine_model(stock, engine):
    """The engine's ChromaRadiance on the reference model's own weight buffers (views)."""
    import model

    w = {name: stock.tensor(name) for name in model.weight_specs()}
    m = model.ChromaRadiance(w, "cuda")
    s = model.ForwardScratch(H, W, "cuda")
    return m, s


def test_host_tables_match_reference(stock):
    """model.rope_table / dct_features / key_masks restate RoPE::gen_pe, compute_dct_features and
    the key masks main.cu builds; the harness holds the reference's own."""
    import model

    pe = torch.from_numpy(model.rope_table(H, W)).cuda().flatten()
    assert (pe - stock.tensor("pe")).abs().max().item() <= 2e-6
    dct = torch.from_numpy(model.dct_features()).cuda().flatten()
    assert (dct - stock.tensor("dct")).abs().max().item() <= 2e-6
    masks = torch.from_numpy(model.key_masks([REAL_COND, REAL_UNCOND], H, W)).cuda()
    assert torch.equal(masks[0], stock.tensor("mask_cond")) and torch.equal(masks[1], stock.tensor("mask_uncond"))


def test_modulation_matches_reference(stock, engine_model):
    m, s = engine_model
    stock.modulation(TIMESTEP)
    s.timestep.fill_(TIMESTEP)
    got = m.compute_modulation(s)
    torch.cuda.synchronize()
    cos, rel = compare(got, stock.tensor("mod"))
    print(f"approximator vs reference: cosine {cos:.8f}, max|d|/max|ref| {rel:.3e}")
    assert cos >= 0.99999 and rel <= 5e-3


def test_nerf_decode_matches_reference(stock, engine_model):
    """One half's decode of the same transformer image rows (random rows here), no blend."""
    import b2g
    import model

    m, s = engine_model
    img = torch.randn((s.P, model.HIDDEN), generator=torch.Generator(device="cuda").manual_seed(3), device="cuda")
    want = torch.empty((3 * H * W,), device="cuda")
    stock.nerf_decode(img, want)
    s.x[s.T:s.L].copy_(img)
    s.x[s.L + s.T:].copy_(img)
    m.nerf_decode(s, stock.tensor("x").view(1, 3, H, W), stock.tensor("dct").view(256, 64))
    got = torch.empty((3, H, W), device="cuda")
    b2g.nerf_final(s.nx[0], None, m.final_norm, m.conv_w, m.conv_b, 1.0, H, W, got)
    torch.cuda.synchronize()
    cos, rel = compare(got, want)
    print(f"nerf_decode vs reference: cosine {cos:.8f}, max|d|/max|ref| {rel:.3e}")
    assert cos >= 0.9999 and rel <= 2e-2


def _engine_inputs(stock):
    import model

    L = 512 + (H // 16) * (W // 16)
    return (stock.tensor("x").view(1, 3, H, W), stock.tensor("context_cond").view(512, 4096),
            stock.tensor("context_uncond").view(512, 4096), stock.tensor("pe").view(L, 256),
            stock.tensor("dct").view(256, 64), torch.stack([stock.tensor("mask_cond"), stock.tensor("mask_uncond")]))


def test_engine_forward_cfg_matches_reference(stock, engine_model):
    """The north star's full-forward bar: the engine's whole step against the reference's
    forward_cfg on the same weights and inputs, velocity cosine >= 0.999."""
    m, s = engine_model
    s.timestep.fill_(TIMESTEP)
    v = m.forward_cfg(s, *_engine_inputs(stock), CFG)
    torch.cuda.synchronize()
    import b2g

    b2g.check_device_error()
    assert torch.isfinite(v).all()
    cos, rel = compare(v, stock.tensor("velocity"))
    print(f"engine forward_cfg vs reference: cosine {cos:.6f}, max|d|/max|ref| {rel:.3e}")
    assert cos >= 0.999 and rel <= 5e-2


def test_engine_forward_cfg_graph_equals_eager(stock, engine_model):
    """The step captured in one CUDA graph and replayed gives the eager step's velocity exactly
    (the timestep is read from device memory, so the graph also serves other timesteps)."""
    m, s = engine_model
    args = _engine_inputs(stock)
    s.timestep.fill_(TIMESTEP)
    eager = m.forward_cfg(s, *args, CFG).clone()
    side = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            m.forward_cfg(s, *args, CFG)
    s.velocity.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(s.velocity, eager)
    s.timestep.fill_(0.3)
    g.replay()
    torch.cuda.synchronize()
    assert not torch.equal(s.velocity, eager)
    del g
