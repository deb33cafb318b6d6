"""Benchmark of the B200 GEMM engine on BASELINE configs 2 and 1, plus the reference's own arm.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b2g|reference]
                    [--workload config2|config1]

config2 (default; the configuration the metric is quoted on): one "step" = one Chroma
double-stream block and one single-stream block at 512^2 (T=512 text + I=1024 image tokens,
hidden 3072, 24 heads x 128, MLP 12288): every GEMM of both blocks (txt/img qkv, proj, MLP
with GELU, linear1, linear2, with bias and gated residuals) and both attentions (qk-norm,
RoPE, QK^T and PV over 24 heads, 0/-inf key mask on 400 of the 512 text tokens).  Weights
~N(0,0.02) bf16, biases ~N(0,0.02), activations ~N(0,1), gates ~N(0,1), seeded.
  value     TFLOP/s over all ranks: (linear + unmasked attention FLOPs = 753.77 GFLOP per
            step) * steps * ranks / (max over ranks of the summed per-step CUDA-event time).
            The engine replays the step as two CUDA graphs; weights (680 MB) are larger than
            L2, and a 256 MB buffer is also written before every step, outside the events.
  roofline  dominant kernel = the engine's tcgen05 GEMM (the linear layers): GEMM FLOPs /
            summed GEMM launch time.  Per-launch times come from events recorded between the
            launches inside a second copy of the graphs, replayed after the timed steps, scaled
            so they sum to the timed step (the timed graphs carry no events between launches,
            so consecutive kernels overlap their set-up and tail; the events in the copy stop
            that overlap); peak = MEASURED_PEAKS.json bf16_tflops.
  e2e       the whole denoising step at 512^2 through the public API (
            model.ChromaRadiance.forward_cfg, chroma.cuh:1499-1584): img_in, txt_in, the
            approximator, 19 double + 38 single blocks over both guidance halves, two NeRF
            decodes and cfg_blend, as one CUDA graph; per step the noise, both T5 contexts and
            the timestep copied in from pinned host memory and the velocity copied back inside
            the events.  The reference arm times its own forward_cfg the same way.  Beside it,
            dropin_forward_cfg: the reference's forward_cfg built through the drop-in headers.
            e2e_block_pair is the timed block pair with all of its activations copied in and out
            every step (PCIe-bound, 104 MB per step).
  tp1024    config 4's block pair at 1024^2: unsharded on one GPU, tensor-parallel over N GPUs
            (speed-up over rank 0's unsharded time, per-operation split, on-box parity).
config1: one GEMM, the single-stream linear1 at 512^2 (M=1536 K=3072 N=21504, bias, bf16 out),
inputs from numpy PCG64 seed 0, identical for both arms.
cpu_baseline  the fp32 C oracle (oracle/oracle.c, OpenMP, all host cores) on a bounded row
            sample of the single-stream linear1 GEMM (rank 0, N=1 only).

--impl reference runs the reference's own code (its cuBLASLt linear / linear_lt, rms_norm,
cuDNN attention and elementwise kernels, compiled from its sources into oracle/_ref/) on the
same workload, timed the same way, and never imports the engine.  Multi-GPU (torchrun): every
rank runs its own replica (weak scaling, no collective on the data path); rank 0 prints.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "chroma-radiance_b200"))
sys.path.insert(0, str(REPO / "oracle"))

METRIC = json.loads((REPO / "BASELINE.json").read_text())["metric"]
M, K, N = 1536, 3072, 21504
FLOP = 2.0 * M * N * K
FLUSH_BYTES = 256 << 20
WORKLOAD = "config1: single-stream linear1 GEMM+bias, M=1536 K=3072 N=21504 (512^2: 1024 img + 512 txt tokens)"


def make_inputs(oracle_mod):
    """Seeded host inputs shared by both arms: bf16 bit patterns and an F32 bias."""
    o = oracle_mod.Oracle()
    rng = np.random.default_rng(0)
    x = o.to_bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    w = o.to_bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    bias = o.to_f32(o.to_bf16_bits(rng.standard_normal(N, dtype=np.float32) * np.float32(0.02)), 2)
    return o, x, w, bias


def measured_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


def profile_traffic(name: str) -> float | None:
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary, if any."""
    p = REPO / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip())
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every few ms in a thread."""

    REASONS = {
        "hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
        "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_baseline(o, x, w, bias) -> dict:
    """fp32 C oracle on all host cores: a bounded sample of the config-1 GEMM (~10 s)."""
    rows = 32
    t = time.perf_counter()
    o.linear(x[:rows], 2, w, 2, bias)
    dt = time.perf_counter() - t
    target = 10.0
    rows2 = int(min(M, max(rows, rows * target / max(dt, 1e-3))))
    t = time.perf_counter()
    o.linear(x[:rows2], 2, w, 2, bias)
    dt = time.perf_counter() - t
    return {"value": 2.0 * rows2 * N * K / dt / 1e12, "unit": "TFLOP/s", "cores": o.num_threads(),
            "kind": "port", "sample": f"single-stream linear1 GEMM (the config-1 shape, one of the block pair's "
                                      f"GEMMs): {rows2} of {M} rows of X against all of W ({rows2 * 2 * N * K / 1e9:.1f} "
                                      f"GFLOP, {dt:.1f} s, bf16 inputs widened to fp32, fp32 accumulate)"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference_config1(args) -> None:
    """The reference's linear_lt (cuBLASLt) from oracle/_ref, timed with CUDA events in C."""
    import ctypes

    import oracle as oracle_mod

    world, rank, local = dist_setup()
    if rank != 0:
        return  # rank 0 alone runs the reference arm
    os.environ.setdefault("CUDA_VISIBLE_DEVICES", str(local))
    if not oracle_mod.REF_PATH.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_cublaslt.so was not built "
                          "(the reference sources were absent at build time)"}))
        return
    o, x, w, bias = make_inputs(oracle_mod)
    ref = oracle_mod.Ref()
    ms, ms_e2e = ctypes.c_double(0), ctypes.c_double(0)
    ref.bench_linear_lt(M, K, N, oracle_mod.CUDA_R_16BF, x.ctypes.data, w.ctypes.data, bias.ctypes.data,
                        args.steps, args.warmup, FLUSH_BYTES, ctypes.byref(ms), ctypes.byref(ms_e2e))
    per = ms.value / args.steps
    per_e2e = ms_e2e.value / args.steps
    value = FLOP / (per * 1e-3) / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (numpy PCG64 seed 0)",
        "config": {"workload": WORKLOAD, "out_dtype": "f32 (linear_lt has no bf16 output)",
                   "l2": "flushed before every step (256 MB write)",
                   "cublaslt_version": int(ref.cublaslt_version())},
        "cpu_baseline": {"kind": "reference", "cores": 0, "value": round(value, 2), "unit": "TFLOP/s",
                         "sample": "the reference has no CPU path; this arm is its own cuBLASLt linear_lt "
                                   "(cublas_ops.cuh:214) built from its sources and run on the B200"},
        "e2e": {"value": round(FLOP / (per_e2e * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 4},
    }
    print(json.dumps(line))


def run_engine_config1(args) -> None:
    import torch

    import b2g
    import oracle as oracle_mod

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    b2g.init()
    o, x_h, w_h, bias_h = make_inputs(oracle_mod)
    x = torch.from_numpy(x_h.view(np.int16)).to(dev).view(torch.bfloat16)
    w = torch.from_numpy(w_h.view(np.int16)).to(dev).view(torch.bfloat16)
    bias = torch.from_numpy(bias_h).to(dev)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        b2g.gemm(x, w, bias, out=out)
    barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    n_launch0 = b2g.launch_count()
    with ClockSampler(local) as clk:
        barrier()
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            evs[i][0].record(stream)
            b2g.gemm(x, w, bias, out=out)
            evs[i][1].record(stream)
        barrier()
    launches = b2g.launch_count() - n_launch0
    per_step = [a.elapsed_time(b) for a, b in evs]
    total_ms = sum(per_step)
    b2g.check_device_error()

    # End to end through the public API with host buffers.
    x_pin = torch.from_numpy(x_h.view(np.int16)).pin_memory()
    out_pin = torch.empty((M, N), dtype=torch.int16).pin_memory()
    x_dev = torch.empty((M, K), dtype=torch.int16, device=dev)
    e2e_steps = max(3, min(args.steps, 50))
    for _ in range(2):
        x_dev.copy_(x_pin, non_blocking=True)
        b2g.gemm(x_dev.view(torch.bfloat16), w, bias, out=out)
        out_pin.copy_(out.view(torch.int16), non_blocking=True)
    barrier()
    e2e_ms = 0.0
    for i in range(e2e_steps):
        flush.fill_(i & 0xFF)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        x_dev.copy_(x_pin, non_blocking=True)
        b2g.gemm(x_dev.view(torch.bfloat16), w, bias, out=out)
        out_pin.copy_(out.view(torch.int16), non_blocking=True)
        b.record(stream)
        b.synchronize()
        e2e_ms += a.elapsed_time(b)
    e2e_per = e2e_ms / e2e_steps

    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([total_ms, e2e_per], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_per = float(t[0]), float(t[1])
    per = total_ms / args.steps
    value = FLOP * args.steps * world / (total_ms * 1e-3) / 1e12
    peaks = measured_peaks()
    achieved = FLOP / (per * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (numpy PCG64 seed 0)",
        "config": {"workload": WORKLOAD, "out_dtype": "bf16", "parallelism": f"replicas x{world}",
                   "l2": "flushed before every step (256 MB write, outside the event pair)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                     "traffic": profile_traffic("tc_gemm_pair_config1.md"),
                     "peak_source": peaks["source"] + " (burst bf16)",
                     "kernel": "tc_gemm_pair_kernel<6,none,bf16> (2-CTA 256x256 tiles)"},
        "e2e": {"value": round(FLOP * world / (e2e_per * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2},
        "clocks": clk.summary(),
        "gpu_launches": int(launches),
        "step_ms_min_median": [round(min(per_step), 5), round(statistics.median(per_step), 5)],
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(o, x_h, w_h, bias_h)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


T_TXT, I_IMG, MASKED = 512, 1024, 400
CFG_HALVES = 2         # conditional + unconditional (forward_cfg)
UNCOND_TEXT_KEYS = 2   # the unconditional half's live text keys (an empty prompt)

WORKLOAD2 = ("config2: one double-stream + one single-stream Chroma block at 512^2 (T=512 txt + I=1024 img "
             "tokens, hidden 3072, 24x128 heads, MLP 12288, key mask on 400 of 512 txt tokens)")


def _ref_blocks_ms(ref, T: int, I: int, steps: int, warmup: int, seed: int = 0) -> float:
    """ms per step of the reference's block pair (double + single block) at T txt + I img tokens."""
    import ctypes

    dp, sp = (ctypes.c_void_p * 32)(), (ctypes.c_void_p * 11)()
    rc = ref.lib.ref_alloc_blocks(seed, T, I, MASKED, dp, sp)
    if rc != 0:
        raise RuntimeError(f"ref_alloc_blocks failed: {rc}")
    ms = ctypes.c_double(0)
    rc = ref.lib.ref_bench_blocks(dp, sp, T, I, steps, warmup, FLUSH_BYTES, ctypes.byref(ms))
    if rc != 0:
        raise RuntimeError(f"ref_bench_blocks failed: CUDA error {rc}")
    return ms.value / steps


def _no_gpu_line(speak: bool = True) -> bool:
    """True when no GPU is visible; then prints the reference arm's `unavailable` line (when
    `speak`, i.e. on rank 0)."""
    import torch

    if torch.cuda.device_count() > 0:
        return False
    if speak:
        print(json.dumps({"impl": "reference", "unavailable": "no CUDA device visible: the reference's path is its "
                      "GPU code (cuBLASLt, cuDNN and its own kernels); it has no CPU implementation"}))
    return True


def _ref_world_max(world: int, vals: list) -> list:
    """Max over ranks of host floats, over a gloo group (the reference arm never touches the
    engine or torch's CUDA state)."""
    if world == 1:
        return vals
    import datetime

    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    t = torch.tensor(vals, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def attention_leg(torch, dev, flush, steps: int, warmup: int, ref=None) -> dict:
    """The attention kernel alone, engine against the reference's cuDNN SDPA, at the config-2
    and config-4 sequence lengths (L = 1536 and 4608; 24 heads x 128, key bias -inf on 400 of
    the 512 text keys).  The operands are bf16 with identical values in both arms, each in its
    own layout: the engine reads q, k, v as column views of the [L, 3 * 3072] buffer its qkv
    epilogue writes and writes bf16 [L, 3072] (flash_attn_kernel); the reference's
    cudnn_sdpa_forward (cudnn_attention.cuh:408-443, graph->execute) reads [24, L, 128] and
    writes [24, L, 128].  Per call: CUDA events around it, a 256 MB L2 flush before it outside
    the events; the median over `steps` calls.  FLOPs: 4 L^2 H D (unmasked), and 4 L (L - 400)
    H D for the live keys."""
    H, D = 24, 128
    out = {}
    for T, I in ((T_TXT, I_IMG), (T_1024, I_1024)):
        L = T + I
        g = torch.Generator(device=dev).manual_seed(11)
        qkv = torch.randn((L, 3, H, D), generator=g, device=dev).to(torch.bfloat16)
        mask = torch.zeros(L, device=dev)
        mask[T - MASKED:T] = float("-inf")
        flop, live = 4.0 * L * L * H * D, 4.0 * L * (L - MASKED) * H * D
        if ref is None:
            import b2g

            flat = qkv.view(L, 3 * H * D)
            q, k, v = flat[:, :H * D], flat[:, H * D:2 * H * D], flat[:, 2 * H * D:]
            o = torch.empty((L, H * D), dtype=torch.bfloat16, device=dev)
            stream = torch.cuda.current_stream(dev)

            def call():
                b2g.attention_bf16(q, k, v, H, D, attn_mask=mask, out=o)

            for _ in range(warmup):
                call()
            torch.cuda.synchronize(dev)
            ms = []
            for i in range(steps):
                flush.fill_(i & 0xFF)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                call()
                b.record(stream)
                b.synchronize()
                ms.append(a.elapsed_time(b))
            what = "flash_attn_kernel (b2g_attention_bf16), bf16 out"
        else:
            q, k, v = (qkv[:, j].permute(1, 0, 2).contiguous() for j in range(3))
            o = torch.empty((H, L, D), dtype=torch.bfloat16, device=dev)
            torch.cuda.synchronize(dev)
            ms = ref.bench_sdpa_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), mask.data_ptr(), o.data_ptr(), H, L, D,
                                     steps, warmup, flush.data_ptr(), flush.numel())
            what = "cuDNN SDPA (cudnn_sdpa_forward: graph->execute), bf16 out"
        med = statistics.median(ms)
        out[f"L{L}"] = {"us": round(1e3 * med, 1), "tflops": round(flop / (med * 1e-3) / 1e12, 1),
                        "tflops_live_keys": round(live / (med * 1e-3) / 1e12, 1), "kernel": what}
        del qkv, q, k, v, o
    out["workload"] = ("attention alone, 24 heads x 128, bf16 operands with identical values in both arms, key "
                       "bias -inf on 400 of 512 text keys; median of per-call CUDA-event times, L2 flushed before "
                       "each call")
    return out


def run_reference_config2(args) -> None:
    """The reference's block code (oracle/_ref/libref_attention.so): its own linear(),
    linear_gated_residual(), rms_norm, cuDNN attention and elementwise kernels in its own call
    order, on inputs from its own Philox generator; timed with CUDA events in C.  With N ranks
    every rank runs one replica on its own GPU (as the engine arm does), and the value is the
    aggregate over ranks from the slowest rank's time.  Rank 0 also times the reference's block
    pair at 1024^2 (L=4608) on its GPU: the single-GPU baseline of the tensor-parallel leg."""
    import oracle as oracle_mod

    world, rank, local = dist_setup()
    os.environ.setdefault("CUDA_VISIBLE_DEVICES", str(local))
    if not oracle_mod.ATTN_REF_PATH.exists():
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_attention.so was not built "
                              "(the reference sources were absent at build time)"}))
        return
    if _no_gpu_line(rank == 0):
        return
    import blocks

    ref = oracle_mod.AttnRef()
    with ClockSampler(local) as clk:
        per = _ref_blocks_ms(ref, T_TXT, I_IMG, args.steps, args.warmup)
    per = _ref_world_max(world, [per])[0]
    tp_ref = None
    if rank == 0 and not args.no_tp1024:
        lin4, att4 = blocks.block_pair_flops(T_1024, I_1024)
        per4 = _ref_blocks_ms(ref, T_1024, I_1024, args.steps, max(3, args.warmup), seed=4)
        tp_ref = {"workload": WORKLOAD_TP1024.split(";")[0] + " (the reference has no tensor-parallel path: its "
                  "block code on one GPU)", "n_gpus": 1, "ms_per_step": round(per4, 5),
                  "tflops": round((lin4 + att4) / (per4 * 1e-3) / 1e12, 2)}
    # The whole denoising step: the reference's own forward_cfg (its harness build), the same
    # workload, copies and timing as the engine arm's e2e.
    import harness
    import model

    h = harness.ForwardCfgHarness(oracle_mod.MODEL_REF_PATH)
    h.setup(42, FC_H, FC_W, *FC_REAL)
    n_fc = max(3, min(args.steps, 20))
    # The per-part legs first, as in the engine arm: before the sustained step loop drives the
    # GPU into its power cap, after a short idle.
    _settle()
    approx_ms = h.bench_modulation(FC_TIMESTEP, max(5, min(args.steps, 30)), 3, FLUSH_BYTES)
    import torch

    glu = nerf_glu_leg(torch, torch.device("cuda", 0), None, None, (FC_H // 16) * (FC_W // 16),
                       max(5, min(args.steps, 30)), h=h)
    fc_dev, fc_e2e = h.bench(FC_TIMESTEP, FC_CFG, n_fc, 3, FLUSH_BYTES)
    fc_dev, fc_e2e = _ref_world_max(world, [fc_dev, fc_e2e])
    fc_flop = model.step_flops(FC_H, FC_W)["total"]
    lin, att = blocks.block_pair_flops(T_TXT, I_IMG)
    value = (lin + att) * world / (per * 1e-3) / 1e12
    if rank != 0:
        return
    import torch

    dev = torch.device("cuda", 0)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    _settle(torch)
    attn = attention_leg(torch, dev, flush, max(5, min(args.steps, 50)), max(3, args.warmup), ref=ref)
    approx = approximator_leg(torch, dev, flush, None, None, 0, ms_list=approx_ms)
    approx["workload"] += "; the reference's own ChromaApproximator (linear() on cuBLASLt) in its forward_cfg build"
    t5_ms = ref.bench_t5_leg(T5_LAYERS, T5_TOKENS, T5_D, T5_FF, T5_HEADS, 5, 2, flush.data_ptr(), flush.numel())
    t5 = t5_line(statistics.median(t5_ms), "the reference's own calls in t5.cuh's order: linear() on fp16 weights "
                 "for q, k, v, o, wi_0, wi_1, wo (each casting its F32 input to fp16), t5_attention (fp32 cuBLAS "
                 "SGEMMs), gelu_cuda on the gate; RMSNorms, gate product and residual adds left out, as in the "
                 "engine's leg; L2 flushed before each of 5 passes (median)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (reference Philox, seed 0)",
        "config": {"workload": WORKLOAD2, "flop_per_step": lin + att, "parallelism": f"replicas x{world}",
                   "l2": "weights 680 MB > L2; 256 MB buffer written before every step, outside the events"},
        "cpu_baseline": {"kind": "reference", "cores": 0, "value": round(value, 2), "unit": "TFLOP/s",
                         "sample": "the reference has no CPU path; this arm is its own block code (chroma.cuh "
                                   "double/single block GEMM + attention calls, cublas_ops.cuh, cuDNN SDPA) "
                                   "built from its sources and run on the B200"},
        "e2e": {"value": round(fc_flop * world / (fc_e2e * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": (3 * FC_H * FC_W + 2 * 512 * 4096) * 4, "d2h_bytes_per_step": 3 * FC_H * FC_W * 4,
                "ms_per_step": round(fc_e2e, 4), "device_ms_per_step": round(fc_dev, 4), "flop_per_step": fc_flop,
                "steps": n_fc,
                "workload": WORKLOAD3 + "; the reference's own ChromaRadiance::forward_cfg (cuBLASLt, cuDNN, its "
                            "kernels) on stream 0, weights in its Tensor fields from its own Philox generator; per "
                            "step the noise and both T5 contexts copied in from pinned host memory and the velocity "
                            "copied back inside the events"},
        "clocks": clk.summary(),
        "tp1024": tp_ref,
        "attention": attn,
        "approximator": approx,
        "nerf_glu_block": glu,
        "t5": t5,
    }), flush=True)


class _Marks:
    """Timing events recorded between the launches of a captured block (external event nodes)."""

    def __init__(self, torch, stream):
        self.torch, self.stream = torch, stream
        self.events, self.labels = [], []
        self.start = torch.cuda.Event(enable_timing=True, external=True)

    def begin(self):
        self.start.record(self.stream)

    def __call__(self, label):
        ev = self.torch.cuda.Event(enable_timing=True, external=True)
        ev.record(self.stream)
        self.events.append(ev)
        self.labels.append(label)

    def durations(self):
        out, prev = {}, self.start
        for lab, ev in zip(self.labels, self.events):
            out[lab] = out.get(lab, 0.0) + prev.elapsed_time(ev)
            prev = ev
        return out


def run_engine_config2(args) -> None:
    import torch

    import b2g
    import blocks

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    b2g.init()
    T, I = T_TXT, I_IMG
    L = T + I
    H = blocks.HIDDEN
    gdev = torch.Generator(device=dev).manual_seed(0)
    txt_w, img_w = blocks.random_stream(gdev, dev), blocks.random_stream(gdev, dev)
    sw = blocks.random_single(gdev, dev)
    ang = torch.rand((L, blocks.DHEAD // 2), generator=gdev, device=dev) * 6.2831853
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    mask = torch.zeros(L, device=dev)
    mask[T - MASKED:T] = float("-inf")
    # Step inputs: generated on the host (seeded) and kept pinned for the end-to-end leg.
    gh = torch.Generator().manual_seed(1)
    host = {}
    for name, rows, dt in (("txt_mod1", T, torch.bfloat16), ("img_mod1", I, torch.bfloat16),
                           ("txt_mod2", T, torch.bfloat16), ("img_mod2", I, torch.bfloat16),
                           ("txt", T, torch.float32), ("img", I, torch.float32),
                           ("x_mod", L, torch.bfloat16), ("x", L, torch.float32)):
        host[name] = torch.randn((rows, H), generator=gh).to(dt).pin_memory()
    host["gates"] = torch.randn((5, H), generator=gh).pin_memory()
    d = {k: v.to(dev) for k, v in host.items()}
    gt = d["gates"]
    scratch = blocks.Scratch(T, I, dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def run_double(mark=None):
        blocks.double_block(txt_w, img_w, d["txt_mod1"], d["img_mod1"], d["txt_mod2"], d["img_mod2"], d["txt"],
                            d["img"], gt[0], gt[1], gt[2], gt[3], pe, mask, scratch, mark)

    def run_single(mark=None):
        blocks.single_block(sw, d["x_mod"], d["x"], gt[4], pe, mask, scratch, mark)

    run_double()
    run_single()  # sizes the engine's workspaces before capture
    torch.cuda.synchronize(dev)
    cap = torch.cuda.Stream(dev)

    def capture(with_marks):
        gs, ms = [], []
        for fn in (run_double, run_single):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(cap):
                mk = _Marks(torch, cap) if with_marks else None
                with torch.cuda.graph(g, stream=cap):
                    if mk:
                        mk.begin()
                    fn(mk)
            gs.append(g)
            ms.append(mk)
        return gs, ms

    # The timed graphs hold only the engine's launches (consecutive kernels overlap set-up and
    # tail through programmatic dependent launch); a second pair of graphs with timing events
    # between the launches gives the per-operation breakdown.
    n0 = b2g.launch_count()
    graphs, _ = capture(False)
    launches_per_step = b2g.launch_count() - n0
    marked, marks = capture(True)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        for g in graphs:
            g.replay()
    barrier()
    per_step, per_op = [], {}
    with ClockSampler(local) as clk:
        barrier()
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for g in graphs:
                g.replay()
            b.record(stream)
            b.synchronize()
            per_step.append(a.elapsed_time(b))
        barrier()
    total_ms = sum(per_step)
    for i in range(max(3, min(args.steps, 20))):
        flush.fill_(i & 0xFF)
        for g in marked:
            g.replay()
        torch.cuda.synchronize(dev)
        for mk in marks:
            for lab, ms in mk.durations().items():
                per_op.setdefault(lab, []).append(ms)
    b2g.check_device_error()

    # End to end with host buffers: inputs in on one side stream, outputs back on another.
    cin, cout = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    outs = {k: torch.empty_like(host[k]).pin_memory() for k in ("txt", "img", "x")}
    dbl_in = ("txt_mod1", "img_mod1", "txt_mod2", "img_mod2", "txt", "img", "gates")
    sgl_in = ("x_mod", "x")
    h2d = sum(host[k].numel() * host[k].element_size() for k in dbl_in + sgl_in)
    d2h = sum(v.numel() * v.element_size() for v in outs.values())

    def e2e_step():
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_din, e_sin, e_dd, e_dout = (torch.cuda.Event() for _ in range(4))
        a.record(stream)
        cin.wait_event(a)
        with torch.cuda.stream(cin):
            for k in dbl_in:
                d[k].copy_(host[k], non_blocking=True)
            e_din.record(cin)
            for k in sgl_in:
                d[k].copy_(host[k], non_blocking=True)
            e_sin.record(cin)
        stream.wait_event(e_din)
        graphs[0].replay()
        e_dd.record(stream)
        cout.wait_event(e_dd)
        with torch.cuda.stream(cout):
            outs["txt"].copy_(d["txt"], non_blocking=True)
            outs["img"].copy_(d["img"], non_blocking=True)
            e_dout.record(cout)
        stream.wait_event(e_sin)
        graphs[1].replay()
        outs["x"].copy_(d["x"], non_blocking=True)
        stream.wait_event(e_dout)
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b)

    for _ in range(3):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 50))
    e2e_ms = 0.0
    for i in range(e2e_steps):
        flush.fill_(i & 0xFF)
        torch.cuda.synchronize(dev)
        e2e_ms += e2e_step()
    e2e_per = e2e_ms / e2e_steps
    del graphs, marked

    fc = forward_cfg_leg(args, torch, dev, flush, dropin=(world == 1 and not args.no_dropin))
    if rank == 0:
        _settle(torch)
    attn = attention_leg(torch, dev, flush, max(5, min(args.steps, 50)), max(3, args.warmup)) if rank == 0 else None
    t5 = (t5_encoder_leg(torch, b2g, dev, torch.Generator(device=dev).manual_seed(5), torch.cuda.current_stream(dev),
                         flush) if rank == 0 else None)
    tp_leg = tp1024_leg(args, torch, world, rank, dev, txt_w, img_w, sw, flush) if not args.no_tp1024 else None

    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([total_ms, e2e_per, fc["ms_per_step"]], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_per, fc["ms_per_step"] = float(t[0]), float(t[1]), float(t[2])
    ops = blocks.block_pair_ops(T, I)
    flop_step = sum(f for _, _, f in ops)
    per = total_ms / args.steps
    value = flop_step * args.steps * world / (total_ms * 1e-3) / 1e12
    mean_op = {lab: statistics.mean(v) for lab, v in per_op.items()}
    # The marked replay's event nodes keep consecutive kernels from overlapping, so its
    # per-operation times sum above the timed step: scale them to the timed step time.
    marked_ms = sum(mean_op.values())
    fit = per / marked_ms if marked_ms > 0 else 1.0
    mean_op = {lab: v * fit for lab, v in mean_op.items()}
    gemm_flop = sum(f for lab, kind, f in ops if kind == "gemm")
    gemm_ms = sum(mean_op[lab] for lab, kind, _ in ops if kind == "gemm")
    peaks = measured_peaks()
    achieved = gemm_flop / (gemm_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (torch Philox/CPU generators, seeds 0/1)",
        "config": {"workload": WORKLOAD2, "flop_per_step": flop_step, "parallelism": f"replicas x{world}",
                   "l2": "weights 680 MB > L2; 256 MB buffer written before every step, outside the events",
                   "execution": "two CUDA graphs (double block, single block) per step"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                     "traffic": profile_traffic("block_pair_config2_launches.md"),
                     "peak_source": peaks["source"] + " (burst bf16)",
                     "kernel": "tc_gemm: the block pair's 6 linear-layer launches, FLOP-weighted",
                     "gemm_ms_per_step": round(gemm_ms, 5)},
        "breakdown_us": {lab: round(1e3 * mean_op[lab], 1) for lab, _, _ in ops},
        "breakdown_tflops": {lab: round(f / (mean_op[lab] * 1e-3) / 1e12, 1) for lab, _, f in ops},
        "e2e": dict(fc, value=round(fc["flop_per_step"] * world / (fc["ms_per_step"] * 1e-3) / 1e12, 3),
                    ms_per_step=round(fc["ms_per_step"], 4)),
        "e2e_block_pair": {"value": round(flop_step * world / (e2e_per * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_per, 4),
                           "workload": "the timed block pair with all of its activations (modulated inputs, "
                                       "residual streams, gates) copied in and the residual streams copied out "
                                       "every step: PCIe-bound"},
        "clocks": clk.summary(),
        "gpu_launches": int(launches_per_step * args.steps),
        "step_ms_min_median": [round(min(per_step), 5), round(statistics.median(per_step), 5)],
        "tp1024": tp_leg,
        "attention": attn,
        "t5": t5,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle as oracle_mod

        o, x_h, w_h, bias_h = make_inputs(oracle_mod)
        line["cpu_baseline"] = cpu_baseline(o, x_h, w_h, bias_h)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()



# ---------------------------------------------------------------------------- the whole step
WORKLOAD3 = ("config3: one denoising step at 512^2, ChromaRadiance::forward_cfg (chroma.cuh:1499-1584): img_in, "
             "txt_in, the approximator, 19 double + 38 single blocks over both guidance halves (conditional: "
             "112 of 512 text keys live, unconditional: 2), two NeRF decodes and cfg_blend (scale 4), timestep "
             "0.7, random-init weights (19 GB)")
FC_H = FC_W = 512
FC_REAL = (111, 1)
FC_TIMESTEP, FC_CFG = 0.7, 4.0


def approximator_shapes() -> list:
    """(label, M, N, K) of the approximator's GEMMs (chroma.cuh:188-212, 467-508)."""
    import model

    M, A = model.MOD_ROWS, model.APPROX_DIM
    out = [("in_proj", M, A, 64)]
    for i in range(model.APPROX_LAYERS):
        out += [(f"layer{i}.in", M, A, A), (f"layer{i}.out", M, A, A)]
    return out + [("out_proj", M, model.HIDDEN, A)]


def approximator_bytes(M: int, N: int, K: int) -> int:
    """Algorithmic HBM bytes of one approximator GEMM: the bf16 weight, the F32 activations in
    (cast to bf16 by linear(), cublas_ops.cuh:486-490) and the F32 output."""
    return N * K * 2 + M * K * 4 + M * N * 4


def approximator_leg(torch, dev, flush, stream, run, steps: int, ms_list=None) -> dict:
    """The approximator alone (compute_modulation: 12 GEMMs at M=344, 556 MB of bf16 weights, the
    weight-streaming 'skinny' shape): median per-call time over `steps` calls (CUDA events, L2
    flushed before each), TFLOP/s and achieved HBM GB/s of its algorithmic bytes against
    MEASURED_PEAKS.json hbm_gbs.  The engine's call is captured once in a CUDA graph and
    replayed (forward_cfg runs it inside its step graph); with `run(mark)` also a per-GEMM
    split from a second capture with timing events between the launches.  `ms_list` (the
    reference arm) gives the per-call times instead of running anything."""
    shapes = approximator_shapes()
    flop = sum(2.0 * M * N * K for _, M, N, K in shapes)
    byts = sum(approximator_bytes(M, N, K) for _, M, N, K in shapes)
    graph = marked = marks = None
    if ms_list is None:
        for _ in range(3):
            run()
        torch.cuda.synchronize(dev)
        cap = torch.cuda.Stream(dev)
        graph, marked = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        marks = _Marks(torch, cap)
        with torch.cuda.stream(cap):
            with torch.cuda.graph(graph, stream=cap):
                run()
            with torch.cuda.graph(marked, stream=cap):
                marks.begin()
                run(marks)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(dev)
        ms_list = []
        for i in range(steps):
            flush.fill_(i & 0xFF)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            graph.replay()
            b.record(stream)
            b.synchronize()
            ms_list.append(a.elapsed_time(b))
    med = statistics.median(ms_list)
    peaks = measured_peaks()
    out = {"us": round(1e3 * med, 1), "tflops": round(flop / (med * 1e-3) / 1e12, 1),
           "hbm_gbs": round(byts / (med * 1e-3) / 1e9, 1), "hbm_frac": round(byts / (med * 1e-3) / 1e9 /
                                                                            peaks["hbm_gbs"], 3),
           "flop": flop, "bytes": byts,
           "workload": "the approximator (compute_modulation, guidance 0): 12 GEMMs at M=344 (64->5120, 10 x "
                       "5120->5120, 5120->3072) with their RMSNorms; median of per-call CUDA-event times, L2 "
                       "flushed before each call; bytes = bf16 weights + F32 activations in + F32 outputs"
                       + ("" if run is None else "; the engine's call replayed as a CUDA graph")}
    if marked is not None:
        flush.fill_(0)
        torch.cuda.synchronize(dev)
        marked.replay()
        torch.cuda.synchronize(dev)
        per = marks.durations()
        del graph, marked
        out["per_gemm"] = {lab: {"us": round(1e3 * per[lab], 1),
                                 "hbm_gbs": round(approximator_bytes(M, N, K) / (per[lab] * 1e-3) / 1e9, 1),
                                 "tflops": round(2.0 * M * N * K / (per[lab] * 1e-3) / 1e12, 1)}
                           for lab, M, N, K in shapes if lab in per}
    return out


def nerf_glu_leg(torch, dev, flush, stream, P: int, steps: int, m=None, h=None) -> dict:
    """One NeRF GLU block (nerf_glu_block, chroma.cuh:1253-1306) alone at one guidance half's
    P patches, both arms on their own block-0 weights and the same seeded x [P, 256, 64] and
    s [P, 3072]: the reference's whole block (param_generator linear, weight slices and L2
    norms, rms_norm, three cuBLAS batched products, silu_mul, residual add; `h`, its harness),
    or the engine's cast of s, param_generator GEMM and fused GLU kernel (`m`).  Median per call
    (CUDA events, L2 flushed before each)."""
    g = torch.Generator(device=dev).manual_seed(31)
    x = torch.randn((P, 256, 64), generator=g, device=dev)
    sv = torch.randn((P, 3072), generator=g, device=dev)
    if h is not None:
        ms = h.bench_nerf_glu_block(0, x, sv, steps, 3, FLUSH_BYTES)
        what = "the reference's nerf_glu_block: 14 launches (cuBLASLt linear, cuBLAS batched products, its kernels)"
    else:
        import b2g

        blk = m.nerf[0]
        s16 = torch.empty((P, 3072), dtype=torch.bfloat16, device=dev)
        params = torch.empty((P, blk.param_w.shape[0]), device=dev)

        def run():
            b2g.convert_f32(sv, s16)
            b2g.gemm(s16, blk.param_w, blk.param_b, out=params)
            b2g.nerf_glu_block(params, blk.norm, x)

        for _ in range(3):
            run()
        torch.cuda.synchronize(dev)
        ms = []
        for i in range(steps):
            flush.fill_(i & 0xFF)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            run()
            b.record(stream)
            b.synchronize()
            ms.append(a.elapsed_time(b))
        what = "the engine: cast of s, param_generator GEMM (tc_gemm), nerf_glu_kernel (3 launches)"
    return {"us": round(1e3 * statistics.median(ms), 1), "patches": P, "kernels": what,
            "workload": "one NeRF GLU block at 512^2 for one guidance half (1024 patches), block 0's weights, "
                        "seeded x and s; median of per-call CUDA-event times, L2 flushed before each"}


def forward_cfg_leg(args, torch, dev, flush, dropin: bool) -> dict:
    """The engine's whole denoising step (model.ChromaRadiance.forward_cfg) through the public API,
    captured in one CUDA graph; every step copies its inputs (noise, both T5 contexts, the
    timestep) in from pinned host memory and the velocity back, inside the events.  After the
    timed steps, one eager step is split by part.  With `dropin`, the reference's own
    forward_cfg built through the drop-in headers (every GEMM and attention in libb2g.so) is
    timed beside it, on its own random weights."""
    import b2g
    import model

    g = torch.Generator(device=dev).manual_seed(42)
    m = model.ChromaRadiance(model.random_weights(g, dev), dev)
    s = model.ForwardScratch(FC_H, FC_W, dev)
    gh = torch.Generator().manual_seed(3)
    host = {"x": torch.randn((1, 3, FC_H, FC_W), generator=gh).pin_memory(),
            "cc": torch.randn((model.TXT_TOKENS, model.CTX_DIM), generator=gh).pin_memory(),
            "cu": torch.randn((model.TXT_TOKENS, model.CTX_DIM), generator=gh).pin_memory(),
            "t": torch.tensor([FC_TIMESTEP]).pin_memory()}
    d = {k: torch.empty_like(v, device=dev) for k, v in host.items() if k != "t"}
    vel_h = torch.empty((1, 3, FC_H, FC_W)).pin_memory()
    pe = torch.from_numpy(model.rope_table(FC_H, FC_W)).to(dev)
    dct = torch.from_numpy(model.dct_features()).to(dev)
    masks = torch.from_numpy(model.key_masks(list(FC_REAL), FC_H, FC_W)).to(dev)
    for k in d:
        d[k].copy_(host[k])
    s.timestep.copy_(host["t"])

    def run():
        m.forward_cfg(s, d["x"], d["cc"], d["cu"], pe, dct, masks, FC_CFG)

    run()  # sizes the library's workspaces before capture
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    # The per-part legs first, before the sustained step loop drives the GPU into its power cap
    # (the reference arm orders its legs the same way), after a short idle.
    _settle(torch)
    approx = approximator_leg(torch, dev, flush, stream, lambda mark=None: m.compute_modulation(s, mark),
                              max(5, min(args.steps, 30)))
    glu = nerf_glu_leg(torch, dev, flush, stream, s.P, max(5, min(args.steps, 30)), m=m)
    run()
    torch.cuda.synchronize(dev)
    cap = torch.cuda.Stream(dev)
    n0 = b2g.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            run()
    launches = b2g.launch_count() - n0
    stream = torch.cuda.current_stream(dev)

    def step():
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for k in d:
            d[k].copy_(host[k], non_blocking=True)
        s.timestep.copy_(host["t"], non_blocking=True)
        graph.replay()
        vel_h.copy_(s.velocity, non_blocking=True)
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b)

    for _ in range(max(3, min(args.warmup, 5))):
        step()
    n = max(3, min(args.steps, 20))
    times = []
    for i in range(n):
        flush.fill_(i & 0xFF)
        torch.cuda.synchronize(dev)
        times.append(step())
    b2g.check_device_error()
    ms = sum(times) / n

    def timed(fn) -> float:
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b)

    import blocks as blocks_mod

    parts = {"embed": timed(lambda: m.embed(s, d["x"], d["cc"], d["cu"])),
             "approximator": timed(lambda: m.compute_modulation(s)),
             "blocks": timed(lambda: blocks_mod.forward_pass(m.blocks, s.x, pe, masks, s.blocks, s.T)),
             "nerf_decode": timed(lambda: m.nerf_decode(s, d["x"], dct)),
             "nerf_final_cfg_blend": timed(lambda: b2g.nerf_final(s.nx[0], s.nx[1], m.final_norm, m.conv_w, m.conv_b,
                                                                  FC_CFG, FC_H, FC_W,
                                                                  s.velocity.view(3, FC_H, FC_W)))}
    flops = model.step_flops(FC_H, FC_W)
    out = {"unit": "TFLOP/s", "ms_per_step": ms, "flop_per_step": flops["total"],
           "h2d_bytes_per_step": sum(host[k].numel() * host[k].element_size() for k in host),
           "d2h_bytes_per_step": vel_h.numel() * 4, "steps": n,
           "workload": WORKLOAD3 + "; through the public API (model.ChromaRadiance.forward_cfg), one CUDA graph of "
                       f"{launches} engine launches; per step the noise, both T5 contexts and the timestep are "
                       "copied in from pinned host memory and the velocity copied back inside the events; FLOPs "
                       "= every GEMM and attention of the step (unmasked), the element-wise work not counted",
           "parts_ms_eager": {k: round(v, 3) for k, v in parts.items()},
           "parts_tflop": {k: round(flops[k] / 1e12, 4) for k in ("embed", "approximator", "blocks", "nerf")},
           "launches_per_step": launches, "step_ms_min_median": [round(min(times), 4),
                                                                 round(statistics.median(times), 4)],
           "approximator": approx, "nerf_glu_block": glu}
    del graph, m, s
    torch.cuda.empty_cache()
    if dropin:
        import harness

        if harness.DROPIN_PATH.exists():
            h = harness.ForwardCfgHarness(harness.DROPIN_PATH)
            h.setup(42, FC_H, FC_W, *FC_REAL)
            dev_ms, e2e_ms = h.bench(FC_TIMESTEP, FC_CFG, n, 3, FLUSH_BYTES)
            out["dropin_forward_cfg"] = {
                "ms_per_step": round(e2e_ms, 4), "device_ms_per_step": round(dev_ms, 4),
                "what": "the reference's own ChromaRadiance::forward_cfg, unchanged, built through the drop-in "
                        "headers (cublas_ops.cuh, cudnn_attention.cuh, attention.cuh): every GEMM and attention "
                        "in libb2g.so, everything else the reference's own kernels; same copies as this e2e"}
    return out


# ---------------------------------------------------------------------------- 1024^2 TP leg
T_1024, I_1024 = 512, 4096
WORKLOAD_TP1024 = ("config4's block pair at 1024^2: one double-stream + one single-stream block, T=512 txt + "
                   "I=4096 img tokens (L=4608), hidden 3072, 24x128 heads, MLP 12288, key mask on 400 of 512 txt "
                   "tokens; 1 GPU: the unsharded block pair; N GPUs: tensor parallel (column-split qkv/linear1/mlp0 "
                   "by heads and MLP columns, row-split proj/mlp2/linear2 with the all-rank reduction fused into the "
                   "GEMM over NVLink peer memory, one cross-rank barrier kernel per row-split layer)")


def _settle(torch=None, seconds: float = 2.0) -> None:
    """Idle before a group of short per-part legs, in both arms alike: right after a sustained
    load (a timed step loop, or initialising 20 GB of weights) the GPU runs short
    memory-bound work up to ~30% slower for under a second (measured on the approximator:
    476-485 us right after 200 block pairs, 373-375 us after 1 s idle)."""
    import time

    if torch is not None:
        torch.cuda.synchronize()
    time.sleep(seconds)


class _EagerMarks:
    """Events recorded between eagerly launched operations (per-operation time split)."""

    def __init__(self, torch, stream):
        self.torch, self.stream = torch, stream
        self.start = torch.cuda.Event(enable_timing=True)
        self.items = []

    def begin(self):
        self.start.record(self.stream)

    def __call__(self, label):
        ev = self.torch.cuda.Event(enable_timing=True)
        ev.record(self.stream)
        self.items.append((label, ev))

    def durations(self) -> dict:
        out, prev = {}, self.start
        for lab, ev in self.items:
            out[lab] = out.get(lab, 0.0) + prev.elapsed_time(ev)
            prev = ev
        return out


def _tp_categories(us: dict) -> dict:
    """Sums of a per-operation split: column-split GEMMs, attention, row-split GEMMs (with the
    fused all-rank reduction at N > 1) and cross-rank barriers."""
    cat = {"column_gemms": 0.0, "attention": 0.0, "row_gemms_with_reduction": 0.0, "barriers": 0.0,
           "all_reduce": 0.0, "bias_gated_residual": 0.0}
    for lab, v in us.items():
        if lab.endswith(".barrier"):
            cat["barriers"] += v
        elif lab.endswith(".all_reduce") or lab.endswith(".reduce"):
            cat["all_reduce"] += v
        elif lab.endswith(".residual"):
            cat["bias_gated_residual"] += v
        elif "attention" in lab:
            cat["attention"] += v
        elif lab.split(".")[-1] in ("proj", "mlp2", "linear2"):
            cat["row_gemms_with_reduction"] += v
        else:
            cat["column_gemms"] += v
    return {k: round(v, 1) for k, v in cat.items()}


def tp1024_leg(args, torch, world, rank, dev, txt_w, img_w, sw, flush) -> dict:
    """BASELINE config 4's block pair at 1024^2 on every rank of this run (chroma.cuh:808-1157 at
    L=4608).  One GPU: the unsharded block pair.  N GPUs: tp.py's fused tensor-parallel path, and
    on rank 0 also the unsharded block pair on its own GPU (the 1-GPU time the speed-up is taken
    against, and the parity reference: the replicated residual streams after one step from the
    same seeded inputs, max|d|/max|ref| and cosine of the update).  The NCCL all-reduce, pull
    and push variants are timed beside the fused one.  Every path (the unsharded one included)
    is timed as a CUDA graph replay of its whole block pair, captured after an eager run (the
    cross-rank barriers keep their epoch on the device, so replays stay in step); the
    per-operation split comes from a second capture with timing events between the launches.
    An L2 flush (256 MB write) and, at N > 1, a barrier before every step, outside the events;
    device time, max over ranks."""
    import datetime

    import blocks
    import tp

    T, I = T_1024, I_1024
    L, H = T + I, blocks.HIDDEN
    g = torch.Generator(device=dev).manual_seed(4)   # identical inputs on every rank
    act = {k: torch.randn((n, H), generator=g, device=dev).to(torch.bfloat16) for k, n in
           (("txt_mod1", T), ("img_mod1", I), ("txt_mod2", T), ("img_mod2", I), ("x_mod", L))}
    res = {k: torch.randn((n, H), generator=g, device=dev) for k, n in (("txt", T), ("img", I), ("x", L))}
    gt = [torch.randn(H, generator=g, device=dev) for _ in range(5)]
    ang = torch.rand((L, blocks.DHEAD // 2), generator=g, device=dev) * 6.2831853
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    mask = torch.zeros(L, device=dev)
    mask[T - MASKED:T] = float("-inf")
    stream = torch.cuda.current_stream(dev)
    steps, warm = args.steps, max(3, args.warmup)
    lin, att = blocks.block_pair_flops(T, I)
    if world > 1:
        import torch.distributed as dist

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def timed(fn, sync_ranks: bool) -> list:
        if sync_ranks:
            barrier()
        for _ in range(warm):
            fn()
        torch.cuda.synchronize(dev)
        out = []
        for i in range(steps):
            flush.fill_(i & 0xFF)
            if sync_ranks:
                barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            b.synchronize()
            out.append(a.elapsed_time(b))
        return out

    cap = torch.cuda.Stream(dev)
    held = []   # every captured graph; released before the leg returns (NCCL's among them)

    def graphed(fn):
        """fn (already run eagerly: every workspace exists) captured in a CUDA graph, and again
        with timing events between its launches; returns (replay, marked graph, marks)."""
        torch.cuda.synchronize(dev)
        g, gm = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        mk = _Marks(torch, cap)
        with torch.cuda.stream(cap):
            with torch.cuda.graph(g, stream=cap):
                fn()
            with torch.cuda.graph(gm, stream=cap):
                mk.begin()
                fn(mk)
        held.extend([g, gm])
        return g.replay, gm, mk

    def split(captured, sync_ranks: bool) -> dict:
        _, gm, mk = captured
        if sync_ranks:
            barrier()
        gm.replay()
        torch.cuda.synchronize(dev)
        return {k: 1e3 * v for k, v in mk.durations().items()}

    def delta(a, b):
        return (a - b).double().flatten()

    out = {"workload": WORKLOAD_TP1024, "n_gpus": world, "steps": steps, "warmup": warm,
           "flop_per_step": lin + att}
    # --- the unsharded block pair (the whole leg at N = 1; rank 0's reference at N > 1)
    uns_ms, uns_split, ref = None, None, None
    if rank == 0:
        s1 = blocks.Scratch(T, I, dev)
        ures = {k: v.clone() for k, v in res.items()}

        def unsharded(mark=None):
            blocks.double_block(txt_w, img_w, act["txt_mod1"], act["img_mod1"], act["txt_mod2"], act["img_mod2"],
                                ures["txt"], ures["img"], gt[0], gt[1], gt[2], gt[3], pe, mask, s1, mark)
            blocks.single_block(sw, act["x_mod"], ures["x"], gt[4], pe, mask, s1, mark)

        unsharded()
        torch.cuda.synchronize(dev)
        ref = {k: delta(ures[k], res[k]) for k in res}
        cu = graphed(unsharded)
        per = timed(cu[0], False)
        uns_ms = sum(per) / steps
        uns_split = split(cu, False)
        del cu, s1, ures
        held.clear()
    if world == 1:
        out.update({"mode": "unsharded block pair, 1 GPU", "ms_per_step": round(uns_ms, 5),
                    "tflops": round((lin + att) / (uns_ms * 1e-3) / 1e12, 2),
                    "breakdown_us": {k: round(v, 1) for k, v in uns_split.items()},
                    "categories_us": _tp_categories(uns_split), "unsharded_ms_per_step": round(uns_ms, 5),
                    "speedup_vs_1gpu": 1.0, "parity": None})
        return out
    barrier()
    # --- the tensor-parallel block pair (every rank)
    ops = tp.EngineOps()
    tw, iw, ts = tp.shard_stream(txt_w, rank, world), tp.shard_stream(img_w, rank, world), tp.shard_single(sw, rank,
                                                                                                          world)
    scratch = tp.TPScratch(T, I, world, dev)
    comm = tp.SymmetricComm(L, H, None, dev)

    def load_res():
        comm.res_double[:T].copy_(res["txt"])
        comm.res_double[T:].copy_(res["img"])
        comm.res_single.copy_(res["x"])

    def fused(mark=None):
        tp.tp_double_block_fused(ops, comm, tw, iw, act["txt_mod1"], act["img_mod1"], act["txt_mod2"],
                                 act["img_mod2"], gt[0], gt[1], gt[2], gt[3], pe, mask, scratch, mark)
        tp.tp_single_block_fused(ops, comm, ts, act["x_mod"], gt[4], pe, mask, scratch, mark)

    load_res()
    barrier()
    fused()
    barrier()
    parity = None
    if rank == 0:
        got = {"txt": delta(comm.res_double[:T], res["txt"]), "img": delta(comm.res_double[T:], res["img"]),
               "x": delta(comm.res_single, res["x"])}
        parity = {}
        for k in got:
            parity[k] = {"max_rel": float((got[k] - ref[k]).abs().max() / ref[k].abs().max()),
                         "cosine": float((got[k] @ ref[k]) / (got[k].norm() * ref[k].norm()))}
        parity["against"] = ("the unsharded block pair on rank 0's GPU, same seeded weights and inputs: the update "
                             "of the replicated residual streams (txt, img, single-block x) after one step")
        parity["within_tolerance"] = all(v["max_rel"] <= 1e-2 and v["cosine"] >= 0.9999
                                         for k, v in parity.items() if isinstance(v, dict))
    cf = graphed(fused)
    per_f = timed(cf[0], True)
    sp = split(cf, True)
    nres = {k: v.clone() for k, v in res.items()}

    def nccl(mark=None):
        tp.tp_double_block(ops, tw, iw, act["txt_mod1"], act["img_mod1"], act["txt_mod2"], act["img_mod2"],
                           nres["txt"], nres["img"], gt[0], gt[1], gt[2], gt[3], pe, mask, scratch, mark)
        tp.tp_single_block(ops, ts, act["x_mod"], nres["x"], gt[4], pe, mask, scratch, mark)

    nccl()   # eager first (NCCL's communicator and the workspaces), then captured
    barrier()
    cn = graphed(nccl)
    per_n = timed(cn[0], True)
    sp_n = split(cn, True)
    runs = {}
    for name, push in (("p2p", False), ("push", True), ("store", "store")):
        pres = {k: v.clone() for k, v in res.items()}

        def path(mark=None, pres=pres, push=push):
            tp.tp_double_block_p2p(ops, comm, tw, iw, act["txt_mod1"], act["img_mod1"], act["txt_mod2"],
                                   act["img_mod2"], pres["txt"], pres["img"], gt[0], gt[1], gt[2], gt[3], pe, mask,
                                   scratch, mark, push=push)
            tp.tp_single_block_p2p(ops, comm, ts, act["x_mod"], pres["x"], gt[4], pe, mask, scratch, mark, push=push)

        path()
        barrier()
        if rank == 0:
            got = {k: delta(pres[k], res[k]) for k in res}
            parity[name] = {k: {"max_rel": float((got[k] - ref[k]).abs().max() / ref[k].abs().max()),
                                "cosine": float((got[k] @ ref[k]) / (got[k].norm() * ref[k].norm()))} for k in got}
            parity["within_tolerance"] = parity["within_tolerance"] and all(
                v["max_rel"] <= 1e-2 and v["cosine"] >= 0.9999 for v in parity[name].values())
        cp = graphed(path)
        runs[name] = (timed(cp[0], True), split(cp, True))
    per_p, sp_p = runs["p2p"]
    per_q, sp_q = runs["push"]
    per_s, sp_s = runs["store"]
    b2g_mod = __import__("b2g")
    b2g_mod.check_device_error()
    labels, labels_n, labels_p, labels_q, labels_s = sorted(sp), sorted(sp_n), sorted(sp_p), sorted(sp_q), sorted(sp_s)
    t = torch.tensor([sum(per_f), sum(per_n), sum(per_p), sum(per_q), sum(per_s)] + [sp[k] for k in labels] +
                     [sp_n[k] for k in labels_n] + [sp_p[k] for k in labels_p] + [sp_q[k] for k in labels_q] +
                     [sp_s[k] for k in labels_s], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    f_ms, n_ms, p_ms, q_ms, s_ms = (float(t[i]) / steps for i in range(5))
    vals = t[5:].tolist()
    splits_out = []
    for lab in (labels, labels_n, labels_p, labels_q, labels_s):
        splits_out.append({k: float(v) for k, v in zip(lab, vals[:len(lab)])})
        vals = vals[len(lab):]
    sp, sp_n, sp_p, sp_q, sp_s = splits_out
    u = torch.tensor([uns_ms or 0.0], device=dev, dtype=torch.float64)
    dist.all_reduce(u, op=dist.ReduceOp.MAX)   # rank 0's 1-GPU time, on every rank
    uns_ms = float(u[0])
    fused_mode = f"tp{world}, reduction fused into the row-split GEMMs over NVLink peer memory"
    nccl_mode = (f"tp{world}, NCCL all-reduce (bf16) of each row-split GEMM's partial, then bias + gated residual "
                 "(b2g_bias_gated_residual)")
    p2p_mode = (f"tp{world}, two-phase all-reduce over NVLink peer memory (each rank sums its shard of rows from "
                "every rank's partial, then every rank applies the bias + gated residual from the owners' sums)")
    # The headline is the fastest of the communication paths, all measured in this run.
    push_mode = (f"tp{world}, all-reduce by copy-engine copies over NVLink (each shard of partial rows into its "
                 "owner's receive slot, the owner's local sum of its slots copied to every rank), then the bias + "
                 "gated residual from each rank's own sums")
    store_mode = (f"tp{world}, all-reduce by SM stores over NVLink (each partial row stored into its owner's "
                  "receive slot, the owner's sum of its slots stored into every rank's sum buffer), then the bias + "
                  "gated residual from each rank's own sums")
    paths = sorted([(f_ms, fused_mode, sp), (n_ms, nccl_mode, sp_n), (p_ms, p2p_mode, sp_p), (q_ms, push_mode, sp_q),
                    (s_ms, store_mode, sp_s)], key=lambda x: x[0])
    ms, mode, split_us = paths[0]
    out.update({"mode": mode,
                "ms_per_step": round(ms, 5), "tflops": round((lin + att) / (ms * 1e-3) / 1e12, 2),
                "breakdown_us": {k: round(v, 1) for k, v in split_us.items()}, "categories_us": _tp_categories(split_us),
                "unsharded_ms_per_step": round(uns_ms, 5), "speedup_vs_1gpu": round(uns_ms / ms, 3),
                "unsharded_breakdown_us": ({k: round(v, 1) for k, v in uns_split.items()} if uns_split else None),
                "other_modes": [{"mode": md, "ms_per_step": round(t_, 5),
                                 "breakdown_us": {k: round(v, 1) for k, v in sp_.items()}} for t_, md, sp_ in paths[1:]],
                "allreduce_bytes_per_step": 3 * L * H * 2, "parity": parity,
                "parity_of": "the fused path (top level) and the peer-memory paths ('p2p', 'push', 'store'); the NCCL path's "
                             "sums differ from the peer-memory paths' only in summation order",
                "launch": "CUDA graph replay of the whole block pair (every path, the unsharded one included)"})
    del cf, cn, cp
    held.clear()
    torch.cuda.synchronize(dev)
    barrier()
    del comm
    return out


def run_reference_config4(args) -> None:
    """The reference's block pair at 1024^2 on one GPU (it has no tensor-parallel path): rank 0
    runs it; other ranks exit without work."""
    import oracle as oracle_mod

    world, rank, local = dist_setup()
    if rank != 0:
        return
    os.environ.setdefault("CUDA_VISIBLE_DEVICES", str(local))
    if not oracle_mod.ATTN_REF_PATH.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_attention.so was not built"}))
        return
    if _no_gpu_line():
        return
    import blocks

    ref = oracle_mod.AttnRef()
    with ClockSampler(local) as clk:
        per = _ref_blocks_ms(ref, T_1024, I_1024, args.steps, args.warmup, seed=4)
    lin, att = blocks.block_pair_flops(T_1024, I_1024)
    value = (lin + att) / (per * 1e-3) / 1e12
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (reference Philox, seed 4)",
        "config": {"workload": WORKLOAD_TP1024, "flop_per_step": lin + att, "parallelism": "none (1 GPU)"},
        "cpu_baseline": {"kind": "reference", "cores": 0, "value": round(value, 2), "unit": "TFLOP/s",
                         "sample": "the reference has no CPU path; its own block code on one B200"},
        "e2e": {"value": round(value, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "clocks": clk.summary()}), flush=True)


def run_engine_config4(args) -> None:
    """Config 4's block pair at 1024^2 on its own: tp1024_leg as the headline (1 GPU: unsharded;
    N GPUs: the fused tensor-parallel path, strong scaling)."""
    import datetime

    import torch

    import b2g
    import blocks

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    b2g.init()
    g = torch.Generator(device=dev).manual_seed(0)
    txt_w, img_w = blocks.random_stream(g, dev), blocks.random_stream(g, dev)
    sw = blocks.random_single(g, dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    n0 = b2g.launch_count()
    with ClockSampler(local) as clk:
        leg = tp1024_leg(args, torch, world, rank, dev, txt_w, img_w, sw, flush)
    launches = b2g.launch_count() - n0
    peaks = measured_peaks()
    per = leg["ms_per_step"]
    value = leg["tflops"]
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": leg["warmup"], "ms_per_step": per, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (torch Philox generator, seeds 0/4)",
        "config": {"workload": WORKLOAD_TP1024, "flop_per_step": leg["flop_per_step"], "parallelism": f"tp{world}",
                   "l2": "256 MB buffer written before every step, outside the events"},
        "roofline": {"bound": "tensor", "achieved": round(value / world, 2), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(value / world / peaks["bf16_tflops"], 4), "traffic": None,
                     "peak_source": peaks["source"] + " (burst bf16)",
                     "kernel": "whole step per GPU (GEMMs, attention, fused reductions, barriers)"},
        "clocks": clk.summary(), "gpu_launches": int(launches), "tp1024": leg,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


WORKLOAD5 = ("config5: the FP8 transformer at 512^2, one independent job per GPU: one double-stream + one "
             "single-stream block (T=512 txt + I=1024 img tokens) with every linear on E4M3 weights (one fp32 "
             "scale per output channel, absmax/448) and per-token E4M3 activations (modulated inputs, attention "
             "output, MLP hidden state and concat buffer quantised on the device), the bf16 path's epilogues; "
             "key mask on 400 of 512 txt tokens")
T5_LAYERS, T5_TOKENS, T5_D, T5_HEADS, T5_FF = 24, 512, 4096, 64, 10240


def t5_shapes() -> list:
    """(label, GEMMs in the launch, M, N, K) of one T5 layer's linears (t5.cuh:233-275)."""
    d, ff, L = T5_D, T5_FF, T5_TOKENS
    return [("qkv", 3, L, d, d), ("o", 1, L, d, d), ("wi0_wi1", 2, L, ff, d), ("wo", 1, L, d, ff)]


def t5_line(ms: float, what: str) -> dict:
    """The T5 leg's summary from its per-pass time."""
    d, ff, L = T5_D, T5_FF, T5_TOKENS
    gemm_flop = T5_LAYERS * 2.0 * L * (4 * d * d + 2 * ff * d + d * ff)
    att_flop = T5_LAYERS * 4.0 * L * L * d
    return {"ms": round(ms, 4), "tflops": round((gemm_flop + att_flop) / (ms * 1e-3) / 1e12, 2),
            "flop": gemm_flop + att_flop, "gemm_flop": gemm_flop,
            "workload": f"T5-XXL encoder GEMMs and attention for one prompt, {T5_LAYERS} layers x (7 linears + "
                        f"attention), {L} tokens, d_model {d}, FFN {ff}, 64 heads x 64, fp16 weights ~N(0, 0.02); "
                        + what}


def t5_encoder_leg(torch, b2g, dev, gen, stream, flush) -> dict:
    """The T5-XXL encoder's GEMMs and attention for one prompt (t5.cuh:233-275): per layer the
    reference's 7 linears (q, k, v, o 4096x4096; wi_0, wi_1 10240x4096; wo 4096x10240) on fp16
    weights with F32 activations cast to fp16 as linear() casts them (cublas_ops.cuh:491-495),
    F32 outputs, wi_0 with the GELU epilogue, and t5_attention (64 heads x 64, relative-position
    bias, scale 1).  q, k and v read one input: one cast and one grouped launch (gemm_group);
    wi_0 and wi_1 share their input's cast.  The elementwise ops between them (RMSNorm,
    residual adds, the gate product) are not part of this leg: every layer reads the same
    synthetic F32 input."""
    d, ff, L, H = T5_D, T5_FF, T5_TOKENS, T5_HEADS
    ws = [{k: (torch.randn(shape, generator=gen, device=dev) * 0.02).half()
           for k, shape in (("q", (d, d)), ("k", (d, d)), ("v", (d, d)), ("o", (d, d)), ("wi0", (ff, d)),
                            ("wi1", (ff, d)), ("wo", (d, ff)))} for _ in range(T5_LAYERS)]
    x = torch.randn((L, d), generator=gen, device=dev)
    bias = torch.randn((H, L, L), generator=gen, device=dev) * 0.5
    q, k, v, att, o = (torch.empty((L, d), device=dev) for _ in range(5))
    h0, h1, y = torch.empty((L, ff), device=dev), torch.empty((L, ff), device=dev), torch.empty((L, d), device=dev)

    def layers():
        for w in ws:
            b2g.gemm_group([dict(x=x, w=w["q"], out=q), dict(x=x, w=w["k"], out=k), dict(x=x, w=w["v"], out=v)])
            b2g.t5_attention(q.view(L, H, d // H), k.view(L, H, d // H), v.view(L, H, d // H), bias, H, d // H,
                             out=att)
            b2g.gemm(att, w["o"], out=o)
            b2g.gemm_group([dict(x=x, w=w["wi0"], out=h0, epilogue="gelu"), dict(x=x, w=w["wi1"], out=h1)])
            b2g.gemm(h0, w["wo"], out=y)

    layers()
    torch.cuda.synchronize(dev)
    n0 = b2g.launch_count()
    g = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            layers()
    launches = b2g.launch_count() - n0
    for _ in range(3):
        g.replay()
    times = []
    for i in range(5):
        flush.fill_(i & 0xFF)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.replay()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b))
    del g
    # Per-launch split: every layer's launches eagerly, events between them, median over layers.
    w0 = ws[0]
    ops = {"qkv": lambda: b2g.gemm_group([dict(x=x, w=w0["q"], out=q), dict(x=x, w=w0["k"], out=k),
                                          dict(x=x, w=w0["v"], out=v)]),
           "attention": lambda: b2g.t5_attention(q.view(L, H, d // H), k.view(L, H, d // H), v.view(L, H, d // H),
                                                 bias, H, d // H, out=att),
           "o": lambda: b2g.gemm(att, w0["o"], out=o),
           "wi0_wi1": lambda: b2g.gemm_group([dict(x=x, w=w0["wi0"], out=h0, epilogue="gelu"),
                                              dict(x=x, w=w0["wi1"], out=h1)]),
           "wo": lambda: b2g.gemm(h0, w0["wo"], out=y)}
    per = {}
    for lab, fn in ops.items():
        ts = []
        for i in range(9):
            flush.fill_(i & 0xFF)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            b.synchronize()
            ts.append(a.elapsed_time(b))
        per[lab] = statistics.median(ts)
    hbm = measured_peaks()["hbm_gbs"]
    split = {}
    for lab, n, M, N, K in t5_shapes():
        byts = n * N * K * 2 + M * K * 4 + n * M * N * 4  # fp16 weights, the F32 input once, F32 outputs
        gbs = byts / (per[lab] * 1e-3) / 1e9
        split[lab] = {"us": round(1e3 * per[lab], 1), "tflops": round(n * 2.0 * M * N * K / (per[lab] * 1e-3) / 1e12, 1),
                      "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 3)}
    split["attention"] = {"us": round(1e3 * per["attention"], 1)}
    out = t5_line(statistics.median(times),
                  "F32 activations cast to fp16 (q/k/v and wi_0/wi_1 share their input's cast; q/k/v one launch); "
                  "one CUDA graph; L2 flushed before each of 5 timed passes (median); per_launch: each launch "
                  "alone, eager, L2 flushed, median of 9")
    out.update({"launches": launches, "per_launch": split})
    return out


def fp8_library_peak(torch, dev, n: int = 8192, reps: int = 10) -> dict | None:
    """A measured FP8 denominator, made the way MEASURED_PEAKS.json's bf16 one is (a library GEMM
    timed in a burst): torch._scaled_mm (cuBLASLt) on E4M3 [n, n] x [n, n]^T with unit scales,
    bf16 out, best of `reps` CUDA-event timings.  None where torch has no FP8 GEMM."""
    if not hasattr(torch, "_scaled_mm") or not hasattr(torch, "float8_e4m3fn"):
        return None
    g = torch.Generator(device=dev).manual_seed(5)
    a = torch.randn((n, n), generator=g, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn((n, n), generator=g, device=dev).to(torch.float8_e4m3fn)
    one = torch.ones((), device=dev)
    try:
        for _ in range(3):
            torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
    except (RuntimeError, TypeError):
        return None
    return {"tflops": round(2.0 * n ** 3 / (best * 1e-3) / 1e12, 1),
            "how": f"torch._scaled_mm (cuBLASLt) E4M3 {n}^3, unit scales, bf16 out, best of {reps} (burst)"}


def run_engine_config5(args) -> None:
    """Config 5 per GPU (data-parallel replicas, weak scaling): the FP8 block pair timed like
    config 2, the T5 encoder leg, and end to end the FP8 57-block pass over both guidance
    halves with its host I/O."""
    import torch

    import b2g
    import blocks

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    b2g.init()
    T, I = T_TXT, I_IMG
    L = T + I
    H = blocks.HIDDEN
    gdev = torch.Generator(device=dev).manual_seed(0)
    txt_w8 = blocks.quantize_stream(blocks.random_stream(gdev, dev))
    img_w8 = blocks.quantize_stream(blocks.random_stream(gdev, dev))
    sw8 = blocks.quantize_single(blocks.random_single(gdev, dev))
    ang = torch.rand((L, blocks.DHEAD // 2), generator=gdev, device=dev) * 6.2831853
    pe = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).contiguous()
    mask = torch.zeros(L, device=dev)
    mask[T - MASKED:T] = float("-inf")
    q8 = {k: blocks.Q8(*b2g.quantize_e4m3(torch.randn((rows, H), generator=gdev, device=dev).to(torch.bfloat16)))
          for k, rows in (("txt_mod1", T), ("img_mod1", I), ("txt_mod2", T), ("img_mod2", I), ("x_mod", L))}
    res = {k: torch.randn((rows, H), generator=gdev, device=dev) for k, rows in (("txt", T), ("img", I), ("x", L))}
    gt = torch.randn((5, H), generator=gdev, device=dev)
    s8 = blocks.ScratchFP8(T, I, dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step(mark=None):
        blocks.double_block_attention_fp8(txt_w8, img_w8, q8["txt_mod1"], q8["img_mod1"], res["txt"], res["img"],
                                          gt[0], gt[1], pe, mask, s8, mark)
        blocks.double_block_mlp_fp8(txt_w8, img_w8, q8["txt_mod2"], q8["img_mod2"], res["txt"], res["img"], gt[2],
                                    gt[3], s8, mark)
        blocks.single_block_fp8(sw8, q8["x_mod"], res["x"], gt[4], pe, mask, s8, mark)

    step()
    torch.cuda.synchronize(dev)
    cap = torch.cuda.Stream(dev)
    n0 = b2g.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            step()
    launches_per_step = b2g.launch_count() - n0
    marks = _Marks(torch, cap)
    marked = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(marked, stream=cap):
            marks.begin()
            step(marks)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        graph.replay()
    barrier()
    per_step = []
    with ClockSampler(local) as clk:
        barrier()
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            graph.replay()
            b.record(stream)
            b.synchronize()
            per_step.append(a.elapsed_time(b))
        barrier()
    total_ms = sum(per_step)
    per_op = {}
    for i in range(max(3, min(args.steps, 20))):
        flush.fill_(i & 0xFF)
        marked.replay()
        torch.cuda.synchronize(dev)
        for lab, ms in marks.durations().items():
            per_op.setdefault(lab, []).append(ms)
    b2g.check_device_error()
    del graph, marked
    t5 = t5_encoder_leg(torch, b2g, dev, torch.Generator(device=dev).manual_seed(3), stream, flush)

    # End to end: the FP8 57-block pass over both guidance halves, as config 2's e2e.
    pw = blocks.random_pass(gdev, dev)
    pw8 = blocks.quantize_pass(pw)
    del pw
    torch.cuda.empty_cache()
    ps = blocks.ScratchFP8(T, I, dev, halves=CFG_HALVES)
    gp = torch.Generator().manual_seed(2)
    x_h = torch.randn((CFG_HALVES * L, H), generator=gp).pin_memory()
    mods_h = (torch.randn(tuple(pw8.mods.shape), generator=gp) * 0.1).pin_memory()
    img_h = torch.empty((CFG_HALVES, I, H)).pin_memory()
    x_d = torch.empty((CFG_HALVES * L, H), device=dev)
    x_d.copy_(x_h)
    pw8.mods.copy_(mods_h)
    masks = torch.zeros((CFG_HALVES, L), device=dev)
    masks[0] = mask
    masks[1:, UNCOND_TEXT_KEYS:T] = float("-inf")
    blocks.forward_pass_fp8(pw8, x_d, pe, masks, ps, T)
    torch.cuda.synchronize(dev)
    n0 = b2g.launch_count()
    pass_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(pass_graph, stream=cap):
            blocks.forward_pass_fp8(pw8, x_d, pe, masks, ps, T)
    pass_launches = b2g.launch_count() - n0

    def pass_step():
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        x_d.copy_(x_h, non_blocking=True)
        pw8.mods.copy_(mods_h, non_blocking=True)
        pass_graph.replay()
        for h in range(CFG_HALVES):
            img_h[h].copy_(x_d[h * L + T:(h + 1) * L], non_blocking=True)
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b)

    for _ in range(2):
        pass_step()
    pass_ms = statistics.mean(pass_step() for _ in range(5))
    pass_flop = blocks.pass_flops(T, I, halves=CFG_HALVES)
    b2g.check_device_error()
    del pass_graph

    if world > 1:
        t = torch.tensor([total_ms, pass_ms, t5["ms"]], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms, pass_ms, t5_ms = float(t[0]), float(t[1]), float(t[2])
        t5["ms"] = round(t5_ms, 4)
        t5["tflops"] = round(t5["flop"] / (t5_ms * 1e-3) / 1e12, 2)
    ops = blocks.block_pair_ops_fp8(T, I)
    flop_step = sum(f for _, _, f in ops)
    per = total_ms / args.steps
    mean_op = {lab: statistics.mean(v) for lab, v in per_op.items()}
    marked_ms = sum(mean_op.values())
    fit = per / marked_ms if marked_ms > 0 else 1.0
    mean_op = {lab: v * fit for lab, v in mean_op.items()}
    gemm_flop = sum(f for _, kind, f in ops if kind == "gemm")
    gemm_ms = sum(mean_op[lab] for lab, kind, _ in ops if kind == "gemm")
    peaks = measured_peaks()
    lib8 = fp8_library_peak(torch, dev)
    fp8_peak = lib8["tflops"] if lib8 else 2.0 * peaks["bf16_tflops"]
    fp8_src = (f"measured in this run: {lib8['how']}" if lib8 else
               "derived: 2 x " + peaks["source"] + " bf16 burst (kind::f8f6f4 issues twice the bf16 rate)")
    achieved = gemm_flop / (gemm_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(flop_step * args.steps * world / (total_ms * 1e-3) / 1e12, 2),
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 (fp32 accumulate)",
        "data": "synthetic (torch Philox generators, seeds 0-3)",
        "config": {"workload": WORKLOAD5, "flop_per_step": flop_step, "parallelism": f"replicas x{world}",
                   "l2": "E4M3 weights 340 MB > L2; 256 MB buffer written before every step, outside the events",
                   "execution": "one CUDA graph per step"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(fp8_peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / fp8_peak, 4),
                     "traffic": profile_traffic("fp8_block_pair_config5_launches.md"),
                     "peak_source": fp8_src, "derived_peak_2x_bf16": round(2.0 * peaks["bf16_tflops"], 1),
                     "kernel": "tc_gemm E4M3: the block pair's 6 linear-layer launches, FLOP-weighted",
                     "gemm_ms_per_step": round(gemm_ms, 5)},
        "breakdown_us": {lab: round(1e3 * mean_op[lab], 1) for lab, _, _ in ops},
        "t5_encoder": t5,
        "e2e": {"value": round(pass_flop * world / (pass_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": x_h.numel() * 4 + mods_h.numel() * 4, "d2h_bytes_per_step": img_h.numel() * 4,
                "ms_per_step": round(pass_ms, 4),
                "workload": f"the FP8 block loop at 512^2 through the public API: both guidance halves through "
                            f"{blocks.DOUBLE_BLOCKS} double + {blocks.SINGLE_BLOCKS} single blocks with their own "
                            f"E4M3 weights, every block's inputs modulated into E4M3 on the device "
                            f"(modulate_to_e4m3); host I/O as config2's e2e; one CUDA graph of {pass_launches} "
                            f"launches", "flop_per_step": pass_flop},
        "clocks": clk.summary(),
        "gpu_launches": int(launches_per_step * args.steps),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


NERF_P, NERF_S, NERF_HID, NERF_MLP, NERF_COND = 1024, 256, 64, 256, 3072
NERF_PARAMS = 3 * NERF_HID * NERF_MLP  # 49152 param_gen outputs per patch: w_gate, w_value, w_fc2
WORKLOAD_NERF = ("nerf: the GEMMs of one NeRF decoder GLU block at 512^2 (nerf_glu_block, chroma.cuh:1253-1302), "
                 "P=1024 patches x 256 pixels x 64 channels: param_gen linear F32 s [1024, 3072] x bf16 W "
                 "[49152, 3072]^T + F32 bias -> F32 params (linear(): activations rounded to bf16), then "
                 "batched_matmul_Bt x3 (x [P,256,64] . w_gate/w_value [P,256,64]^T -> [P,256,256]; h [P,256,256] "
                 ". w_fc2 [P,64,256]^T -> [P,256,64], F32, operands rounded as cuBLAS's FAST_16BF mode does)")


def nerf_inputs(torch, dev):
    """Seeded inputs of one NeRF GLU block's GEMMs (weights ~N(0, 0.02), activations ~N(0, 1))."""
    g = torch.Generator(device=dev).manual_seed(7)
    P, S, D, F = NERF_P, NERF_S, NERF_HID, NERF_MLP
    t = {"s": torch.randn((P, NERF_COND), generator=g, device=dev),
         "w": (torch.randn((NERF_PARAMS, NERF_COND), generator=g, device=dev) * 0.02).to(torch.bfloat16),
         "b": torch.randn(NERF_PARAMS, generator=g, device=dev) * 0.02,
         "x": torch.randn((P, S, D), generator=g, device=dev),
         "wg": torch.randn((P, F, D), generator=g, device=dev) * 0.125,
         "wv": torch.randn((P, F, D), generator=g, device=dev) * 0.125,
         "w2": torch.randn((P, D, F), generator=g, device=dev) * 0.0625}
    t["params"] = torch.empty((P, NERF_PARAMS), device=dev)
    t["x1"] = torch.empty((P, S, F), device=dev)
    t["x2"] = torch.empty((P, S, F), device=dev)
    t["out"] = torch.empty((P, S, D), device=dev)
    return t


def nerf_flops() -> dict:
    P, S, D, F = NERF_P, NERF_S, NERF_HID, NERF_MLP
    return {"param_gen": 2.0 * P * NERF_PARAMS * NERF_COND, "gate": 2.0 * P * S * F * D, "value": 2.0 * P * S * F * D,
            "fc2": 2.0 * P * S * D * F}


def nerf_step_ops(t, linear, bmm) -> list:
    """The four GEMMs of the block, as (label, callable) in the reference's order."""
    P, S, D, F = NERF_P, NERF_S, NERF_HID, NERF_MLP
    return [("param_gen", lambda: linear(t["s"], t["w"], t["b"], t["params"])),
            ("gate", lambda: bmm(t["x"], t["wg"], t["x1"])),
            ("value", lambda: bmm(t["x"], t["wv"], t["x2"])),
            ("fc2", lambda: bmm(t["x1"], t["w2"], t["out"]))]


def time_ops(torch, ops, steps, warmup, flush, graph: bool) -> tuple[float, dict]:
    """Mean ms of the whole step (the ops in order) and of each op alone, CUDA events on the
    current stream, L2 flushed before every timed step; graph=True replays CUDA graphs."""
    def runner(fns):
        if not graph:
            return lambda: [f() for f in fns]
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(g, stream=cap):
                for f in fns:
                    f()
        return g.replay

    def timed(run, n):
        for _ in range(warmup):
            run()
        torch.cuda.synchronize()
        tot = 0.0
        for i in range(n):
            flush.fill_(i & 0xFF)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            run()
            b.record()
            b.synchronize()
            tot += a.elapsed_time(b)
        return tot / n

    fns = [f for _, f in ops]
    for f in fns:
        f()  # sizes any workspace before capture
    torch.cuda.synchronize()
    step = timed(runner(fns), steps)
    per = {lab: timed(runner([f]), max(3, steps // 4)) for lab, f in ops}
    return step, per


def nerf_line(impl, args, step_ms, per_ms, extra) -> dict:
    fl = nerf_flops()
    total = sum(fl.values())
    line = {"metric": METRIC, "value": round(total / (step_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (param_gen), tf32-rounded f32 (batched)",
            "data": "synthetic (torch Philox generator, seed 7)",
            "config": {"workload": WORKLOAD_NERF, "flop_per_step": total,
                       "l2": "256 MB buffer written before every step, outside the events"},
            "breakdown_us": {k: round(v * 1e3, 1) for k, v in per_ms.items()},
            "breakdown_tflops": {k: round(fl[k] / (per_ms[k] * 1e-3) / 1e12, 1) for k in per_ms}}
    if impl == "reference":
        line["impl"] = "reference"
    line.update(extra)
    return line


def run_engine_nerf(args) -> None:
    import types

    import torch

    import b2g

    world, rank, local = dist_setup()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    b2g.init()
    t = nerf_inputs(torch, dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    ops = nerf_step_ops(t, b2g.linear, b2g.batched_matmul_Bt)
    n0 = b2g.launch_count()
    for _, f in ops:
        f()
    launches = b2g.launch_count() - n0
    # Eager on stream 0, as the reference arm: linear() and batched_matmul_Bt mirror the
    # reference's stream-0 calls.
    with ClockSampler(local) as clk:
        step_ms, per = time_ops(torch, ops, args.steps, args.warmup, flush, graph=False)
    b2g.check_device_error()
    peaks = measured_peaks()
    fl = nerf_flops()
    ach = fl["param_gen"] / (per["param_gen"] * 1e-3) / 1e12
    # End to end: s copied in from pinned host memory and the block's output copied back.
    s_h = t["s"].cpu().pin_memory()
    out_h = torch.empty(t["out"].shape).pin_memory()
    ops_e2e = [("in", lambda: t["s"].copy_(s_h, non_blocking=True))] + ops + \
              [("out", lambda: out_h.copy_(t["out"], non_blocking=True))]
    e2e_ms, _ = time_ops(torch, ops_e2e, max(3, args.steps // 2), args.warmup, flush, graph=False)
    # The engine's own path for the whole block: the cast of s, param_gen and nerf_glu_kernel
    # (weight preparation, rms_norm, the three products, silu_mul and the residual add fused).
    blk = types.SimpleNamespace(param_w=t["w"], param_b=t["b"], norm=torch.ones(NERF_HID, device=dev))
    glu = nerf_glu_leg(torch, dev, flush, torch.cuda.current_stream(dev), NERF_P, args.steps,
                       m=types.SimpleNamespace(nerf=[blk]))
    line = nerf_line("b2g", args, step_ms, per, {
        "glu_block": glu,
        "roofline": {"bound": "tensor", "achieved": round(ach, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(ach / peaks["bf16_tflops"], 4), "traffic": None,
                     "peak_source": peaks["source"] + " (burst bf16)",
                     "kernel": "tc_gemm: the param_gen linear (92% of the step's FLOPs)"},
        "e2e": {"value": round(sum(fl.values()) / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": s_h.numel() * 4, "d2h_bytes_per_step": out_h.numel() * 4,
                "ms_per_step": round(e2e_ms, 4)},
        "clocks": clk.summary(), "gpu_launches": int(launches * args.steps)})
    print(json.dumps(line), flush=True)


def run_reference_nerf(args) -> None:
    """The reference's own linear() and batched_matmul_Bt (cuBLASLt / cuBLAS, built from its
    sources into oracle/_ref) on the same inputs, eager on stream 0 as the reference runs them."""
    world, rank, local = dist_setup()
    if rank != 0:
        return
    import oracle as oracle_mod
    import torch

    if not oracle_mod.REF_PATH.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_cublaslt.so was not built "
                          "(the reference sources were absent at build time)"}))
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ref = oracle_mod.Ref()
    t = nerf_inputs(torch, dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def linear(x, w, b, out):
        ref.linear(x.data_ptr(), 0, w.data_ptr(), 2, b.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1], w.shape[0])

    def bmm(a, b, c):
        ref.batched_matmul_Bt(a.data_ptr(), b.data_ptr(), c.data_ptr(), a.shape[0], a.shape[1], a.shape[2], b.shape[1])

    ops = nerf_step_ops(t, linear, bmm)
    with ClockSampler(local) as clk:
        step_ms, per = time_ops(torch, ops, args.steps, args.warmup, flush, graph=False)
    line = nerf_line("reference", args, step_ms, per, {
        "cpu_baseline": {"kind": "reference", "cores": 0, "value": round(sum(nerf_flops().values()) /
                                                                         (step_ms * 1e-3) / 1e12, 2),
                         "unit": "TFLOP/s", "sample": "the reference has no CPU path; this arm is its own linear() "
                                                      "and batched_matmul_Bt (cublas_ops.cuh:359, 558) on the B200"},
        "e2e": {"value": round(sum(nerf_flops().values()) / (step_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "clocks": clk.summary(), "cublaslt_version": int(ref.cublaslt_version())})
    print(json.dumps(line), flush=True)


def run_engine_skinny(args) -> None:
    """The approximator alone (the weight-streaming M=344 GEMMs, 556 MB of bf16 weights) on
    random weights of its shapes, through model.ChromaRadiance.compute_modulation's own code:
    approximator_leg's median, HBM GB/s and per-GEMM split.  Small enough for a full ncu
    capture of its GEMMs."""
    import types

    import torch

    import b2g
    import model

    world, rank, local = dist_setup()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    b2g.init()
    g = torch.Generator(device=dev).manual_seed(42)
    A, Hd, R = model.APPROX_DIM, model.HIDDEN, model.MOD_ROWS

    def w(n, k):
        return (torch.randn((n, k), generator=g, device=dev) * 0.02).to(torch.bfloat16)

    def b(n):
        return torch.randn(n, generator=g, device=dev) * 0.02

    ap = types.SimpleNamespace(in_proj_w=w(A, 64), in_proj_b=b(A), out_proj_w=w(Hd, A), out_proj_b=b(Hd),
                               ones=torch.ones(A, device=dev),
                               approx=[model.ApproxLayer(1 + b(A), w(A, A), b(A), w(A, A), b(A))
                                       for _ in range(model.APPROX_LAYERS)])
    sc = types.SimpleNamespace(timestep=torch.full((1,), FC_TIMESTEP, device=dev),
                               vec=torch.empty((R, 64), device=dev), ax=torch.empty((R, A), device=dev),
                               an=torch.empty((R, A), dtype=torch.bfloat16, device=dev),
                               ah=torch.empty((R, A), dtype=torch.bfloat16, device=dev),
                               mod=torch.empty((R, Hd), device=dev))
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    n0 = b2g.launch_count()
    with ClockSampler(local) as clk:
        leg = approximator_leg(torch, dev, flush, stream,
                               lambda mark=None: model.ChromaRadiance.compute_modulation(ap, sc, mark), args.steps)
    launches = b2g.launch_count() - n0
    b2g.check_device_error()
    peaks = measured_peaks()
    print(json.dumps({
        "metric": METRIC, "value": leg["tflops"], "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": 3, "ms_per_step": round(leg["us"] / 1e3, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (torch Philox, seed 42)",
        "config": {"workload": "skinny: " + leg["workload"], "parallelism": "none (1 GPU)",
                   "l2": "256 MB buffer written before every call, outside the events"},
        "roofline": {"bound": "hbm", "achieved": leg["hbm_gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": leg["hbm_frac"], "traffic": None, "peak_source": peaks["source"] + " (copy GB/s)",
                     "kernel": "tc_gemm_kernel: the approximator's 12 GEMMs"},
        "approximator": leg, "clocks": clk.summary(), "gpu_launches": int(launches)}), flush=True)


def run_engine_config3(args) -> None:
    """Config 3 alone: the whole denoising step at 512^2 (forward_cfg_leg) on rank 0, the e2e of
    the default line without the block-pair, TP and drop-in legs."""
    import torch

    import b2g

    world, rank, local = dist_setup()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    b2g.init()
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    n0 = b2g.launch_count()
    with ClockSampler(local) as clk:
        fc = forward_cfg_leg(args, torch, dev, flush, dropin=False)
    launches = b2g.launch_count() - n0
    value = fc["flop_per_step"] / (fc["ms_per_step"] * 1e-3) / 1e12
    print(json.dumps({
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": 1, "steps": fc["steps"],
        "warmup": args.warmup, "ms_per_step": round(fc["ms_per_step"], 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (torch Philox, seed 42)",
        "config": {"workload": WORKLOAD3, "flop_per_step": fc["flop_per_step"], "parallelism": "none (1 GPU)",
                   "l2": "256 MB buffer written before every step, outside the events"},
        "e2e": dict(fc, value=round(value, 3)), "clocks": clk.summary(), "gpu_launches": int(launches)}),
        flush=True)


def main():
    # The fused tensor-parallel path needs plain peer mappings only; keep torch's symmetric
    # memory from binding its buffers to an NVLink multicast object.
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 100 for config2, 200 config1)")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b2g", "reference"], default="b2g")
    ap.add_argument("--workload", choices=["config2", "config1", "config3", "config4", "config5", "nerf", "skinny"], default="config2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp1024", action="store_true", help="skip the 1024^2 tensor-parallel leg")
    ap.add_argument("--no-dropin", action="store_true", help="skip the drop-in build's forward_cfg")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.steps is None:
        args.steps = {"config2": 100, "config1": 200, "config3": 10, "config4": 30, "skinny": 30, "config5": 100, "nerf": 40}[args.workload]
    fn = {("b2g", "config1"): run_engine_config1, ("reference", "config1"): run_reference_config1,
          ("b2g", "config2"): run_engine_config2, ("reference", "config2"): run_reference_config2,
          ("b2g", "config3"): run_engine_config3,
          ("b2g", "skinny"): run_engine_skinny,
          ("reference", "skinny"): lambda a: print(json.dumps({
              "impl": "reference", "unavailable": "the reference's approximator runs inside its forward_cfg build; "
                                                  "its time is the 'approximator' object of the default reference "
                                                  "line"})),
          ("reference", "config3"): lambda a: print(json.dumps({
              "impl": "reference", "unavailable": "config 3 alone has no reference line: the reference's forward_cfg "
                                                  "is the e2e of the default (config2) reference arm"})),
          ("b2g", "config4"): run_engine_config4, ("b2g", "config5"): run_engine_config5,
          ("b2g", "nerf"): run_engine_nerf, ("reference", "nerf"): run_reference_nerf,
          ("reference", "config5"): lambda a: print(json.dumps({
              "impl": "reference", "unavailable": "the reference has no FP8 path (its quantised linears are INT8, "
                                                  "cublas_ops.cuh:294-791); its bf16 block code is the config2 "
                                                  "reference arm"})),
          ("reference", "config4"): run_reference_config4}
    fn[(args.impl, args.workload)](args)


if __name__ == "__main__":
    main()
