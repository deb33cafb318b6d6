"""Benchmark of the B200 GEMM engine on BASELINE config 1, plus the reference's own arm.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b2g|reference]

Workload (the single-stream linear1 GEMM at 512^2): X bf16
[1536, 3072] ~ N(0,1), W bf16 [21504, 3072] ~ N(0, 0.02), bias [21504] ~ N(0, 0.02) (bf16
values), seed 0, fp32 accumulation.  The engine writes a bf16 output; the reference's
linear_lt writes F32 (it has no bf16-output mode).  One "step" = one GEMM over that batch.
Inputs come from numpy (PCG64, seed 0), identical for both arms.

  value     TFLOP/s over all ranks: 2*M*N*K*steps*ranks / (max over ranks of the summed
            per-step CUDA-event time); inputs resident in HBM; L2 flushed (256 MB write)
            before every step, outside the event pair.
  e2e       same metric through the public API with host buffers: per step, X copied from
            pinned host memory, GEMM, output copied back, all inside the event pair.
  roofline  tensor-bound: achieved = algorithmic FLOP per launch / mean launch time of the
            GEMM kernel (events on its stream), peak = MEASURED_PEAKS.json bf16_tflops.
  cpu_baseline  the fp32 C oracle (oracle/oracle.c, OpenMP, all host cores) on a bounded
            sample of the same GEMM (rank 0, N=1 only).

--impl reference runs the reference's own linear_lt (cuBLASLt, compiled from its sources
into oracle/_ref/) on the same inputs, timed the same way, and never imports the engine.
Multi-GPU (torchrun): every rank runs its own replica (weak scaling, no collective on the
data path); rank 0 prints the line.
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


def profile_traffic() -> float | None:
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary, if any."""
    p = REPO / "profiles" / "tc_gemm_config1.md"
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
            "kind": "port", "sample": f"{rows2} of {M} rows of X against all of W ({rows2 * 2 * N * K / 1e9:.1f} "
                                      f"GFLOP, {dt:.1f} s, bf16 inputs widened to fp32, fp32 accumulate)"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args) -> None:
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


def run_engine(args) -> None:
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
                     "traffic": profile_traffic(), "peak_source": peaks["source"] + " (burst bf16)",
                     "kernel": "tc_gemm_kernel<256,4,none,bf16>"},
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


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b2g", "reference"], default="b2g")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
