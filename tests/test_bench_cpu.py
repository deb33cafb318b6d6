"""CPU checks of bench.py's bookkeeping: FLOP counts of the block pair (BASELINE: 347.89
GFLOP of linears and 28.99 GFLOP of attention per block at 512^2) and that every workload and
arm is wired to a function."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import blocks

REPO = Path(__file__).resolve().parents[1]


def test_block_pair_flops_match_baseline():
    lin, att = blocks.block_pair_flops(512, 1024)
    assert abs(lin / 2 - 347.89e9) < 0.01e9
    assert abs(att / 2 - 28.99e9) < 0.01e9
    ops = blocks.block_pair_ops(512, 1024)
    assert sum(f for _, _, f in ops) == lin + att


def test_bench_help_lists_workloads():
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--help"], capture_output=True, text=True)
    assert r.returncode == 0
    for w in ("config1", "config2", "config4", "config5", "nerf"):
        assert w in r.stdout


def test_reference_arm_without_gpu_reports_unavailable_or_runs():
    """Without a GPU the reference arms print one `unavailable` JSON line (the reference's path
    is GPU code only; config5 has no counterpart at all: no FP8 path)."""
    for w in ("config2", "config4", "config5"):
        r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--workload", w],
                           capture_output=True, text=True, timeout=120)
        assert r.returncode == 0
        assert '"unavailable"' in r.stdout


def test_fp8_block_pair_ops():
    """The FP8 block pair has the bf16 pair's FLOPs plus three zero-FLOP quantisation steps, each
    right after the operation whose output it quantises."""
    ops8 = blocks.block_pair_ops_fp8(512, 1024)
    ops = blocks.block_pair_ops(512, 1024)
    assert sum(f for _, _, f in ops8) == sum(f for _, _, f in ops)
    labels = [lab for lab, _, _ in ops8]
    assert [lab for lab, kind, _ in ops8 if kind == "quantize"] == ["double.quantize_attn", "double.quantize_h",
                                                                    "single.quantize_cat"]
    assert labels.index("double.quantize_attn") == labels.index("double.attention") + 1
    assert labels.index("single.quantize_cat") == labels.index("single.attention") + 1


def test_nerf_step_flops():
    """One NeRF GLU block's GEMMs at 512^2: param_gen 2*1024*49152*3072 and three batched
    products of 2*1024*256*256*64 each (chroma.cuh:1262-1302)."""
    sys.argv = ["bench.py"]
    sys.path.insert(0, str(REPO))
    import bench

    fl = bench.nerf_flops()
    assert bench.NERF_PARAMS == 3 * 64 * 256
    assert fl["param_gen"] == 2.0 * 1024 * 49152 * 3072
    assert fl["gate"] == fl["value"] == fl["fc2"] == 2.0 * 1024 * 256 * 256 * 64
