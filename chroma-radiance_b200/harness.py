"""ctypes binding of the forward_cfg harness (dropin/forward_cfg_harness.cu): the reference's own
ChromaRadiance::forward_cfg (chroma.cuh:1499-1584) on seeded random-init weights.

Two builds of the same harness exist:
  DROPIN_PATH  the reference's model code compiled through the drop-in headers, so every GEMM
               and attention runs in libb2g.so (dropin/build_reference_with_b2g.sh --shared);
  the stock build (the reference's cuBLASLt / cuDNN / cuBLAS code) lives with the test
               oracle (oracle/_ref/libref_model.so) and is loaded by path by its users.
Each build keeps its own model; weights and inputs are exported by checkpoint name, so another
implementation can run on the very same device buffers (`tensor`).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent
DROPIN_PATH = PKG / "dropin" / "build" / "libforward_cfg_harness_b2g.so"
DTYPES = {0: "float32", 1: "float16", 2: "bfloat16"}


class _Cai:
    """A device buffer exposed through __cuda_array_interface__ (zero-copy into torch)."""

    def __init__(self, ptr: int, numel: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class ForwardCfgHarness:
    def __init__(self, path: str | Path):
        self.path = Path(path)
        lib = ctypes.CDLL(str(self.path), mode=ctypes.RTLD_LOCAL)
        i64, vp = ctypes.c_int64, ctypes.c_void_p
        lib.fc_setup.argtypes = [ctypes.c_ulonglong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.fc_tensor.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_int),
                                  ctypes.POINTER(i64)]
        lib.fc_num_tensors.restype = ctypes.c_int
        lib.fc_tensor_name.argtypes = [ctypes.c_int]
        lib.fc_tensor_name.restype = ctypes.c_char_p
        lib.fc_forward.argtypes = [ctypes.c_float, ctypes.c_float]
        lib.fc_modulation.argtypes = [ctypes.c_float]
        lib.fc_nerf_decode.argtypes = [vp, vp]
        lib.fc_bench_nerf_glu_block.argtypes = [ctypes.c_int, vp, vp, i64, ctypes.c_int, ctypes.c_int, i64,
                                                ctypes.POINTER(ctypes.c_double)]
        lib.fc_bench_modulation.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_int, i64,
                                            ctypes.POINTER(ctypes.c_double)]
        lib.fc_bench.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int, i64,
                                 ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        self.lib = lib
        self.H = self.W = None

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{self.path.name}: {what} failed with CUDA error {rc}")

    def setup(self, seed: int, H: int, W: int, real_cond: int, real_uncond: int) -> None:
        """Random-init model (seed) and forward_cfg inputs for an H x W image; real_cond /
        real_uncond prompt tokens set the two key masks (one padding token more attends)."""
        self._check(self.lib.fc_setup(seed, H, W, real_cond, real_uncond), "fc_setup")
        self.H, self.W = H, W

    def names(self) -> list[str]:
        return [self.lib.fc_tensor_name(i).decode() for i in range(self.lib.fc_num_tensors())]

    def tensor(self, name: str):
        """The device buffer `name` as a flat torch tensor (a view, no copy)."""
        import torch

        p, dt, n = ctypes.c_void_p(), ctypes.c_int(), ctypes.c_int64()
        if self.lib.fc_tensor(name.encode(), ctypes.byref(p), ctypes.byref(dt), ctypes.byref(n)) != 0:
            raise KeyError(name)
        if dt.value == 0:
            return torch.as_tensor(_Cai(p.value, n.value, "<f4"), device="cuda")
        t = torch.as_tensor(_Cai(p.value, n.value, "<i2"), device="cuda")
        return t.view(torch.bfloat16 if dt.value == 2 else torch.float16)

    def forward(self, timestep: float, cfg_scale: float) -> None:
        """One forward_cfg; the result is tensor("velocity")."""
        self._check(self.lib.fc_forward(timestep, cfg_scale), "fc_forward")

    def modulation(self, timestep: float) -> None:
        """compute_modulation(timestep, 0) into tensor("mod") [344 * 3072]."""
        self._check(self.lib.fc_modulation(timestep), "fc_modulation")

    def nerf_decode(self, img, out) -> None:
        """nerf_decode of image rows img [P, 3072] (F32, device) into out [3 * H * W]."""
        self._check(self.lib.fc_nerf_decode(img.data_ptr(), out.data_ptr()), "fc_nerf_decode")

    def bench(self, timestep: float, cfg_scale: float, iters: int, warmup: int, flush_bytes: int) -> tuple:
        """(ms per step with resident inputs, ms per step with the step's inputs copied in and the
        velocity copied out), CUDA events on stream 0."""
        d, e = ctypes.c_double(), ctypes.c_double()
        self._check(self.lib.fc_bench(timestep, cfg_scale, iters, warmup, flush_bytes, ctypes.byref(d),
                                      ctypes.byref(e)), "fc_bench")
        return d.value / iters, e.value / iters

    def bench_modulation(self, timestep: float, iters: int, warmup: int, flush_bytes: int) -> list:
        """Per-call milliseconds of compute_modulation (the approximator), CUDA events on stream 0."""
        ms = (ctypes.c_double * iters)()
        self._check(self.lib.fc_bench_modulation(timestep, iters, warmup, flush_bytes, ms), "fc_bench_modulation")
        return list(ms)

    def bench_nerf_glu_block(self, blk: int, x, s, iters: int, warmup: int, flush_bytes: int) -> list:
        """Per-call milliseconds of the reference's nerf_glu_block `blk` on x F32 [P, 256, 64]
        (updated in place) and s F32 [P, 3072] (device tensors)."""
        ms = (ctypes.c_double * iters)()
        self._check(self.lib.fc_bench_nerf_glu_block(blk, x.data_ptr(), s.data_ptr(), x.shape[0], iters, warmup,
                                                     flush_bytes, ms), "fc_bench_nerf_glu_block")
        return list(ms)
