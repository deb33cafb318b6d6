"""Tensor-parallel Chroma block pair (large images across 2/4/8 GPUs).

One process per GPU.  Each rank holds a slice of every block's weights, made once at load
time (the TP-shard layout of the weight arena):
  column-split (by heads / MLP columns, no communication):
      qkv      rows [q_h0:q_h1, k_h0:k_h1, v_h0:v_h1] of qkv_w      (24/TP heads per rank)
      mlp0     rows [m0:m1] of mlp0_w                                (12288/TP columns)
      linear1  rows q, k, v of the rank's heads + MLP rows [m0:m1]
  row-split (K-split) to match, producing a partial sum without bias:
      proj     columns [h0*128:h1*128] of proj_w   (a view: the GEMM reads any row stride)
      mlp2     columns [m0:m1] of mlp2_w           (a view)
      linear2  columns of the rank's heads and MLP slice, packed once into [3072, HDl+MLPl]
After each row-split layer one bf16 all-reduce (NCCL over NVLink) sums the partials of all
ranks; bias and the gated residual are then applied once, in F32 (b2g_bias_gated_residual).
Per block pair: 2 all-reduces in the double block (proj with txt and img rows together, then
the MLP) and 1 in the single block, of [L, 3072] bf16 each.  Attention, qk-norm and RoPE are
head-local.  Small images instead run one independent replica per GPU (bench.py config 2).

The compute steps go through an `ops` object (EngineOps: libb2g kernels + torch.distributed);
the CPU tests substitute an fp32 torch stand-in with gloo ranks to check the sharding logic.
"""
from __future__ import annotations

import collections
import datetime
import threading
import time
from dataclasses import dataclass

import torch

from blocks import DHEAD, HEADS, HIDDEN, MLP, SingleWeights, StreamWeights, _rope_table


@dataclass(frozen=True)
class Dims:
    """Block dimensions (Chroma: hidden 3072, 24 heads x 128, MLP 12288)."""

    hidden: int = HIDDEN
    heads: int = HEADS
    dhead: int = DHEAD
    mlp: int = MLP


# ---------------------------------------------------------------------------- failure handling
# The reference is single-GPU and exits on any error; the tensor-parallel path adds ranks that
# can fail independently.  Three layers keep a failure from turning into a hang:
#   * on the device, every wait of the engine's kernels (pipeline barriers, the cross-rank
#     barrier kernel) gives up after 2 s and reports through b2g_check_device_error;
#   * between steps, StepWatch: each rank posts its step number to the process group's store
#     and checks that every peer reached the previous one before launching the next, so a rank
#     that left is noticed on the host before any kernel waits for it;
#   * for NCCL collectives, a non-blocking communicator (nccl_options) and CollectiveWatchdog,
#     a host thread that aborts the communicator (ncclCommAbort) when a collective outlives its
#     deadline, so the pending all-reduce ends with an error instead of waiting for good.


class RankLost(RuntimeError):
    """A peer rank did not reach a step within the deadline (it left or stalled)."""


class CollectiveTimeout(RuntimeError):
    """A collective did not complete within the watchdog's deadline; its group was aborted."""


class StepWatch:
    """Host-side liveness check between tensor-parallel steps over a c10d store.

    arrive(step) posts this rank's arrival at `step`; check(step) waits (at most `timeout_s`)
    until every rank has posted `step` and raises RankLost naming the ranks that have not."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "b2g/step"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.prefix = prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def arrive(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), "1")

    def check(self, step: int) -> None:
        keys = [self._key(step, r) for r in range(self.world)]
        try:
            self.store.wait(keys, self.timeout)
        except Exception as e:  # the store raises on timeout; name who is missing
            missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
            raise RankLost(f"rank(s) {missing} did not reach step {step} within "
                           f"{self.timeout.total_seconds():.1f} s") from e


def nccl_options(blocking: bool = False):
    """ProcessGroupNCCL options with a non-blocking communicator (ncclCommInitRankConfig with
    blocking = 0): NCCL calls return at once, and an abort can end an in-flight collective."""
    import torch.distributed as dist

    opts = dist.ProcessGroupNCCL.Options()
    opts.config.blocking = 1 if blocking else 0
    return opts


class CollectiveWatchdog:
    """Tracks asynchronous collectives (objects with is_completed()) and calls `abort` once
    when one has been outstanding longer than `deadline_s`; the next track()/check() then
    raises CollectiveTimeout.  `poll()` does one pass (tests drive it with their own clock);
    start() runs it every `poll_s` seconds in a daemon thread."""

    def __init__(self, abort, deadline_s: float = 30.0, poll_s: float = 0.005, clock=time.monotonic):
        self.abort, self.deadline, self.poll_s, self.clock = abort, deadline_s, poll_s, clock
        self.pending = collections.deque()
        self.error: CollectiveTimeout | None = None
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread = None

    def track(self, work, label: str = "collective"):
        self.check()
        with self._lock:
            self.pending.append((work, self.clock(), label))
        return work

    def check(self) -> None:
        if self.error is not None:
            raise self.error

    def poll(self) -> None:
        with self._lock:
            while self.pending and self.pending[0][0].is_completed():
                self.pending.popleft()
            late = next(((lab, t) for w, t, lab in self.pending
                         if not w.is_completed() and self.clock() - t > self.deadline), None)
            if late is None or self.error is not None:
                return
            self.error = CollectiveTimeout(f"{late[0]} did not complete within {self.deadline:.1f} s; "
                                           f"the process group was aborted")
            self.pending.clear()
        self.abort()

    def _run(self) -> None:
        while not self._stop.wait(self.poll_s):
            self.poll()

    def start(self) -> "CollectiveWatchdog":
        self._thread = threading.Thread(target=self._run, name="b2g-collective-watchdog", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()


class EngineOps:
    """The product path: libb2g's tensor-core GEMMs, fused attention and bias/gate kernel,
    and an all-reduce over the default process group (NCCL on GPUs).  With a watchdog, each
    all-reduce is issued asynchronously and tracked, so a collective that never completes
    aborts the group instead of hanging the step."""

    def __init__(self, watchdog: CollectiveWatchdog | None = None):
        import b2g

        self.b2g = b2g
        self.watchdog = watchdog

    def gemm_group(self, problems):
        return self.b2g.gemm_group(problems)

    def gemm(self, x, w, bias=None, out=None, epilogue="none", gate=None):
        return self.b2g.gemm(x, w, bias, out=out, epilogue=epilogue, gate=gate)

    def qkv_rope(self, problems, n_head):
        return self.b2g.gemm_qkv_rope(problems, n_head)

    def attention_bf16(self, q, k, v, n_head, d_head, attn_mask=None, out=None):
        return self.b2g.attention_bf16(q, k, v, n_head, d_head, attn_mask=attn_mask, out=out)

    def bias_gated_residual(self, y, bias, gate, residual):
        self.b2g.bias_gated_residual(y, bias, gate, residual)

    def all_reduce(self, t):
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            if self.watchdog is None:
                dist.all_reduce(t)
            else:
                self.watchdog.track(dist.all_reduce(t, async_op=True), "all_reduce")


@dataclass
class TPStreamWeights:
    qkv_w: torch.Tensor   # [3*HDl, 3072]   q, k, v rows of this rank's heads
    qkv_b: torch.Tensor   # [3*HDl]
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    proj_w: torch.Tensor  # [3072, HDl] view (row stride 3072)
    proj_b: torch.Tensor  # [3072] full: applied after the all-reduce
    mlp0_w: torch.Tensor  # [MLPl, 3072]
    mlp0_b: torch.Tensor  # [MLPl]
    mlp2_w: torch.Tensor  # [3072, MLPl] view (row stride 12288)
    mlp2_b: torch.Tensor  # [3072] full


@dataclass
class TPSingleWeights:
    linear1_w: torch.Tensor  # [3*HDl + MLPl, 3072]
    linear1_b: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    linear2_w: torch.Tensor  # [3072, HDl + MLPl] packed
    linear2_b: torch.Tensor  # [3072] full


def _split(world: int, d: Dims) -> tuple[int, int]:
    if d.heads % world or d.mlp % world:
        raise ValueError(f"tensor parallelism {world} must divide {d.heads} heads and {d.mlp} MLP columns")
    return d.heads // world, d.mlp // world


def head_range(rank: int, world: int, d: Dims = Dims()) -> tuple[int, int]:
    hl, _ = _split(world, d)
    return rank * hl * d.dhead, (rank + 1) * hl * d.dhead


def mlp_range(rank: int, world: int, d: Dims = Dims()) -> tuple[int, int]:
    _, ml = _split(world, d)
    return rank * ml, (rank + 1) * ml


def shard_stream(w: StreamWeights, rank: int, world: int, d: Dims = Dims()) -> TPStreamWeights:
    c0, c1 = head_range(rank, world, d)
    m0, m1 = mlp_range(rank, world, d)
    qkv_rows = [slice(j * d.hidden + c0, j * d.hidden + c1) for j in range(3)]
    return TPStreamWeights(
        qkv_w=torch.cat([w.qkv_w[r] for r in qkv_rows]).contiguous(),
        qkv_b=torch.cat([w.qkv_b[r] for r in qkv_rows]).contiguous(),
        q_norm=w.q_norm, k_norm=w.k_norm,
        proj_w=w.proj_w[:, c0:c1], proj_b=w.proj_b,
        mlp0_w=w.mlp0_w[m0:m1], mlp0_b=w.mlp0_b[m0:m1],
        mlp2_w=w.mlp2_w[:, m0:m1], mlp2_b=w.mlp2_b)


def shard_single(w: SingleWeights, rank: int, world: int, d: Dims = Dims()) -> TPSingleWeights:
    c0, c1 = head_range(rank, world, d)
    m0, m1 = mlp_range(rank, world, d)
    H = d.hidden
    rows = [slice(j * H + c0, j * H + c1) for j in range(3)] + [slice(3 * H + m0, 3 * H + m1)]
    return TPSingleWeights(
        linear1_w=torch.cat([w.linear1_w[r] for r in rows]).contiguous(),
        linear1_b=torch.cat([w.linear1_b[r] for r in rows]).contiguous(),
        q_norm=w.q_norm, k_norm=w.k_norm,
        linear2_w=torch.cat([w.linear2_w[:, c0:c1], w.linear2_w[:, H + m0:H + m1]], dim=1).contiguous(),
        linear2_b=w.linear2_b)


class TPScratch:
    """Per-rank activation buffers of one block pair, allocated once."""

    def __init__(self, T: int, I: int, world: int, dev, d: Dims = Dims()):
        hl, ml = _split(world, d)
        L, HDl = T + I, hl * d.dhead
        self.d, self.hl, self.HDl, self.ml = d, hl, HDl, ml
        self.qkv = torch.empty((L, 3 * HDl), dtype=torch.bfloat16, device=dev)  # normed, rotated
        self.attn = torch.empty((L, HDl), dtype=torch.bfloat16, device=dev)
        self.part = torch.empty((L, d.hidden), dtype=torch.bfloat16, device=dev)
        self.h_txt = torch.empty((T, ml), dtype=torch.bfloat16, device=dev)
        self.h_img = torch.empty((I, ml), dtype=torch.bfloat16, device=dev)
        self.cat = torch.empty((L, HDl + ml), dtype=torch.bfloat16, device=dev)


def _no_mark(label: str) -> None:
    pass


def _qkv_attention_double(ops, txt_w: TPStreamWeights, img_w: TPStreamWeights, txt_mod1, img_mod1, pe, mask,
                          s: TPScratch, mark=_no_mark) -> None:
    """The rank's heads: qkv projections with qk_norm and RoPE in the epilogue (txt rows take
    pe rows [0, T), img rows [T, L)), then attention over the txt + img sequence into s.attn."""
    T, HDl = txt_mod1.shape[0], s.HDl
    pe = _rope_table(pe, s)
    ops.qkv_rope([dict(x=txt_mod1, w=txt_w.qkv_w, bias=txt_w.qkv_b, out=s.qkv[:T], pe=pe[:T],
                       q_norm=txt_w.q_norm, k_norm=txt_w.k_norm),
                  dict(x=img_mod1, w=img_w.qkv_w, bias=img_w.qkv_b, out=s.qkv[T:], pe=pe[T:],
                       q_norm=img_w.q_norm, k_norm=img_w.k_norm)], s.hl)
    mark("double.qkv")
    q, k, v = s.qkv[:, :HDl], s.qkv[:, HDl:2 * HDl], s.qkv[:, 2 * HDl:]
    ops.attention_bf16(q, k, v, s.hl, s.d.dhead, attn_mask=mask, out=s.attn)
    mark("double.attention")


def tp_double_block(ops, txt_w: TPStreamWeights, img_w: TPStreamWeights, txt_mod1, img_mod1, txt_mod2, img_mod2, txt,
                    img, txt_gate1, img_gate1, txt_gate2, img_gate2, pe, mask, s: TPScratch, mark=None) -> None:
    """This rank's share of double_block (chroma.cuh:808-964); txt, img replicated F32 streams.
    `mark(label)`, when given, is called after every step (timing events between them)."""
    T, HDl = txt.shape[0], s.HDl
    mk = mark or _no_mark
    _qkv_attention_double(ops, txt_w, img_w, txt_mod1, img_mod1, pe, mask, s, mk)
    ops.gemm_group([dict(x=s.attn[:T], w=txt_w.proj_w, out=s.part[:T]),
                    dict(x=s.attn[T:], w=img_w.proj_w, out=s.part[T:])])
    mk("double.proj")
    ops.all_reduce(s.part)
    mk("double.proj.all_reduce")
    ops.bias_gated_residual(s.part[:T], txt_w.proj_b, txt_gate1, txt)
    ops.bias_gated_residual(s.part[T:], img_w.proj_b, img_gate1, img)
    mk("double.proj.residual")
    ops.gemm_group([dict(x=txt_mod2, w=txt_w.mlp0_w, bias=txt_w.mlp0_b, out=s.h_txt, epilogue="gelu"),
                    dict(x=img_mod2, w=img_w.mlp0_w, bias=img_w.mlp0_b, out=s.h_img, epilogue="gelu")])
    mk("double.mlp0")
    ops.gemm_group([dict(x=s.h_txt, w=txt_w.mlp2_w, out=s.part[:T]),
                    dict(x=s.h_img, w=img_w.mlp2_w, out=s.part[T:])])
    mk("double.mlp2")
    ops.all_reduce(s.part)
    mk("double.mlp2.all_reduce")
    ops.bias_gated_residual(s.part[:T], txt_w.mlp2_b, txt_gate2, txt)
    ops.bias_gated_residual(s.part[T:], img_w.mlp2_b, img_gate2, img)
    mk("double.mlp2.residual")


def _linear1(ops, w: TPSingleWeights, x_mod, pe, s: TPScratch) -> None:
    """The rank's linear1 in one launch, as the unsharded block runs it: its q, k, v columns get
    qk_norm + RoPE into s.qkv, its MLP columns bias + GELU straight into the linear2 input
    s.cat[:, HDl:] (the split falls on a head boundary at every TP degree)."""
    ops.qkv_rope([dict(x=x_mod, w=w.linear1_w, bias=w.linear1_b, out=s.qkv, pe=_rope_table(pe, s),
                       q_norm=w.q_norm, k_norm=w.k_norm, gelu_out=s.cat[:, s.HDl:])], s.hl)


def tp_single_block(ops, w: TPSingleWeights, x_mod, x, gate, pe, mask, s: TPScratch, mark=None) -> None:
    """This rank's share of single_block (chroma.cuh:1101-1157); x the replicated F32 stream.
    `mark` as in tp_double_block."""
    HDl = s.HDl
    mk = mark or _no_mark
    _linear1(ops, w, x_mod, pe, s)
    mk("single.linear1")
    q, k, v = s.qkv[:, :HDl], s.qkv[:, HDl:2 * HDl], s.qkv[:, 2 * HDl:]
    ops.attention_bf16(q, k, v, s.hl, s.d.dhead, attn_mask=mask, out=s.cat[:, :HDl])
    mk("single.attention")
    ops.gemm(s.cat, w.linear2_w, out=s.part)
    mk("single.linear2")
    ops.all_reduce(s.part)
    mk("single.linear2.all_reduce")
    ops.bias_gated_residual(s.part, w.linear2_b, gate, x)
    mk("single.linear2.residual")


# ---------------------------------------------------------------------------- fused reduction
class SymmetricComm:
    """Peer-mapped (NVLink) buffers for the fused row-split layers (b2g_gemm_tp_reduce), made
    with torch's symmetric memory: a bf16 partial buffer [rows, hidden], two replicated F32
    residual copies (the double block's txt rows then img rows, and the single block's
    stream), and the tile arrival counters (rank 0's copy is the one used).  `barrier()` is the
    cross-rank barrier each fused layer needs before its outputs are read or its partial buffer
    is reused (b2g_tp_barrier_next on a peer-mapped flag array)."""

    COUNTER_SLOTS = 8192

    def __init__(self, rows: int, hidden: int, group, dev):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        import b2g

        self.b2g = b2g
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.part = symm.empty((rows, hidden), dtype=torch.bfloat16, device=dev)
        self.res_double = symm.empty((rows, hidden), dtype=torch.float32, device=dev)
        self.res_single = symm.empty((rows, hidden), dtype=torch.float32, device=dev)
        self.counters = symm.empty(self.COUNTER_SLOTS, dtype=torch.int32, device=dev)
        self.sums = symm.empty((rows, hidden), dtype=torch.bfloat16, device=dev)
        self.rows = rows
        shard = (rows + self.world - 1) // self.world
        self.recv = symm.empty((self.world, shard, hidden), dtype=torch.bfloat16, device=dev)
        self.flags = symm.empty(self.world, dtype=torch.int32, device=dev)
        self.counters.zero_()
        self.flags.zero_()
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        self._handles = [symm.rendezvous(t, name) for t in
                         (self.part, self.res_double, self.res_single, self.counters, self.flags, self.sums,
                          self.recv)]
        torch.cuda.synchronize(dev)
        dist.barrier(group)  # every rank's zeroed counters and flags are in place

        def peers(t, h):  # every rank's address of this tensor, in this process
            off = t.data_ptr() - h.buffer_ptrs[self.rank]
            return [p + off for p in h.buffer_ptrs]

        part = peers(self.part, self._handles[0])
        self._part_ptrs = torch.tensor(part, dtype=torch.int64, device=dev)
        self._res_ptrs = {name: torch.tensor(peers(t, h), dtype=torch.int64, device=dev) for name, t, h in
                          (("double", self.res_double, self._handles[1]),
                           ("single", self.res_single, self._handles[2]))}
        counters0 = peers(self.counters, self._handles[3])[0]
        self._flag_ptrs = torch.tensor(peers(self.flags, self._handles[4]), dtype=torch.int64, device=dev)
        self._sum_ptrs = torch.tensor(peers(self.sums, self._handles[5]), dtype=torch.int64, device=dev)
        self._recv_ptrs = torch.tensor(peers(self.recv, self._handles[6]), dtype=torch.int64, device=dev)
        self._recv_host = peers(self.recv, self._handles[6])     # for the copy-engine pushes
        self._sum_host = peers(self.sums, self._handles[5])
        self.epoch_ctr = torch.zeros(1, dtype=torch.int32, device=dev)   # the barrier's epoch, kept on the device
        self.desc = {}
        for name, t in (("double", self.res_double), ("single", self.res_single)):
            d = b2g.TpReduceDesc()
            d.world, d.rank = self.world, self.rank
            d.part_ptrs = self._part_ptrs.data_ptr()
            d.res_ptrs = self._res_ptrs[name].data_ptr()
            d.ld_part, d.ld_res = self.part.stride(0), t.stride(0)
            d.counters = counters0
            d.counter_slots = self.COUNTER_SLOTS
            self.desc[name] = d

    def reduce(self, which: str, problems: list[dict], row0: list[int], mark=None, label: str = "") -> None:
        """One row-split layer with its all-rank reduction fused into the GEMM, then the
        cross-rank barrier.  `mark(label)`, when given, is called after each of the two."""
        self.b2g.gemm_tp_reduce(problems, row0, self.desc[which])
        if mark:
            mark(label)
        self.barrier()
        if mark:
            mark(label + ".barrier")

    def reduce_p2p(self, segments: list[dict], mark=None, label: str = "") -> None:
        """The all-reduce of the bf16 partial in self.part (written by a plain row-split GEMM) over
        NVLink peer memory in two phases, each after a cross-rank barrier: this rank sums its
        shard of rows from every rank's partial into self.sums (b2g_tp_reduce_shard), then
        applies residual += gate * (sum + bias) from every rank's sums to its own residual
        segments (b2g_tp_gather_residual; dict(row0, bias, gate, residual))."""
        self.barrier()
        self.b2g.tp_reduce_shard(self._part_ptrs, self.sums, self.world, self.rank)
        if mark:
            mark(label + ".reduce")
        self.barrier()
        self.b2g.tp_gather_residual(self._sum_ptrs, self.sums, self.world, segments)
        if mark:
            mark(label + ".residual")

    def reduce_push(self, segments: list[dict], mark=None, label: str = "") -> None:
        """The all-reduce of self.part (written by a plain row-split GEMM) in the push form, every
        NVLink transfer a copy-engine copy: each shard of partial rows into its owner's receive
        slot (b2g_tp_push_rows), barrier, the owner sums its slots (b2g_tp_reduce_slots, local)
        and copies its sums to every rank (b2g_tp_push_sums), barrier, then each rank applies
        bias + gate from its own sum buffer (b2g_bias_gated_residual per segment:
        dict(row0, bias, gate, residual))."""
        self.b2g.tp_push_rows(self.part, self._recv_host, self.world, self.rank)
        self.barrier()
        self.b2g.tp_reduce_slots(self.recv, self.sums, self.world, self.rank)
        self.b2g.tp_push_sums(self._sum_host, self.sums, self.world, self.rank)
        if mark:
            mark(label + ".reduce")
        self.barrier()
        for g in segments:
            r = g["residual"]
            self.b2g.bias_gated_residual(self.sums[g["row0"]:g["row0"] + r.shape[0]], g.get("bias"), g["gate"], r)
        if mark:
            mark(label + ".residual")

    def reduce_store(self, segments: list[dict], mark=None, label: str = "") -> None:
        """The all-reduce of self.part in the store form, every NVLink transfer an SM store: each
        row of the partial into its owner's receive slot (b2g_tp_scatter_rows), barrier, the
        owner sums its slots and stores the sums into every rank's sum buffer
        (b2g_tp_reduce_slots_bcast), barrier, then each rank applies bias + gate from its own
        sums (b2g_bias_gated_residual per segment: dict(row0, bias, gate, residual))."""
        self.b2g.tp_scatter_rows(self.part, self._recv_ptrs, self.world, self.rank)
        self.barrier()
        self.b2g.tp_reduce_slots_bcast(self.recv, self._sum_ptrs, self.rows, self.part.shape[1], self.world,
                                       self.rank)
        if mark:
            mark(label + ".reduce")
        self.barrier()
        for g in segments:
            r = g["residual"]
            self.b2g.bias_gated_residual(self.sums[g["row0"]:g["row0"] + r.shape[0]], g.get("bias"), g["gate"], r)
        if mark:
            mark(label + ".residual")

    def barrier(self) -> None:
        """All ranks' fused layers are done (bounded wait in libb2g's own barrier kernel).  The
        epoch lives in device memory (b2g_tp_barrier_next), so a CUDA graph of a step that
        holds barriers replays correctly."""
        self.b2g.tp_barrier_next(self._flag_ptrs, self.flags, self.epoch_ctr, self.world, self.rank)


def tp_double_block_fused(ops, comm: SymmetricComm, txt_w: TPStreamWeights, img_w: TPStreamWeights, txt_mod1,
                          img_mod1, txt_mod2, img_mod2, txt_gate1, img_gate1, txt_gate2, img_gate2, pe, mask,
                          s: TPScratch, mark=None) -> None:
    """tp_double_block with each row-split layer's all-reduce fused into its GEMM: the
    replicated txt and img streams are comm.res_double[:T] and [T:].  `mark(label)`, when
    given, is called after every launch (for timing events between them)."""
    T, HDl = txt_mod1.shape[0], s.HDl
    _qkv_attention_double(ops, txt_w, img_w, txt_mod1, img_mod1, pe, mask, s, mark or _no_mark)
    comm.reduce("double", [dict(x=s.attn[:T], w=txt_w.proj_w, bias=txt_w.proj_b, gate=txt_gate1),
                           dict(x=s.attn[T:], w=img_w.proj_w, bias=img_w.proj_b, gate=img_gate1)], [0, T],
                mark, "double.proj")
    ops.gemm_group([dict(x=txt_mod2, w=txt_w.mlp0_w, bias=txt_w.mlp0_b, out=s.h_txt, epilogue="gelu"),
                    dict(x=img_mod2, w=img_w.mlp0_w, bias=img_w.mlp0_b, out=s.h_img, epilogue="gelu")])
    (mark or _no_mark)("double.mlp0")
    comm.reduce("double", [dict(x=s.h_txt, w=txt_w.mlp2_w, bias=txt_w.mlp2_b, gate=txt_gate2),
                           dict(x=s.h_img, w=img_w.mlp2_w, bias=img_w.mlp2_b, gate=img_gate2)], [0, T],
                mark, "double.mlp2")


def tp_single_block_fused(ops, comm: SymmetricComm, w: TPSingleWeights, x_mod, gate, pe, mask, s: TPScratch,
                          mark=None) -> None:
    """tp_single_block with linear2's all-reduce fused into its GEMM: the replicated stream is
    comm.res_single.  `mark` as in tp_double_block_fused."""
    HDl = s.HDl
    mk = mark or _no_mark
    _linear1(ops, w, x_mod, pe, s)
    mk("single.linear1")
    q, k, v = s.qkv[:, :HDl], s.qkv[:, HDl:2 * HDl], s.qkv[:, 2 * HDl:]
    ops.attention_bf16(q, k, v, s.hl, s.d.dhead, attn_mask=mask, out=s.cat[:, :HDl])
    mk("single.attention")
    comm.reduce("single", [dict(x=s.cat, w=w.linear2_w, bias=w.linear2_b, gate=gate)], [0], mark, "single.linear2")


def _row_split_p2p(ops, comm: SymmetricComm, problems: list[dict], row0: list[int], segments: list[dict], mk,
                   label: str, push) -> None:
    """One row-split layer (its GEMM writes comm.part) and its all-reduce + residual update over
    peer memory: pull form (push False: SymmetricComm.reduce_p2p, loads from the peers), push
    form by copy engines (push True: reduce_push) or by SM stores (push "store": reduce_store)."""
    ops.gemm_group([dict(x=p["x"], w=p["w"], out=comm.part[r:r + p["x"].shape[0]]) for p, r in zip(problems, row0)])
    mk(label)
    reduce = comm.reduce_store if push == "store" else comm.reduce_push if push else comm.reduce_p2p
    reduce(segments, mk, label)


def tp_double_block_p2p(ops, comm: SymmetricComm, txt_w: TPStreamWeights, img_w: TPStreamWeights, txt_mod1, img_mod1,
                        txt_mod2, img_mod2, txt, img, txt_gate1, img_gate1, txt_gate2, img_gate2, pe, mask,
                        s: TPScratch, mark=None, push=False) -> None:
    """tp_double_block with each row-split layer's all-reduce and residual update done by the
    two-phase peer-memory kernels (_row_split_p2p: pull, copy-engine push or store form); txt, img are this rank's
    replicated F32 streams."""
    T = txt_mod1.shape[0]
    mk = mark or _no_mark
    _qkv_attention_double(ops, txt_w, img_w, txt_mod1, img_mod1, pe, mask, s, mk)
    _row_split_p2p(ops, comm, [dict(x=s.attn[:T], w=txt_w.proj_w), dict(x=s.attn[T:], w=img_w.proj_w)], [0, T],
                   [dict(row0=0, bias=txt_w.proj_b, gate=txt_gate1, residual=txt),
                    dict(row0=T, bias=img_w.proj_b, gate=img_gate1, residual=img)], mk, "double.proj", push)
    ops.gemm_group([dict(x=txt_mod2, w=txt_w.mlp0_w, bias=txt_w.mlp0_b, out=s.h_txt, epilogue="gelu"),
                    dict(x=img_mod2, w=img_w.mlp0_w, bias=img_w.mlp0_b, out=s.h_img, epilogue="gelu")])
    mk("double.mlp0")
    _row_split_p2p(ops, comm, [dict(x=s.h_txt, w=txt_w.mlp2_w), dict(x=s.h_img, w=img_w.mlp2_w)], [0, T],
                   [dict(row0=0, bias=txt_w.mlp2_b, gate=txt_gate2, residual=txt),
                    dict(row0=T, bias=img_w.mlp2_b, gate=img_gate2, residual=img)], mk, "double.mlp2", push)


def tp_single_block_p2p(ops, comm: SymmetricComm, w: TPSingleWeights, x_mod, x, gate, pe, mask, s: TPScratch,
                        mark=None, push=False) -> None:
    """tp_single_block with linear2's all-reduce and residual update by the two-phase
    peer-memory kernels (pull, copy-engine push or store form); x this rank's replicated F32 stream."""
    HDl = s.HDl
    mk = mark or _no_mark
    _linear1(ops, w, x_mod, pe, s)
    mk("single.linear1")
    q, k, v = s.qkv[:, :HDl], s.qkv[:, HDl:2 * HDl], s.qkv[:, 2 * HDl:]
    ops.attention_bf16(q, k, v, s.hl, s.d.dhead, attn_mask=mask, out=s.cat[:, :HDl])
    mk("single.attention")
    _row_split_p2p(ops, comm, [dict(x=s.cat, w=w.linear2_w)], [0],
                   [dict(row0=0, bias=w.linear2_b, gate=gate, residual=x)], mk, "single.linear2", push)
