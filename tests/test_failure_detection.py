"""Failure detection of the multi-GPU path, tested without faulting, trapping or hanging a GPU.

On the host (CPU, `gloo` ranks):
  * a rank that leaves between steps is noticed by the survivors through tp.StepWatch (the
    process group's store) before they launch the next step: RankLost names it;
  * without that check, the survivors' next collective ends with an error within the process
    group's short timeout (it does not wait for good);
  * tp.CollectiveWatchdog aborts a collective's group once when the collective outlives its
    deadline (an injected timeout: a fake work object that never completes) and leaves
    completed collectives alone.
On one GPU:
  * libb2g's cross-rank barrier kernel waits for a rank whose flag is never set (a local
    buffer stands in for the absent rank's flag array); its bounded wait runs out after 2 s,
    the kernel returns, b2g_check_device_error reports the barrier, and the next GEMM on the
    same context is still correct (against the C oracle).
"""
from __future__ import annotations

import ctypes
import datetime
import os
import queue
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import tp
from conftest import rel_err


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---------------------------------------------------------------------------- watchdog (host)
class FakeWork:
    def __init__(self, done: bool = False):
        self.done = done

    def is_completed(self) -> bool:
        return self.done


class FakeClock:
    def __init__(self):
        self.t = 0.0

    def __call__(self) -> float:
        return self.t


def test_watchdog_aborts_once_after_deadline():
    aborted = []
    clock = FakeClock()
    wd = tp.CollectiveWatchdog(lambda: aborted.append(clock.t), deadline_s=2.0, clock=clock)
    wd.track(FakeWork(done=True), "done")
    stuck = wd.track(FakeWork(done=False), "all_reduce (injected: never completes)")
    clock.t = 1.9
    wd.poll()
    assert aborted == [] and wd.error is None
    clock.t = 2.1
    wd.poll()
    wd.poll()                                    # a second pass must not abort again
    assert aborted == [2.1]
    with pytest.raises(tp.CollectiveTimeout, match="never completes"):
        wd.check()
    with pytest.raises(tp.CollectiveTimeout):    # and nothing new is accepted afterwards
        wd.track(FakeWork(done=True))
    assert not stuck.is_completed()


def test_watchdog_leaves_completed_collectives_alone():
    aborted = []
    clock = FakeClock()
    wd = tp.CollectiveWatchdog(lambda: aborted.append(1), deadline_s=1.0, clock=clock)
    works = [wd.track(FakeWork(), f"c{i}") for i in range(5)]
    clock.t = 0.5
    for w in works:
        w.done = True
    clock.t = 100.0
    wd.poll()
    assert aborted == [] and not wd.pending
    wd.check()


def test_watchdog_thread_aborts_a_stuck_collective():
    fired = []
    wd = tp.CollectiveWatchdog(lambda: fired.append(time.monotonic()), deadline_s=0.2, poll_s=0.01).start()
    try:
        t0 = time.monotonic()
        wd.track(FakeWork(done=False), "all_reduce")
        while not fired and time.monotonic() - t0 < 5.0:
            time.sleep(0.01)
        assert fired and 0.2 <= fired[0] - t0 < 2.0
        with pytest.raises(tp.CollectiveTimeout):
            wd.check()
    finally:
        wd.stop()


def test_nccl_options_are_non_blocking():
    if not dist.is_nccl_available():
        pytest.skip("torch built without NCCL")
    assert tp.nccl_options().config.blocking == 0
    assert tp.nccl_options(blocking=True).config.blocking == 1


# ---------------------------------------------------------------------------- gloo ranks
def _leave(results) -> None:
    results.close()
    results.join_thread()   # the queue's feeder thread must flush before the process ends
    os._exit(0)


def _rank_main(rank, world, port, leaver, use_watch, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    store = dist.distributed_c10d._get_default_store()
    watch = tp.StepWatch(store, rank, world, timeout_s=3.0)
    done = tp.StepWatch(store, rank, world, timeout_s=30.0, prefix="b2g/done")
    wd = tp.CollectiveWatchdog(lambda: dist.distributed_c10d._get_default_group().abort(), deadline_s=20.0).start()
    ops = tp.EngineOps.__new__(tp.EngineOps)   # the host side only: no engine library needed on CPU
    ops.watchdog = wd
    t = torch.ones(64)
    try:
        for step in range(3):
            if rank == leaver and step == 2:
                # leave between steps with nothing in flight: every peer has finished step 1,
                # so none of them still waits on data this rank sent
                done.check(step - 1)
                results.put((rank, "left", None))
                _leave(results)
            if use_watch:
                watch.arrive(step)
                watch.check(step)
            ops.all_reduce(t)
            wd.pending[-1][0].wait()
            wd.check()
            done.arrive(step)
        results.put((rank, "finished", None))
    except tp.RankLost as e:
        results.put((rank, "RankLost", str(e)))
    except Exception as e:                      # the collective's own error
        results.put((rank, type(e).__name__, str(e)[:200]))
    finally:
        wd.stop()
    # rank 0 hosts the store the others still use: it leaves last
    survivors = [f"b2g/exit/{r}" for r in range(1, world) if r != leaver]
    if rank == 0:
        try:
            store.wait(survivors, datetime.timedelta(seconds=30))
        except Exception:
            pass
    else:
        store.set(f"b2g/exit/{rank}", "1")
    _leave(results)                             # skip a teardown that would talk to the lost rank


def _run_ranks(world: int, leaver: int, use_watch: bool, limit_s: float = 60.0) -> dict:
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, leaver, use_watch, results)) for r in range(world)]
    t0 = time.monotonic()
    for p in procs:
        p.start()
    out = {}
    try:
        while len(out) < world and time.monotonic() - t0 < limit_s:
            try:
                r, kind, msg = results.get(timeout=1.0)
                out[r] = (kind, msg, time.monotonic() - t0)
            except queue.Empty:
                pass
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()                        # our own child, by handle
    return out


def test_rank_leaving_between_steps_is_noticed_before_the_next_step():
    out = _run_ranks(world=3, leaver=2, use_watch=True)
    assert out.get(2, ("?",))[0] == "left"
    for r in (0, 1):
        kind, msg, t = out[r]
        assert kind == "RankLost" and "[2]" in msg and "step 2" in msg, out
        assert t < 45.0


def test_collective_with_a_departed_rank_errors_instead_of_hanging():
    out = _run_ranks(world=2, leaver=1, use_watch=False)
    assert out.get(1, ("?",))[0] == "left"
    kind, msg, t = out[0]
    assert kind not in ("finished", "?"), out   # the all-reduce without its peer raised
    assert t < 45.0


# ---------------------------------------------------------------------------- one GPU
@pytest.mark.gpu
def test_tp_barrier_wait_expires_and_reports(engine, oracle):
    dev = "cuda:0"
    lib = engine.load()
    own = torch.zeros(2, dtype=torch.int32, device=dev)       # this rank's flag array
    absent = torch.zeros(2, dtype=torch.int32, device=dev)    # stands in for rank 1's array
    ptrs = torch.tensor([own.data_ptr(), absent.data_ptr()], dtype=torch.int64, device=dev)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    engine.tp_barrier(ptrs, own, 2, 0, 1)   # rank 0 of 2; nothing ever sets own[1]
    code = ctypes.c_int(0)
    st = lib.b2g_check_device_error(ctypes.byref(code))
    waited = time.monotonic() - t0
    assert st == 5 and code.value & 8, (st, code.value, lib.b2g_last_error())
    assert b"tensor-parallel barrier" in lib.b2g_last_error()
    assert 1.5 <= waited < 30.0
    assert absent[0].item() == 1 and own[0].item() == 1       # rank 0's arrival was posted
    # the error word was cleared, and the context still computes correctly
    assert lib.b2g_check_device_error(ctypes.byref(code)) == 0 and code.value == 0
    g = torch.Generator().manual_seed(8)
    x = torch.randn((192, 256), generator=g).to(torch.bfloat16)
    w = (torch.randn((320, 256), generator=g) * 0.05).to(torch.bfloat16)
    b = torch.randn(320, generator=g) * 0.05
    want = oracle.linear(x.view(torch.int16).numpy().view(np.uint16), 2,
                         w.view(torch.int16).numpy().view(np.uint16), 2, b.numpy())
    got = engine.gemm(x.to(dev), w.to(dev), b.to(dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    engine.check_device_error()
    assert rel_err(got.cpu().numpy(), want) <= 1e-4


@pytest.mark.gpu
def test_tp_barrier_next_keeps_its_epoch_on_the_device(engine):
    """b2g_tp_barrier_next at world 1 (its own arrival completes it): the device counter advances
    once per call, eager and under CUDA graph replay alike, and the flag array follows it."""
    dev = "cuda:0"
    own = torch.zeros(1, dtype=torch.int32, device=dev)
    ctr = torch.zeros(1, dtype=torch.int32, device=dev)
    ptrs = torch.tensor([own.data_ptr()], dtype=torch.int64, device=dev)
    for _ in range(3):
        engine.tp_barrier_next(ptrs, own, ctr, 1, 0)
    torch.cuda.synchronize()
    assert ctr.item() == 3 and own.item() == 3
    g = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            engine.tp_barrier_next(ptrs, own, ctr, 1, 0)
            engine.tp_barrier_next(ptrs, own, ctr, 1, 0)
    torch.cuda.synchronize()
    assert ctr.item() == 3          # capture launches nothing
    for _ in range(4):
        g.replay()
    torch.cuda.synchronize()
    engine.check_device_error()
    assert ctr.item() == 11 and own.item() == 11
    del g
