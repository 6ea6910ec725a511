"""Failure handling of the sharded reductions, on CPU ranks (gloo).

Three ranks run the sharded step through ShardedReducer (each rank's
partial comes from the oracle in place of the kernel, written into the
reducer's partial buffers the way the kernel writes them), complete one
step, and then one rank fails between steps:

  leave       rank 2 announces that it leaves and exits;
  silent      rank 2 stays alive but never starts step 2;
  exit        rank 2 exits without a word, and the survivors go straight
              into step 2's collectives (no liveness check);
  hang        rank 2 stays alive but never joins step 2's collectives.

The survivors must raise on the host within a bound -- RankFailure before
any launch of step 2 (leave, silent), CollectiveFailure when a peer's
connection closed (exit), CollectiveTimeout with the communicator aborted
(hang) -- and never hang.  This follows the reference's host-side failure
model (injected errors surface as exceptions; its RecordingBackend tests in
runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesSuite.scala), one
layer up, at the collective.
"""
import os
import socket
import sys
import time
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

N_TOTAL = 30_011
MONITOR_TIMEOUT_S = 3.0
COLLECTIVE_TIMEOUT_S = 3.0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _step(red, x, xi, monitor: bool):
    if monitor:
        red.begin_step()
    red.sum_f32_async(x, stream=0)
    red.sum_i32_async(xi, stream=0)
    red.argmax_f32_async(x, stream=0)
    red.wait_checked(COLLECTIVE_TIMEOUT_S)
    return float(red.f64.item()), int(red.i32.item()), int(red.arg[0].item())


def _finish(q, item):
    q.put(item)
    q.close()
    q.join_thread()  # flush before the process ends


def _worker(rank: int, world: int, port: int, scenario: str, q, release):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from _cpu_partials import OraclePartials
    from flight4s_b200 import sharded
    from oracle import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # the process group's own timeout is the last bound, well above the checks
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    monitor = sharded.RankMonitor(timeout_s=MONITOR_TIMEOUT_S)
    red = sharded.ShardedReducer(OraclePartials(), torch.device("cpu"), N_TOTAL, monitor=monitor)
    xa = orc.uniform_f32(N_TOTAL, seed=5)
    xia = orc.uniform_i32(N_TOTAL, seed=5, lo=-1000, hi=1000)
    x = torch.from_numpy(xa[red.offset:red.offset + red.count].copy())
    xi = torch.from_numpy(xia[red.offset:red.offset + red.count].copy())
    use_monitor = scenario in ("leave", "silent")
    first = _step(red, x, xi, monitor=True)
    if rank == world - 1:  # the failing rank
        if scenario == "leave":
            monitor.leave()
            _finish(q, (rank, "left", first, 0.0))
            dist.destroy_process_group()
            return
        if scenario == "exit":
            _finish(q, (rank, "exited", first, 0.0))
            os._exit(0)
        _finish(q, (rank, "stalled", first, 0.0))
        release.wait(60)  # silent / hang: alive, but takes no part in step 2
        os._exit(0)
    t0 = time.monotonic()
    try:
        _step(red, x, xi, monitor=use_monitor)
        outcome = "no error"
    except sharded.CollectiveTimeout:
        outcome = "CollectiveTimeout"
    except sharded.CollectiveFailure:
        outcome = "CollectiveFailure"
    except sharded.RankFailure:
        outcome = "RankFailure"
    elapsed = time.monotonic() - t0
    _finish(q, (rank, outcome, first, elapsed))
    release.wait(60)  # rank 0 hosts the store: stay until every rank has reported
    os._exit(0)


# scenario -> (outcomes allowed on the survivors, bound in seconds).  After
# an exit, a survivor sees either the closed connection or, when its own
# collective waits on a survivor that already gave up, the bound: both are
# CollectiveFailure (CollectiveTimeout is its subclass).
# (leave: the peer announces itself, so detection takes milliseconds; the
# bound leaves room for a loaded host scheduling three spawned processes.)
EXPECTED = {"leave": ({"RankFailure"}, 3.0), "silent": ({"RankFailure"}, MONITOR_TIMEOUT_S + 2.0),
            "exit": ({"CollectiveFailure", "CollectiveTimeout"}, COLLECTIVE_TIMEOUT_S + 2.0),
            "hang": ({"CollectiveTimeout"}, COLLECTIVE_TIMEOUT_S + 2.0)}


@pytest.mark.parametrize("scenario", ["leave", "silent", "exit", "hang"])
def test_survivors_raise_within_a_bound(scenario):
    from oracle import oracle as orc
    world = 3
    t_start = time.monotonic()
    ctx = mp.get_context("spawn")
    q, release = ctx.Queue(), ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q, release)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = {}
        for _ in range(world):
            rank, outcome, first, elapsed = q.get(timeout=50)
            results[rank] = (outcome, first, elapsed)
    finally:
        release.set()
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    # step 1 combined correctly on every rank (the i32 sum and argmax bit-exact)
    xa = orc.uniform_f32(N_TOTAL, seed=5)
    xia = orc.uniform_i32(N_TOTAL, seed=5, lo=-1000, hi=1000)
    exact, abs_sum = orc.sum_f32_exact(xa)
    v, idx = orc.argmax_f32(xa)
    for rank in range(world):
        s, i, key = results[rank][1]
        assert abs(s - exact) <= 1e-12 * abs_sum
        assert i == orc.sum_i32(xia)
        assert key == orc.argmax_packed_key(v, idx)
    want, bound = EXPECTED[scenario]
    for rank in range(world - 1):
        outcome, _, elapsed = results[rank]
        assert outcome in want, (rank, outcome)
        assert elapsed <= bound, (rank, elapsed)
    assert time.monotonic() - t_start < 60
