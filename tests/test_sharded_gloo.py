"""The sharded reductions' combine step on CPU: world_size 2 gloo ranks,
per-rank partials from the oracle, combined by the product's collectives;
must equal the whole-array oracle results (bit-exact for i32 and argmax)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from flight4s_b200 import sharded


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, n: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import oracle as orc
    x = orc.uniform_f32(n, seed=42)
    xi = orc.uniform_i32(n, seed=42, lo=-1000, hi=1000)

    def partial(rank, offset, count):
        part = x[offset:offset + count]
        s, _ = orc.sum_f32_exact(np.ascontiguousarray(part))
        i = orc.sum_i32(np.ascontiguousarray(xi[offset:offset + count]))
        v, idx = orc.argmax_f32(np.ascontiguousarray(part))
        key = orc.argmax_packed_key(v, idx + offset) if idx >= 0 else -(1 << 63)
        return s, i, key

    out = sharded.cpu_sharded_combine(partial, n)
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_combine_matches_whole_array(world):
    from oracle import oracle as orc
    n = 100_003
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x = orc.uniform_f32(n, seed=42)
    xi = orc.uniform_i32(n, seed=42, lo=-1000, hi=1000)
    exact, abs_sum = orc.sum_f32_exact(x)
    v, idx = orc.argmax_f32(x)
    for rank in range(world):
        s, i, key = results[rank]
        assert abs(s - exact) <= 1e-12 * abs_sum
        assert i == orc.sum_i32(xi)
        assert key == orc.argmax_packed_key(v, idx)


def _u32_worker(rank: int, world: int, port: int, q):
    """Typed-sum partials travel as their collective type: u32 bits as i32."""
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    vals = [0xFFFFFFF0, 0x20, 0x7FFFFFFF][:world]
    t = torch.tensor([vals[rank]], dtype=torch.uint32).view(torch.int32)
    assert t.dtype == sharded.sum_partial_dtype("u32")
    sharded.combine_sum_i32(t)
    q.put((rank, sharded.sum_partial_value("u32", t)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_u32_partials_wrap(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_u32_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = sum([0xFFFFFFF0, 0x20, 0x7FFFFFFF][:world]) % 2**32
    assert all(v == want for v in results.values())


# per-case, per-rank (key, global index) partials; index -1 = empty shard
RECORD_CASES = {
    32: [[(7, 5), (7, (1 << 32) + 9), (-3, (1 << 33) + 1)],           # tie: lowest index wins
         [(-(1 << 31), (1 << 32) + 2), ((1 << 31) - 1, (1 << 34) + 7), (0, -1)],  # extreme keys, empty rank
         [(0, -1), (0, -1), (0, -1)],                                   # all empty
         [(5, (1 << 32) - 1), (5, 1 << 32), (4, 3)]],                   # the 32-bit boundary
    64: [[(-(1 << 63) + 1, 4), (123456789012345, 77), (123456789012345, 76)],
         [(0, -1), (-5, (1 << 40) + 3), (-5, (1 << 40) + 2)]],
}


def _record(bits: int, key: int, index: int) -> list[int]:
    if index < 0:
        return [-(1 << 63), -1]
    if bits == 64:
        return [key, index]
    return [key * (1 << 32) + (0xFFFFFFFF - index if index <= 0xFFFFFFFF else 0), index]


def _records_worker(rank: int, world: int, port: int, q):
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    out = {}
    for bits, cases in RECORD_CASES.items():
        for c, case in enumerate(cases):
            rec = torch.tensor(_record(bits, *case[rank]), dtype=torch.int64)
            sharded.combine_argmax_records(rec, bits)
            out[(bits, c)] = rec.tolist()
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_argmax_records_beyond_32_bit_indices(world):
    """The gathered-record combine (f64 keys, and arrays past 2^32
    elements): largest key, lowest global index, empty shards skipped."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_records_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for bits, cases in RECORD_CASES.items():
        for c, case in enumerate(cases):
            live = [(k, i) for k, i in case[:world] if i >= 0]
            if live:
                best = max(k for k, _ in live)
                want = _record(bits, best, min(i for k, i in live if k == best))
            else:
                want = [-(1 << 63), -1]
            for rank in range(world):
                assert results[rank][(bits, c)] == want, (bits, c, rank)


def test_argmax_result_reads_wide_indices():
    import torch
    rec = torch.tensor(_record(32, 0x3F800000, (1 << 32) + 11), dtype=torch.int64)   # 1.0f at index 2^32 + 11
    assert sharded.ShardedReducer.argmax_result(rec) == (1.0, (1 << 32) + 11)
    rec = torch.tensor(_record(32, 0x3F800000, 12), dtype=torch.int64)
    rec[1] = 99  # a stale local index after the packed all_reduce: the packed word decides
    assert sharded.ShardedReducer.argmax_result(rec) == (1.0, 12)


def test_sum_partial_types():
    import torch
    assert sharded.sum_partial_dtype("i32") == torch.int32
    for dtype in ("f16", "bf16", "f32", "f64", "e4m3", "e5m2"):
        assert sharded.sum_partial_dtype(dtype) == torch.float64
    with pytest.raises(ValueError):
        sharded.sum_partial_dtype("bool")


def test_shard_bounds_cover_exactly():
    for n in [0, 1, 7, 2**32]:
        for world in [1, 2, 3, 8]:
            spans = [sharded.shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0
            assert all(a[0] + a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert spans[-1][0] + spans[-1][1] == n


def _batch_worker(rank: int, world: int, port: int, q):
    """Batched steps (kernels back to back, all_reduces after the block,
    partials alternating between two buffers), two batches in flight before
    each wait, then an unbatched step."""
    import sys
    import torch
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.dirname(here))
    from _cpu_partials import OraclePartials
    from oracle import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n = 50_021
    red = sharded.ShardedReducer(OraclePartials(), torch.device("cpu"), n)

    def shards(step):
        lo, hi = red.offset, red.offset + red.count
        return (torch.from_numpy(orc.uniform_f32(n, seed=100 + step)[lo:hi].copy()),
                torch.from_numpy(orc.uniform_i32(n, seed=100 + step, lo=-1000, hi=1000)[lo:hi].copy()))

    out = {}
    for step in range(4):
        x, xi = shards(step)
        with red.batch():
            red.sum_f32_async(x, stream=0)
            red.argmax_f32_async(x, stream=0)
            red.sum_i32_async(xi, stream=0)
        bufs = (red.f64, red.i32, red.arg)  # this step's partials
        if step % 2 == 0:
            held = (step, bufs)  # read after the next batch, which writes the other buffers
            continue
        assert all(a is not b for a, b in zip(held[1], bufs))
        red.wait_checked(30.0)
        for s_, b in (held, (step, bufs)):
            out[s_] = (float(b[0].item()), int(b[1].item()), int(b[2][0].item()))
    x, xi = shards(4)
    s4, i4 = red.sum_f32(x, stream=0), red.sum_i32(xi, stream=0)
    red.argmax_f32_async(x, stream=0)
    red.wait()
    out[4] = (s4, i4, int(red.arg[0].item()))
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_batched_steps_alternate_partials():
    from oracle import oracle as orc
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_batch_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n = 50_021
    for step in range(5):
        x = orc.uniform_f32(n, seed=100 + step)
        xi = orc.uniform_i32(n, seed=100 + step, lo=-1000, hi=1000)
        exact, abs_sum = orc.sum_f32_exact(x)
        v, idx = orc.argmax_f32(x)
        for rank in range(world):
            got = results[rank][step]
            assert abs(got[0] - exact) <= 1e-12 * abs_sum, (rank, step)
            assert got[1] == orc.sum_i32(xi), (rank, step)
            assert got[2] == orc.argmax_packed_key(v, idx), (rank, step)
