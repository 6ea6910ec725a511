"""Launch overlap (programmatic dependent launch) of the full-array
reductions: a reduction launched right after another one on the same stream
starts streaming its input while the first finishes, and waits for it only
before touching the shared workspace and its output.  The results must be
bit-identical to fully serialized launches (same kernels, same grids), for
every op, with one workspace shared by all of them, over many launches."""
import numpy as np
import pytest
import torch

import flight4s_b200 as f4s
from flight4s_b200.sharded import ShardedReducer
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _sequence(hp, bufs, outs, ws, stream, reps):
    x, xi, raw = bufs
    for _ in range(reps):
        hp.reduce_into(f4s.REDUCE_SUM_F32, x, outs[0], stream=stream, workspace=ws)
        hp.reduce_into(f4s.REDUCE_ARGMAX_F32, x, outs[1], stream=stream, workspace=ws)
        hp.reduce_into(f4s.REDUCE_SUM_I32, xi, outs[2], stream=stream, workspace=ws)
        hp.reduce_sum_into("bf16", raw, outs[3], n=raw.numel() // 2, stream=stream, workspace=ws)
        hp.reduce_sum_into("e4m3", raw, outs[4], n=raw.numel(), stream=stream, workspace=ws)
        hp.reduce_argmax_into("f16", raw, outs[5], n=raw.numel() // 2, stream=stream, workspace=ws)
        hp.reduce_argmax_into("f64", raw, outs[6], n=raw.numel() // 8, stream=stream, workspace=ws)


@pytest.mark.parametrize("n", [(1 << 26) + 3, 1 << 22])
def test_overlapped_reductions_match_serialized(hp, torch_dev, n):
    stream = torch.cuda.current_stream()
    x = torch.empty(n, dtype=torch.float32, device=torch_dev)
    xi = torch.empty(n, dtype=torch.int32, device=torch_dev)
    hp.fill_synthetic(x, n, f4s.NORMAL_F32, seed=11)
    hp.fill_synthetic(xi, n, f4s.UNIFORM_I32, seed=11, ilo=-1000, ihi=1000)
    raw = torch.randint(0, 256, (4 * n,), dtype=torch.uint8, device=torch_dev)
    ws = torch.zeros(hp.workspace_bytes, dtype=torch.uint8, device=torch_dev)
    torch.cuda.synchronize()
    results = {}
    for overlap in (False, True):
        hp.set_launch_overlap(overlap)
        outs = [torch.zeros(2, dtype=torch.int64, device=torch_dev) for _ in range(7)]
        _sequence(hp, (x, xi, raw), outs, ws, stream, reps=6)
        torch.cuda.synchronize()
        results[overlap] = [o.cpu().numpy() for o in outs]
    hp.set_launch_overlap(False)
    for a, b in zip(results[False], results[True]):
        assert np.array_equal(a, b)
    # and the serialized results are the right ones
    assert results[False][2].view(np.int32)[0] == orc.sum_i32(xi.cpu().numpy())
    assert int(results[False][1][1]) == int(torch.argmax(x).item())


def test_batched_steps_on_one_gpu(hp, torch_dev):
    """ShardedReducer.batch() with one rank and launch overlap: the three
    reductions of a step back to back, partials alternating between two
    buffers; every step's results against torch on the same device data."""
    n = (1 << 25) + 17
    stream = torch.cuda.current_stream()
    red = ShardedReducer(hp, torch_dev, n)
    hp.set_launch_overlap(True)
    try:
        for step in range(4):
            x = torch.empty(n, dtype=torch.float32, device=torch_dev)
            xi = torch.empty(n, dtype=torch.int32, device=torch_dev)
            hp.fill_synthetic(x, n, f4s.NORMAL_F32, seed=40 + step)
            hp.fill_synthetic(xi, n, f4s.UNIFORM_I32, seed=40 + step, ilo=-1000, ihi=1000)
            # a kernel that writes a reduction's input must not be the one
            # right before it with overlap on: order the fills first
            torch.cuda.synchronize()
            with red.batch(stream):
                red.sum_f32_async(x, stream)
                red.argmax_f32_async(x, stream)
                red.sum_i32_async(xi, stream)
            red.wait(stream)
            s = float(red.f64.item())
            ref = torch.sum(x, dtype=torch.float64).item()
            assert abs(s - ref) <= 1e-9 * torch.sum(x.abs(), dtype=torch.float64).item()
            assert int(red.i32.item()) == int(torch.sum(xi, dtype=torch.int64).item())
            assert ShardedReducer.argmax_result(red.arg)[1] == int(torch.argmax(x).item())
    finally:
        hp.set_launch_overlap(False)
