"""Block sum (the reference's blockReduceSum extended to n elements):
bit-exact partials and result vs the oracle's level-by-level tree."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _run(ctx, hp, x):
    n = x.size
    tiles = (n + 255) // 256
    dx = ctx.allocate("f32", max(n, 1))
    if n:
        dx.copy_from(x) if n == dx.element_count else None
    parts, out = ctx.allocate("f32", max(tiles, 1)), ctx.allocate("f32", 1)
    ws = ctx.allocate("u8", hp.block_reduce_workspace_bytes(n))
    ws.copy_from(np.zeros(ws.element_count, np.uint8))
    hp.block_reduce_sum_f32_into(dx, parts, out, ws, n=n)
    ctx.synchronize()
    return out.copy_to_array()[0], parts.copy_to_array()[:tiles]


def test_reference_known_answer(ctx, hp):
    """CudaResourcesJniSuite.scala:235-238,310: x[i] = i % 8, n = 256 -> 896."""
    x = (np.arange(256) % 8).astype(np.float32)
    total, parts = _run(ctx, hp, x)
    assert total == np.float32(896.0) and parts.tolist() == [896.0]


# up to 2^23 elements the cluster-free kernel runs, above it the cluster kernel
@pytest.mark.parametrize("n", [0, 1, 2, 255, 256, 257, 8191, 8192, 8193, 65535, 65536, 65537, 1 << 20,
                               (1 << 20) + 77, 1 << 23, (1 << 23) + 1, (1 << 24) + 5, (1 << 25) + 3])
def test_bit_exact_vs_oracle(ctx, hp, n):
    x = orc.uniform_f32(n, seed=0x5EED + n)
    total, parts = _run(ctx, hp, x)
    ref_total, ref_parts = orc.block_tree_sum_f32(x)
    assert np.array_equal(parts.view(np.uint32), ref_parts.view(np.uint32))
    assert np.float32(total).view(np.uint32) == np.float32(ref_total).view(np.uint32)
    exact, abs_sum = orc.sum_f32_exact(x)
    assert abs(total - exact) <= 1e-5 * max(abs_sum, 1e-30)  # and close to the exact sum


def test_repeated_launches_reuse_workspace(ctx, hp):
    n = (1 << 20) + 1
    x = orc.uniform_f32(n, seed=3)
    dx, parts, out = ctx.allocate("f32", n), ctx.allocate("f32", (n + 255) // 256), ctx.allocate("f32", 1)
    dx.copy_from(x)
    ws = ctx.allocate("u8", hp.block_reduce_workspace_bytes(n))
    ws.copy_from(np.zeros(ws.element_count, np.uint8))
    ref, _ = orc.block_tree_sum_f32(x)
    for _ in range(5):
        hp.block_reduce_sum_f32_into(dx, parts, out, ws)
    ctx.synchronize()
    assert np.float32(out.copy_to_array()[0]) == np.float32(ref)


@pytest.mark.parametrize("n", [(1 << 20) + 77, (1 << 23) + 5])
def test_captured_in_a_cuda_graph(hp, torch_dev, n):
    """Captured into a CUDA graph (up to 2^23 elements: the tiles kernel and
    its programmatic dependent become two graph nodes), then replayed with a
    kernel writing the input before each replay: every replay gives the
    oracle's bits for the input it saw."""
    import torch
    x = torch.empty(n, dtype=torch.float32, device=torch_dev)
    parts = torch.empty((n + 255) // 256, dtype=torch.float32, device=torch_dev)
    out = torch.empty(1, dtype=torch.float32, device=torch_dev)
    ws = torch.zeros(hp.block_reduce_workspace_bytes(n), dtype=torch.uint8, device=torch_dev)
    src = [torch.from_numpy(orc.uniform_f32(n, seed=s)).to(torch_dev) for s in (11, 12)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        x.copy_(src[0])
        hp.block_reduce_sum_f32_into(x, parts, out, ws, stream=side)  # warm-up outside the capture
        side.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            hp.block_reduce_sum_f32_into(x, parts, out, ws, stream=side)
    torch.cuda.synchronize()
    for s, xs in zip((11, 12, 11), (src[0], src[1], src[0])):
        x.copy_(xs)  # a kernel on the current stream, ordered before the replay
        g.replay()
        torch.cuda.synchronize()
        ref_total, ref_parts = orc.block_tree_sum_f32(orc.uniform_f32(n, seed=s))
        assert np.float32(out.item()).view(np.uint32) == np.float32(ref_total).view(np.uint32)
        assert np.array_equal(parts.cpu().numpy().view(np.uint32), ref_parts.view(np.uint32))
    del g
