"""End-to-end reductions of HOST buffers (chunked copies overlapped with
the kernels) give the same results as the device-resident path."""
import numpy as np
import pytest

import flight4s_b200 as f4s
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [0, 1, 1000, (1 << 20) + 5, 10_000_019])
def test_reduce_host_matches_device(ctx, hp, n):
    rng = np.random.default_rng(n)
    x = ctx.allocate_pinned("f32", n)
    x.copy_from(rng.standard_normal(n).astype(np.float32))
    xi = ctx.allocate_pinned("i32", n)
    xi.copy_from(rng.integers(-1000, 1001, n).astype(np.int32))
    staging = ctx.allocate("u8", 256 + 2 * (1 << 20))  # 1 MiB buffers: many chunks
    s1, s2 = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    r = hp.reduce_host(f4s.REDUCE_SUM_F32, x.array, staging, s1, s2)
    exact, abs_sum = orc.sum_f32_exact(x.array)
    assert abs(float(r[:1].view(np.float64)[0]) - exact) <= 1e-5 * abs_sum
    r = hp.reduce_host(f4s.REDUCE_SUM_I32, xi.array, staging, s1, s2)
    assert int(r[:1].view(np.int32)[0]) == orc.sum_i32(xi.array)
    r = hp.reduce_host(f4s.REDUCE_ARGMAX_F32, x.array, staging, s1, s2).view(np.int64)
    rv, ri = orc.argmax_f32(x.array)
    assert int(r[1]) == ri
    if n:
        assert int(r[0]) == orc.argmax_packed_key(rv, ri)


@pytest.mark.parametrize("n", [0, 7, (1 << 20) + 5, 10_000_019])
def test_reduce_host_sum_argmax_one_transfer(ctx, hp, n):
    rng = np.random.default_rng(n + 1)
    x = ctx.allocate_pinned("f32", n)
    x.copy_from(rng.standard_normal(n).astype(np.float32))
    staging = ctx.allocate("u8", 256 + 2 * (1 << 20))
    s1, s2 = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    s, a = hp.reduce_host_sum_argmax(x.array, staging, s1, s2, index_base=1000)
    exact, abs_sum = orc.sum_f32_exact(x.array)
    assert abs(float(s.view(np.float64)[0]) - exact) <= 1e-5 * abs_sum
    rv, ri = orc.argmax_f32(x.array)
    a = a.view(np.int64)
    if n:
        assert int(a[1]) == ri + 1000 and int(a[0]) == orc.argmax_packed_key(rv, ri + 1000)
    else:
        assert int(a[1]) == -1
