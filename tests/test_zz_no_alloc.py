"""The allocation-free block sum, f4s_block_reduce_sum_f32_noalloc.

Callers that cannot allocate device memory use this entry point instead
of f4s_block_reduce_sum_f32, whose workspace they would have to provide.
Here it is called through the C ABI and must give bit-identical partials
and totals to the regular entry point (the block-sum tests' tolerance is
bit-exact), on two calls in a row, since the second call reuses the
static workspace the first one left behind.  The file sorts last so a
run that stops at the first failure has run every other test already; it
also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

import flight4s_b200 as f4s
from flight4s_b200 import _native
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _regular(ctx, hp, dx, n):
    tiles = max((n + 255) // 256, 1)
    parts, out = ctx.allocate("f32", tiles), ctx.allocate("f32", 1)
    ws = ctx.allocate("u8", hp.block_reduce_workspace_bytes(n))
    ws.copy_from(np.zeros(ws.element_count, np.uint8))
    hp.block_reduce_sum_f32_into(dx, parts, out, ws, n=n)
    ctx.synchronize()
    return out.copy_to_array()[0], parts.copy_to_array()[:(n + 255) // 256]


def _noalloc(ctx, hp, dx, n, parts, out, stream=0):
    _native.check(_native.lib.f4s_block_reduce_sum_f32_noalloc(hp.handle, stream, dx.address, n, parts.address,
                                                               out.address), "block sum (allocation-free)")


@pytest.mark.parametrize("n", [1, 256, 65537, (1 << 20) + 77, (1 << 24) + 5])
def test_noalloc_matches_regular_entry_point_twice(ctx, hp, n):
    x = orc.uniform_f32(n, seed=0xA11C + n)
    dx = ctx.allocate("f32", n)
    dx.copy_from(x)
    ref_total, ref_parts = _regular(ctx, hp, dx, n)
    parts, out = ctx.allocate("f32", max((n + 255) // 256, 1)), ctx.allocate("f32", 1)
    stream = ctx.create_stream(non_blocking=True)
    for _ in range(2):
        parts.copy_from(np.full(parts.element_count, np.nan, np.float32))
        out.copy_from(np.full(1, np.nan, np.float32))
        _noalloc(ctx, hp, dx, n, parts, out, stream.handle)
        stream.synchronize()
        total = out.copy_to_array()[0]
        assert np.float32(total).view(np.uint32) == np.float32(ref_total).view(np.uint32)
        assert np.array_equal(parts.copy_to_array()[:ref_parts.size].view(np.uint32), ref_parts.view(np.uint32))
    stream.close()


def test_noalloc_rejects_sizes_beyond_its_workspace(ctx, hp):
    dx, parts, out = ctx.allocate("f32", 16), ctx.allocate("f32", 16), ctx.allocate("f32", 1)
    st = _native.lib.f4s_block_reduce_sum_f32_noalloc(hp.handle, 0, dx.address, 1_069_547_521, parts.address,
                                                      out.address)
    assert st == _native.STATUS_INVALID_ARGUMENT
    assert "at most 1069547520 elements" in _native.last_status()[2]
    st = _native.lib.f4s_block_reduce_sum_f32_noalloc(hp.handle, 0, dx.address, -1, parts.address, out.address)
    assert st == _native.STATUS_INVALID_ARGUMENT
