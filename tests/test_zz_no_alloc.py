"""The allocation-free block sum, f4s_block_reduce_sum_f32_noalloc.

Callers that cannot allocate device memory use this entry point instead
of f4s_block_reduce_sum_f32, whose workspace they would have to provide.
Here it is called through the C ABI and must give bit-identical partials
and totals to the regular entry point (the block-sum tests' tolerance is
bit-exact), on two calls in a row, since the second call reuses the
static workspace the first one left behind.  The workspace exists once per
CUDA context, so the entry point is also called through a hot path opened
in a second context of the same GPU (made with cuCtxCreate), after and
between calls in the primary context, and again after that hot path is
closed and reopened.  The file sorts last so a run that stops at the first
failure has run every other test already; it also passes on its own in a
fresh process.
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


def _driver_fn(symbol, restype, *argtypes):
    """A CUDA driver entry point by its exported, versioned symbol (the
    classic cuCtxCreate_v2 signature, not a later version's)."""
    fn = getattr(C.CDLL("libcuda.so.1"), symbol)
    fn.restype, fn.argtypes = restype, list(argtypes)
    return fn


class _SecondContext:
    """A context of GPU 0 made with cuCtxCreate (not the primary context),
    with device buffers, copies and a hot path of its own through the C ABI."""

    def __init__(self):
        dev = C.c_int()
        assert _driver_fn("cuDeviceGet", C.c_int, C.POINTER(C.c_int), C.c_int)(C.byref(dev), 0) == 0
        handle = C.c_void_p()
        assert _driver_fn("cuCtxCreate_v2", C.c_int, C.POINTER(C.c_void_p), C.c_uint, C.c_int)(
            C.byref(handle), 0, dev.value) == 0
        popped = C.c_void_p()  # cuCtxCreate made it current: restore the caller's context
        assert _driver_fn("cuCtxPopCurrent_v2", C.c_int, C.POINTER(C.c_void_p))(C.byref(popped)) == 0
        assert popped.value == handle.value
        self.handle = handle.value
        self.buffers = []

    def allocate(self, nbytes):
        addr = C.c_uint64()
        _native.check(_native.lib.f4s_allocate_device_memory(self.handle, nbytes, C.byref(addr)), "allocate")
        self.buffers.append(addr.value)
        return addr.value

    def upload(self, addr, array):
        _native.check(_native.lib.f4s_copy_host_to_device(self.handle, addr, 0, array.ctypes.data, array.nbytes),
                      "copy to device")

    def download(self, addr, count):
        host = np.empty(count, np.float32)
        _native.check(_native.lib.f4s_copy_device_to_host(self.handle, addr, 0, host.ctypes.data, host.nbytes),
                      "copy to host")
        return host

    def open_hotpath(self):
        h = C.c_void_p()
        _native.check(_native.lib.f4s_hotpath_open(self.handle, C.byref(h)), "hot path in a created context")
        return h.value

    def close(self):
        for addr in self.buffers:
            _native.lib.f4s_free_device_memory(self.handle, addr)
        assert _driver_fn("cuCtxDestroy_v2", C.c_int, C.c_void_p)(self.handle) == 0


def test_noalloc_in_a_second_context_of_the_gpu(ctx, hp):
    n = (1 << 23) + 77  # above 2^23 the kernel keeps its ticket and partials in the static workspace
    tiles = (n + 255) // 256
    x = orc.uniform_f32(n, seed=0xC0DE)
    dx = ctx.allocate("f32", n)
    dx.copy_from(x)
    ref_total, ref_parts = _regular(ctx, hp, dx, n)
    want = np.float32(ref_total).view(np.uint32)
    parts, out = ctx.allocate("f32", tiles), ctx.allocate("f32", 1)

    def primary_call():
        out.copy_from(np.full(1, np.nan, np.float32))
        _noalloc(ctx, hp, dx, n, parts, out)
        ctx.synchronize()
        assert np.float32(out.copy_to_array()[0]).view(np.uint32) == want

    primary_call()  # the primary context's workspace is looked up first
    second = _SecondContext()
    hot = None
    try:
        bx, bparts, bout = second.allocate(4 * n), second.allocate(4 * tiles), second.allocate(4)
        second.upload(bx, x)

        def second_call(h):
            second.upload(bout, np.full(1, np.nan, np.float32))
            second.upload(bparts, np.full(tiles, np.nan, np.float32))
            _native.check(_native.lib.f4s_block_reduce_sum_f32_noalloc(h, 0, bx, n, bparts, bout),
                          "block sum (allocation-free, second context)")
            _native.check(_native.lib.f4s_synchronize_context(second.handle), "synchronize")
            assert second.download(bout, 1).view(np.uint32)[0] == want
            assert np.array_equal(second.download(bparts, tiles).view(np.uint32), ref_parts.view(np.uint32))

        hot = second.open_hotpath()
        second_call(hot)
        second_call(hot)
        primary_call()  # back in the primary context: its own workspace
        _native.check(_native.lib.f4s_hotpath_close(hot), "close hot path")
        hot = second.open_hotpath()  # a reopened hot path in the same context
        second_call(hot)
    finally:
        if hot is not None:
            _native.lib.f4s_hotpath_close(hot)
        second.close()
    primary_call()


def test_noalloc_at_its_exact_capacity(ctx, hp):
    n = 1_069_547_520  # the largest n: its workspace needs exactly the 64 KiB the array holds
    assert _native.lib.f4s_block_reduce_workspace_bytes(n) == 64 * 1024
    dx = ctx.allocate("f32", n)
    hp.fill_synthetic(dx, n, f4s.UNIFORM_F32, seed=0xCA9)
    ref_total, ref_parts = _regular(ctx, hp, dx, n)
    parts, out = ctx.allocate("f32", (n + 255) // 256), ctx.allocate("f32", 1)
    for _ in range(2):
        out.copy_from(np.full(1, np.nan, np.float32))
        _noalloc(ctx, hp, dx, n, parts, out)
        ctx.synchronize()
        assert np.float32(out.copy_to_array()[0]).view(np.uint32) == np.float32(ref_total).view(np.uint32)
        assert np.array_equal(parts.copy_to_array().view(np.uint32), ref_parts.view(np.uint32))
    for b in (dx, parts, out):
        b.close()


def test_noalloc_rejects_sizes_beyond_its_workspace(ctx, hp):
    dx, parts, out = ctx.allocate("f32", 16), ctx.allocate("f32", 16), ctx.allocate("f32", 1)
    st = _native.lib.f4s_block_reduce_sum_f32_noalloc(hp.handle, 0, dx.address, 1_069_547_521, parts.address,
                                                      out.address)
    assert st == _native.STATUS_INVALID_ARGUMENT
    assert "at most 1069547520 elements" in _native.last_status()[2]
    st = _native.lib.f4s_block_reduce_sum_f32_noalloc(hp.handle, 0, dx.address, -1, parts.address, out.address)
    assert st == _native.STATUS_INVALID_ARGUMENT
