"""The runtime boundary on a GPU: PTX and cubin modules, function
attributes, cuLaunchKernelEx with and without clusters, streams, events,
pinned transfers, and driver errors surfacing as structured failures.
Mirrors native/tests/cuda_launch_integration_test.cpp and
runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala."""
import ctypes as C

import numpy as np
import pytest

import flight4s_b200 as f4s
from flight4s_b200 import _native

pytestmark = pytest.mark.gpu

# Hand-written PTX: out[i] = base + i, i = blockIdx.x * blockDim.x + threadIdx.x
# (the reference's native/tests/test_kernel.cu kernel, restated in PTX).
WRITE_VALUES_PTX = b"""
.version 8.7
.target sm_100a
.address_size 64
.visible .entry write_values(.param .u64 out, .param .u32 base)
{
  .reg .b32 %r<6>;
  .reg .b64 %rd<4>;
  ld.param.u64 %rd1, [out];
  ld.param.u32 %r1, [base];
  mov.u32 %r2, %ctaid.x;
  mov.u32 %r3, %ntid.x;
  mov.u32 %r4, %tid.x;
  mad.lo.s32 %r5, %r2, %r3, %r4;
  add.s32 %r1, %r1, %r5;
  cvta.to.global.u64 %rd2, %rd1;
  mul.wide.s32 %rd3, %r5, 4;
  add.s64 %rd2, %rd2, %rd3;
  st.global.u32 [%rd2], %r1;
  ret;
}
"""


def test_ptx_module_ordinary_and_clustered_launch(ctx):
    module = ctx.load_ptx(WRITE_VALUES_PTX)
    fn = module.function("write_values", signature=[f4s.DEVPTR, f4s.INT32])
    assert fn.attributes.max_threads_per_block >= 32
    out = ctx.allocate("i32", 64)
    fn.launch(fn.bind(out, 100), f4s.LaunchConfig(f4s.Grid(2), f4s.Block(32)))
    ctx.synchronize()
    assert out.copy_to_array().tolist() == list(range(100, 164))
    fn.launch(fn.bind(out, 200), f4s.LaunchConfig(f4s.Grid(2), f4s.Block(32), cluster=f4s.Cluster(2)))
    ctx.synchronize()
    assert out.copy_to_array().tolist() == list(range(200, 264))
    module.close()


# Hand-written PTX taking a signed 64-bit argument (descriptor code 11):
# out[i] = start + i for i < 4, start passed as one 64-bit value.
WRITE_I64_PTX = b"""
.version 8.7
.target sm_100a
.address_size 64
.visible .entry write_i64(.param .u64 out, .param .u32 tag, .param .s64 start)
{
  .reg .b32 %r<3>;
  .reg .b64 %rd<6>;
  ld.param.u64 %rd1, [out];
  ld.param.s64 %rd2, [start];
  mov.u32 %r1, %tid.x;
  cvt.s64.u32 %rd3, %r1;
  add.s64 %rd4, %rd2, %rd3;
  cvta.to.global.u64 %rd5, %rd1;
  mul.wide.u32 %rd3, %r1, 8;
  add.s64 %rd5, %rd5, %rd3;
  st.global.s64 [%rd5], %rd4;
  ret;
}
"""


def test_signed_int64_argument_launch(ctx):
    module = ctx.load_ptx(WRITE_I64_PTX)
    fn = module.function("write_i64", signature=[f4s.DEVPTR, f4s.UINT32, f4s.INT64])
    out = ctx.allocate("i64", 4)
    start = (1 << 40) - 2
    fn.launch(fn.bind(out, 5, start), f4s.LaunchConfig(f4s.Grid(1), f4s.Block(4)))
    ctx.synchronize()
    assert out.copy_to_array().tolist() == [start + i for i in range(4)]
    module.close()


def test_ptx_with_nul_byte_is_rejected(ctx):
    with pytest.raises(ValueError, match="null byte"):
        ctx.load_ptx(b".version 8.7\x00")


def test_invalid_ptx_reports_jit_error_log(ctx):
    with pytest.raises(f4s.CudaDriverFailure) as info:
        ctx.load_ptx(b".version 8.7\n.target sm_100a\n.address_size 64\n.visible .entry broken( {\n")
    assert info.value.result_name.startswith("CUDA_ERROR_")
    assert info.value.error_log


def test_hotpath_kernels_resolve_with_attributes(ctx, hp):
    for name in ["f4s_reduce_sum_f32", "f4s_reduce_sum_i32", "f4s_reduce_argmax_f32", "f4s_block_reduce_sum_f32",
                 "f4s_vector_add_f32", "f4s_vector_add_bf16", "f4s_softmax_rows_bf16_v4", "f4s_rmsnorm_rows_bf16_v4",
                 "f4s_fp8_quant_flat", "f4s_fp8_dequant_flat", "f4s_fill_synthetic",
                 "f4s_rmsnorm_rows_bf16_tma", "f4s_check_bounded_wait"]:
        fn = hp.module.function(name)
        assert fn.attributes.registers_per_thread > 0 and fn.attributes.local_memory_bytes == 0, name


def test_block_sum_through_launcher_with_cluster(ctx, hp):
    """The cluster block-sum kernel launched through the descriptor-coded
    launcher directly: (in, n, partials, out, workspace), block 1024,
    cluster (8,1,1)."""
    x = (np.arange(256) % 8).astype(np.float32)
    dx, parts, out = ctx.allocate("f32", 256), ctx.allocate("f32", 1), ctx.allocate("f32", 1)
    ws = ctx.allocate("u8", 512)
    ws.copy_from(np.zeros(512, np.uint8))
    dx.copy_from(x)
    fn = hp.module.function("f4s_block_reduce_sum_f32",
                            signature=[f4s.DEVPTR, f4s.INT32, f4s.DEVPTR, f4s.DEVPTR, f4s.DEVPTR])
    fn.launch(fn.bind(dx, 256, parts, out, ws), f4s.LaunchConfig(f4s.Grid(8), f4s.Block(1024), cluster=f4s.Cluster(8)))
    ctx.synchronize()
    assert out.copy_to_array()[0] == 896.0


def test_bad_geometry_rejected_before_driver_and_driver_errors_structured(ctx, hp):
    fn = hp.module.function("f4s_vector_add_f32", signature=[f4s.DEVPTR, f4s.DEVPTR, f4s.DEVPTR, f4s.INT32])
    buf = ctx.allocate("f32", 16)
    inv = fn.bind(buf, buf, buf, 16)
    st = inv.storage()
    rc = _native.lib.f4s_launch_kernel(ctx.handle, fn.handle, 0, 1, 1, 1, 0, 1, 1, 0, 0, 0, 0, 0,
                                       st.address, st.size_bytes, st.offsets, st.codes, st.count)
    assert rc == _native.STATUS_INVALID_ARGUMENT and "block x dimension must be positive" in _native.last_status()[2]
    with pytest.raises(f4s.CudaDriverFailure) as info:
        fn.launch(inv, f4s.LaunchConfig(f4s.Grid(1), f4s.Block(4096)))
    assert info.value.result_name == "CUDA_ERROR_INVALID_VALUE"
    ctx.synchronize()  # context still usable


def test_streams_events_timing_and_partial_pinned_transfers(ctx):
    """CudaResourcesJniSuite.scala:314-352: partial pinned transfers leave
    untouched elements as they were."""
    s = ctx.create_stream(non_blocking=True)
    e0, e1 = ctx.create_event(), ctx.create_event()
    host = ctx.allocate_pinned("i32", 64)
    host.copy_from(np.arange(64, dtype=np.int32))
    dev = ctx.allocate("i32", 64)
    dev.copy_from(np.full(64, -1, np.int32))
    e0.record(s)
    dev.copy_from_async(host, s, offset_elements=16, count=16)
    e1.record(s)
    s.synchronize()
    got = dev.copy_to_array()
    assert got[:16].tolist() == [-1] * 16 and got[16:32].tolist() == list(range(16)) and got[32:].tolist() == [-1] * 32
    assert e0.elapsed_ms(e1) >= 0.0
    assert e1.query()
    s.close()
    e0.close()
    e1.close()
    host.close()
    dev.close()


def test_copy_range_checks(ctx):
    dev = ctx.allocate("u8", 16)
    src = np.zeros(16, np.uint8)
    with pytest.raises(OverflowError):
        _native.check(_native.lib.f4s_copy_host_to_device(ctx.handle, dev.address, 2**64 - 8, src.ctypes.data, 16), "copy")
    with pytest.raises(ValueError, match="must be positive"):
        _native.check(_native.lib.f4s_copy_host_to_device(ctx.handle, dev.address, 0, src.ctypes.data, 0), "copy")
