"""Scenarios run against the fake CUDA driver (tests/fake_driver/fake_cuda.c),
one per process: `python _fake_driver_scenarios.py <scenario> <libfakecuda.so>`
with FLIGHT4S_CUDA_DRIVER pointing at the fake (set by
tests/test_fake_driver.py).  Exit status 0 = pass."""
import ctypes as C
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import flight4s_b200 as f4s
from flight4s_b200 import _native

FAKE = C.CDLL(sys.argv[2])


class Launch(C.Structure):
    _fields_ = [("name", C.c_char * 64), ("grid", C.c_uint * 3), ("block", C.c_uint * 3), ("smem", C.c_uint),
                ("cluster", C.c_int), ("cluster_dim", C.c_uint * 3), ("nparams", C.c_int),
                ("params", (C.c_ubyte * 8) * 32), ("stream", C.c_ulonglong), ("programmatic", C.c_int)]


FAKE.fake_last_launch.restype = C.POINTER(Launch)


def last() -> Launch:
    return FAKE.fake_last_launch().contents


def count() -> int:
    return FAKE.fake_launch_count()


def param(launch: Launch, i: int, size: int = 8) -> int:
    return int.from_bytes(bytes(launch.params[i])[:size], "little")


def expect_failure(fn, code: int, name: str):
    try:
        fn()
    except f4s.CudaDriverFailure as e:
        assert e.result_code == code and e.result_name == name, (e.result_code, e.result_name)
        return e
    raise AssertionError("expected a driver failure")


def launch_records_geometry():
    ctx = f4s.CudaContext.open(0)
    assert ctx.compute_capability == (10, 0)
    mod = ctx.load(b"fake module image")
    fn = mod.function("write_values", signature=[f4s.DEVPTR, f4s.INT32])
    buf = ctx.allocate("i32", 64)
    fn.launch(fn.bind(buf, 100), f4s.LaunchConfig(f4s.Grid(2), f4s.Block(32), cluster=f4s.Cluster(2)))
    L = last()
    assert L.name == b"write_values" and tuple(L.grid) == (2, 1, 1) and tuple(L.block) == (32, 1, 1)
    assert L.cluster == 1 and tuple(L.cluster_dim) == (2, 1, 1)
    assert param(L, 0) == buf.address and param(L, 1, 4) == 100
    fn.launch(fn.bind(buf, 7), f4s.LaunchConfig(f4s.Grid(4, 2), f4s.Block(16, 2), dynamic_shared_memory_bytes=256))
    L = last()
    assert L.cluster == 0 and tuple(L.grid) == (4, 2, 1) and tuple(L.block) == (16, 2, 1) and L.smem == 256
    assert count() == 2
    ctx.close()


def launch_error_propagates():
    ctx = f4s.CudaContext.open(0)
    fn = ctx.load(b"fake").function("write_values", signature=[f4s.DEVPTR, f4s.INT32])
    buf = ctx.allocate("i32", 64)
    e = expect_failure(lambda: fn.launch(fn.bind(buf, 1), f4s.LaunchConfig(f4s.Grid(1), f4s.Block(32))), 719,
                       "CUDA_ERROR_LAUNCH_FAILED")
    assert e.description == "fake driver error description"
    assert count() == 0
    hp = ctx.hotpath()
    expect_failure(lambda: hp.vector_add_f32(buf, buf, buf, n=64), 719, "CUDA_ERROR_LAUNCH_FAILED")


def out_of_memory():
    ctx = f4s.CudaContext.open(0)
    expect_failure(lambda: ctx.allocate("f32", 1 << 20), 2, "CUDA_ERROR_OUT_OF_MEMORY")
    # a hotpath cannot get its workspace either, and says so
    hp = ctx.hotpath()
    expect_failure(lambda: hp.workspace(), 2, "CUDA_ERROR_OUT_OF_MEMORY")


def pop_mismatch():
    """The operation succeeds but another context is on top afterwards:
    reported as CUDA_ERROR_INVALID_CONTEXT (native/src/current_context_scope.cpp:21-33)."""
    ctx = f4s.CudaContext.open(0)
    expect_failure(ctx.synchronize, 201, "CUDA_ERROR_INVALID_CONTEXT")
    expect_failure(lambda: ctx.allocate("f32", 16), 201, "CUDA_ERROR_INVALID_CONTEXT")


def push_failure():
    ctx = f4s.CudaContext.open(0)
    rc = _native.lib.f4s_launch_kernel(ctx.handle, 0x1000, 0, 1, 1, 1, 32, 1, 1, 0, 0, 0, 0, 0, None, 0, None, None, 0)
    assert rc == 201 and _native.last_status()[1] == "CUDA_ERROR_INVALID_CONTEXT"
    assert count() == 0


def jit_error_log():
    ctx = f4s.CudaContext.open(0)
    e = expect_failure(lambda: ctx.load_ptx(b".version 8.7\n"), 218, "CUDA_ERROR_INVALID_PTX")
    assert e.error_log == "fake error log"


def invalid_arguments_never_reach_driver():
    ctx = f4s.CudaContext.open(0)
    fn = ctx.load(b"fake").function("write_values", signature=[f4s.DEVPTR, f4s.INT32])
    buf = ctx.allocate("i32", 64)
    st = fn.bind(buf, 1).storage()
    rc = _native.lib.f4s_launch_kernel(ctx.handle, fn.handle, 0, 3, 1, 1, 32, 1, 1, 0, 1, 2, 1, 1, st.address,
                                       st.size_bytes, st.offsets, st.codes, st.count)
    assert rc == _native.STATUS_INVALID_ARGUMENT and "must be divisible" in _native.last_status()[2]
    hp = ctx.hotpath()
    for bad in [lambda: hp.vector_add_f32(buf.address + 1, buf, buf, n=8),
                lambda: hp.softmax_rows_bf16(buf, buf, -1, 8),
                lambda: hp.reduce_into(f4s.REDUCE_SUM_F32, buf, buf.address + 4, workspace=buf),
                lambda: hp.fill_synthetic(buf, 8, f4s.UNIFORM_I32, seed=1, ilo=3, ihi=2)]:
        try:
            bad()
        except ValueError:
            pass
        else:
            raise AssertionError("expected ValueError")
    assert count() == 0


def hotpath_dispatch():
    ctx = f4s.CudaContext.open(0)
    hp = ctx.hotpath()
    assert hp.sm_count == 148
    big = ctx.allocate("f32", 1 << 28)

    def check(name, grid, block=256, cluster=None):
        L = last()
        assert L.name.decode() == name, (L.name, name)
        assert tuple(L.grid) == (grid, 1, 1) and L.block[0] == block, (name, tuple(L.grid), L.block[0])
        if cluster is None:
            assert L.cluster == 0
        else:
            assert L.cluster == 1 and L.cluster_dim[0] == cluster
        return L

    hp.vector_add_f32(big, big, big, n=1 << 28)
    assert param(check("f4s_vector_add_f32", (1 << 28) // 2048), 3, 4) == 1 << 28
    hp.vector_add_bf16(big, big, big, n=1000)
    check("f4s_vector_add_bf16", 1)
    for dtype, kernel, per_cta in [("f16", "f16", 256 * 16), ("f64", "f64", 256 * 4), ("u32", "i32", 256 * 8)]:
        hp.vector_add(dtype, big, big, big, n=1 << 20)
        L = check(f"f4s_vector_add_{kernel}", (1 << 20) // per_cta)
        assert param(L, 3, 4) == 1 << 20
    hp.softmax_rows_bf16(big, big, 32768, 8192)  # two rows per CTA
    check("f4s_softmax_rows_bf16_v4", 16384)
    hp.softmax_rows_bf16(big, big, 11, 1000)
    check("f4s_softmax_rows_bf16_v1", 6)
    hp.softmax_rows_bf16(big, big, 10, 8 * 2048)  # the widest register rows: one row per CTA
    check("f4s_softmax_rows_bf16_v8", 10)
    hp.softmax_rows_bf16(big, big, 10, 1001)
    check("f4s_softmax_rows_bf16_any", 10)
    hp.rmsnorm_rows_bf16(big, big, big, 32768, 8192)
    check("f4s_rmsnorm_rows_bf16_tma", 296)
    hp.rmsnorm_rows_bf16(big, big, big, 32768, 16384)
    check("f4s_rmsnorm_rows_bf16_v8", 148 * 8)
    hp.rmsnorm_rows_bf16(big, big, big, 5, 1001)
    check("f4s_rmsnorm_rows_bf16_any", 5)
    hp.fp8_quantize_e4m3(big, big, big, 16384, 16384)
    assert param(check("f4s_fp8_quant_flat", (1 << 21) // 16 // 8), 3, 4) == 1 << 21
    hp.fp8_dequantize_e4m3(big, big, big, 16384, 16384)
    check("f4s_fp8_dequant_flat", (1 << 21) // 8 // 8)
    hp.fp8_quantize_e4m3(big, big, big, 3, 200)
    check("f4s_fp8_quant_rows", hp_fp8_rows_grid())
    out = ctx.allocate("i64", 2)
    hp.reduce_into(f4s.REDUCE_SUM_F32, big, out, n=1 << 32)
    L = check("f4s_reduce_sum_f32", 37 * 16 * 4, block=512, cluster=4)  # 16 waves of the fake's 37 clusters
    assert (param(L, 1, 4), param(L, 2, 4)) == (0, 1)  # n = 2^32 split in two u32
    assert L.programmatic == 0  # launch overlap is off by default
    hp.reduce_into(f4s.REDUCE_ARGMAX_F32, big, out, n=1000, index_base=(1 << 32) + 5, accumulate=True)
    L = check("f4s_reduce_argmax_f32", 4, block=512, cluster=4)
    assert (param(L, 5, 4), param(L, 6, 4), param(L, 7, 4)) == (5, 1, 1)
    # with launch overlap the device-resident reductions are programmatic dependents
    hp.set_launch_overlap(True)
    hp.reduce_into(f4s.REDUCE_SUM_I32, big, out, n=1 << 20)
    # 8 vectors per lane per step: 16 clusters of 4 x 512 x 4 x 8 elements
    assert check("f4s_reduce_sum_i32", 16 * 4, block=512, cluster=4).programmatic == 1
    hp.reduce_sum_into("bf16", big, out, n=1000)
    assert last().programmatic == 1
    hp.vector_add_f32(big, big, big, n=1 << 10)  # other operators never are
    assert last().programmatic == 0
    hp.set_launch_overlap(False)
    hp.reduce_into(f4s.REDUCE_SUM_I32, big, out, n=1 << 20)
    assert last().programmatic == 0
    # typed ReduceSum: kernel per input type, grid sized in 16-byte vectors
    for dtype, kernel in [("e4m3", "e4m3"), ("e5m2", "e5m2"), ("f16", "f16"), ("bf16", "bf16"), ("f64", "f64"),
                          ("u32", "i32"), ("i32", "i32"), ("f32", "f32")]:
        hp.reduce_sum_into(dtype, big, out, n=1000)
        check(f"f4s_reduce_sum_{kernel}", 4, block=512, cluster=4)
    hp.reduce_sum_into("e4m3", big, out, n=1 << 20)  # FP8 steps 8 vectors: 4 clusters of 4 x 512 x 16 x 8 elements
    check("f4s_reduce_sum_e4m3", 4 * 4, block=512, cluster=4)
    hp.reduce_sum_into("bf16", big, out, n=1 << 20)  # 16-bit sums step 8 vectors: 8 clusters of 4 x 512 x 8 x 8
    check("f4s_reduce_sum_bf16", 8 * 4, block=512, cluster=4)
    hp.reduce_sum_into("f64", big, out, n=1 << 20)   # 2 elements per vector, 8 per step: 32 clusters
    check("f4s_reduce_sum_f64", 32 * 4, block=512, cluster=4)
    # large inputs: 8 waves of co-resident clusters (the fake reports 37), 16 for the f64 and FP8 sums
    hp.reduce_sum_into("f64", big, out, n=1 << 27)
    check("f4s_reduce_sum_f64", 37 * 16 * 4, block=512, cluster=4)
    hp.reduce_sum_into("e5m2", big, out, n=1 << 30)
    check("f4s_reduce_sum_e5m2", 37 * 16 * 4, block=512, cluster=4)
    hp.reduce_sum_into("f16", big, out, n=1 << 29)
    check("f4s_reduce_sum_f16", 37 * 16 * 4, block=512, cluster=4)
    assert 256 + 16 * (37 * 16) <= hp.workspace_bytes   # one 16-byte partial slot per launched cluster
    before = count()
    ws0 = hp.workspace()
    for code in (0, 1, 10, 11):   # bool and pointer have no accumulator
        rc = _native.lib.f4s_reduce_sum(hp.handle, 0, code, big.address, 8, out.address, ws0.address,
                                        ws0.size_bytes, 0)
        assert rc == _native.STATUS_INVALID_ARGUMENT and "no ReduceSum accumulator" in _native.last_status()[2]
    try:
        hp.reduce_sum_into("f64", big.address + 4, out, n=8)
    except ValueError as e:
        assert "8-byte aligned" in str(e)
    else:
        raise AssertionError("expected ValueError")
    assert count() == before
    # order-fixed policy: one CTA per 256 KiB group up to the resident CTAs, block 512, no cluster
    wso = ctx.allocate("u8", hp.policy_workspace_bytes("f32", 1 << 20, "deterministic"))
    hp.reduce_sum_into("f32", big, out, n=1 << 20, workspace=wso, policy="deterministic")
    L = check("f4s_reduce_ordered_f32", 16, block=512)
    assert (param(L, 1, 4), param(L, 6, 4)) == (1 << 20, 0)
    assert param(L, 5, 8) - param(L, 4, 8) == 256      # group partials follow the 256-byte ticket
    hp.reduce_sum_into("i32", big, out, n=1 << 20, policy="strict")   # integers: exact under any policy
    check("f4s_reduce_sum_i32", 16 * 4, block=512, cluster=4)
    hp.reduce_ordered_final_into(wso.address + 256, 16, out, accumulate=True)
    L = check("f4s_reduce_ordered_final", 1, block=512)
    assert (param(L, 1, 4), param(L, 4, 4)) == (16, 1)
    # Convert: one kernel per pair and mode, grid = one block per 4096 elements
    for (src, dst, kw, kernel) in [("f32", "f16", {"rounding": "toward_positive"}, "f32_f16_ru"),
                                   ("f32", "bf16", {"rounding": "toward_negative"}, "f32_bf16_rd"),
                                   ("f32", "e4m3", {}, "f32_e4m3_sat"),
                                   ("f32", "e5m2", {"saturation": "none", "rounding": "toward_zero"}, "f32_e5m2_nosat"),
                                   ("e5m2", "f32", {}, "e5m2_f32"), ("f64", "f64", {}, "copy_8"),
                                   ("bool", "bool", {}, "copy_1")]:
        hp.convert_into(src, dst, big, big, n=(1 << 20) + 1, **kw)
        L = check(f"f4s_convert_{kernel}", 257)
        assert (param(L, 2, 4), param(L, 3, 4)) == ((1 << 20) + 1, 0)
    before = count()
    for (src, dst), msg in [(("f32", "f64"), "cannot emit a conversion from float to double"),
                            (("f16", "bf16"), "cannot emit a conversion from __half to __nv_bfloat16"),
                            (("i32", "f32"), "cannot emit a conversion from int to float")]:
        try:
            hp.convert_into(src, dst, big, big, n=8)
        except ValueError as e:
            assert msg in str(e), (str(e), msg)
        else:
            raise AssertionError("expected ValueError")
    assert count() == before
    parts = ctx.allocate("f32", 4096)
    ws = ctx.allocate("u8", hp.block_reduce_workspace_bytes(1 << 20))
    # up to 2^23 elements: the tiles kernel (one 1024-thread CTA per 32 tiles),
    # then the one-CTA upper pass launched as its programmatic dependent
    FAKE.fake_launch_at.restype = C.POINTER(Launch)
    for n, ctas in [(1 << 20, 128), (1, 1)]:
        before = count()
        hp.block_reduce_sum_f32_into(big, parts, out, ws, n=n)
        L = [FAKE.fake_launch_at(i).contents for i in range(before, count())]
        assert [x.name.decode() for x in L] == ["f4s_block_sum_tiles_f32", "f4s_block_sum_upper_f32"]
        assert (L[0].grid[0], L[0].block[0], L[1].grid[0], L[1].block[0]) == (ctas, 1024, 1, 512)
        assert (L[0].programmatic, L[1].programmatic) == (0, 1)
    # above: clusters of 8 CTAs, one per 65536 elements
    n_big = (1 << 23) + 1
    ws_big = ctx.allocate("u8", hp.block_reduce_workspace_bytes(n_big))
    hp.block_reduce_sum_f32_into(big, ctx.allocate("f32", (n_big + 255) // 256), out, ws_big, n=n_big)
    check("f4s_block_reduce_sum_f32", 129 * 8, block=1024, cluster=8)
    ctx.close()


def host_ordered_pipeline():
    """Order-fixed sum of a host array: chunks of whole 256 KiB groups, each
    chunk's partials at its own offset of the group array, then F over all
    groups; the fast policy keeps the accumulate-per-chunk pipeline."""
    import numpy as np
    FAKE.fake_launch_at.restype = C.POINTER(Launch)
    ctx = f4s.CudaContext.open(0)
    hp = ctx.hotpath()
    group = 1 << 18
    half = 3 * group
    staging = ctx.allocate("u8", 256 + 2 * half)
    n = 7 * (group // 4) + 5                    # 8 groups, the last one 20 bytes
    host = np.zeros(n, np.float32)
    ws = ctx.allocate("u8", hp.policy_workspace_bytes("f32", n, "deterministic"))
    assert ws.size_bytes == 256 + 8 * 8

    def launches(since):
        return [FAKE.fake_launch_at(i).contents for i in range(since, count())]

    before = count()
    hp.reduce_host_sum("f32", host, staging, 11, 12, policy="deterministic", workspace=ws)
    L = launches(before)
    assert [x.name.decode() for x in L] == ["f4s_reduce_ordered_f32"] * 3 + ["f4s_reduce_ordered_final"]
    for k, (x, elems, grid) in enumerate(zip(L, [3 * group // 4, 3 * group // 4, group // 4 + 5], [3, 3, 2])):
        assert param(x, 0) == staging.address + 256 + (k % 2) * half
        assert (param(x, 1, 4), param(x, 2, 4)) == (elems, 0)
        assert (param(x, 3), param(x, 4)) == (staging.address, ws.address)
        assert param(x, 5) == ws.address + 256 + 8 * 3 * k and param(x, 6, 4) == 0
        assert tuple(x.grid) == (grid, 1, 1) and x.block[0] == 512 and x.stream == 12
    f = L[3]
    assert (param(f, 0), param(f, 1, 4), param(f, 3), param(f, 4, 4)) == (ws.address + 256, 8, staging.address, 0)
    # empty input: F over no groups
    before = count()
    assert hp.reduce_host_sum("f32", host[:0], staging, 11, 12, policy="strict", workspace=ws) == 0.0
    assert [x.name.decode() for x in launches(before)] == ["f4s_reduce_ordered_final"]
    assert param(last(), 1, 4) == 0
    # fast policy: the geometry-sized kernel per chunk of half / 4 elements, accumulating after the first
    before = count()
    hp.reduce_host_sum("f32", host, staging, 11, 12, policy="fast")
    L = launches(before)
    assert [x.name.decode() for x in L] == ["f4s_reduce_sum_f32"] * 3
    assert [param(x, 7, 4) for x in L] == [0, 1, 1]
    # integers are exact under every policy: the same pipeline
    before = count()
    hp.reduce_host_sum("i32", host.view(np.int32), staging, 11, 12, policy="deterministic")
    assert [x.name.decode() for x in launches(before)] == ["f4s_reduce_sum_i32"] * 3
    # staging below two groups, a short workspace, one stream twice: rejected before any launch
    before = count()
    small = ctx.allocate("u8", 256 + 2 * group - 256)
    for args, msg in [((small, 11, 12, ws), "too small for an order-fixed sum"),
                      ((staging, 11, 12, ctx.allocate("u8", 256 + 8 * 7)), "reduction workspace too small"),
                      ((staging, 11, 11, ws), "two distinct non-null streams")]:
        try:
            hp.reduce_host_sum("f32", host, *args[:3], policy="deterministic", workspace=args[3])
        except ValueError as e:
            assert msg in str(e), (str(e), msg)
        else:
            raise AssertionError("expected ValueError")
    assert count() == before
    # Python-side checks: element size of the host array, unknown policy or type
    for call, msg in [(lambda: hp.reduce_host_sum("f64", host, staging, 11, 12), "8-byte elements"),
                      (lambda: hp.reduce_host_sum("f32", host, staging, 11, 12, policy="exact"), "unknown reduction policy"),
                      (lambda: hp.reduce_host_sum("bool", host, staging, 11, 12), "no ReduceSum accumulator")]:
        try:
            call()
        except ValueError as e:
            assert msg in str(e), (str(e), msg)
        else:
            raise AssertionError("expected ValueError")
    assert count() == before
    ctx.close()


def hp_fp8_rows_grid():
    return 148 * 4  # SM count x fake occupancy


if __name__ == "__main__":
    globals()[sys.argv[1]]()
    print("ok", sys.argv[1])
