"""Hot-path operators on a CudaContext (the sm_100a kernels behind the
reference's `ReduceSum` node, its vectorAdd / blockReduceSum kernels, and
the row-wise and FP8 ops).  Declarations and reference citations:
include/flight4s_b200.h.

Inputs and outputs may be CudaDeviceBuffers, torch CUDA tensors or raw
device addresses; streams may be CudaStreams, torch.cuda.Streams, raw
handles or None (the legacy default stream).  `*_into` methods are
asynchronous; the plain methods synchronize and return host values.
"""
from __future__ import annotations

import ctypes as C
from typing import Any, Optional

import numpy as np

from ._native import check, lib
from .runtime import (BFLOAT16, BOOL8, FLOAT16, FLOAT32, FLOAT64, FP8E4M3, FP8E5M2, INT32, UINT32, CudaContext,
                      CudaModule, device_address, stream_handle)

REDUCE_SUM_F32, REDUCE_SUM_I32, REDUCE_ARGMAX_F32 = 0, 1, 2
REDUCE_SUM_U32, REDUCE_SUM_F16, REDUCE_SUM_BF16, REDUCE_SUM_F64, REDUCE_SUM_E4M3, REDUCE_SUM_E5M2 = range(3, 9)

# ReduceSum input types by launch-ABI type code, with each element's size in bytes.
SUM_TYPE_CODES = {"i32": INT32, "u32": UINT32, "f16": FLOAT16, "bf16": BFLOAT16, "f32": FLOAT32, "f64": FLOAT64,
                  "e4m3": FP8E4M3, "e5m2": FP8E5M2}
SUM_TYPE_BYTES = {"i32": 4, "u32": 4, "f16": 2, "bf16": 2, "f32": 4, "f64": 8, "e4m3": 1, "e5m2": 1}
# f4s_reduce_host op of each input type's sum
SUM_HOST_OPS = {"f32": REDUCE_SUM_F32, "i32": REDUCE_SUM_I32, "u32": REDUCE_SUM_U32, "f16": REDUCE_SUM_F16,
                "bf16": REDUCE_SUM_BF16, "f64": REDUCE_SUM_F64, "e4m3": REDUCE_SUM_E4M3, "e5m2": REDUCE_SUM_E5M2}
# max / argmax over the OrderedTypes: f4s_reduce_host ops and element sizes
ARGMAX_HOST_OPS = {"f32": REDUCE_ARGMAX_F32, "i32": 9, "u32": 10, "f16": 11, "bf16": 12, "f64": 13}
ARGMAX_TYPE_BYTES = {"f32": 4, "i32": 4, "u32": 4, "f16": 2, "bf16": 2, "f64": 8}
_HOST_OP_BYTES = {**{op: SUM_TYPE_BYTES[t] for t, op in SUM_HOST_OPS.items()},
                  **{op: ARGMAX_TYPE_BYTES[t] for t, op in ARGMAX_HOST_OPS.items()}}

# Convert (core/src/main/scala/flight4s/core/ir/IR.scala:54-70): type codes, RoundingMode and
# SaturationMode ordinals.  The DSL's FP8 conversions default to SaturateFinite, the rest to NoSaturation.
CONVERT_TYPE_CODES = {"bool": BOOL8, "i32": INT32, "u32": UINT32, "f16": FLOAT16, "bf16": BFLOAT16, "f32": FLOAT32,
                      "f64": FLOAT64, "e4m3": FP8E4M3, "e5m2": FP8E5M2}
ROUNDING = {"nearest_even": 0, "toward_zero": 1, "toward_positive": 2, "toward_negative": 3}
SATURATION = {"none": 0, "finite": 1}

# ReductionPolicy of the reference's ReduceSum (core/src/main/scala/flight4s/core/ir/IR.scala:79-82)
POLICIES = {"strict": 0, "deterministic": 1, "fast": 2}
ORDERED_TYPES = ("f16", "bf16", "f32", "f64", "e4m3", "e5m2")
ORDERED_GROUP_BYTES = 256 * 1024  # order-fixed sums: one f64 partial per 256 KiB group

# Synthetic distributions of f4s_fill_synthetic
UNIFORM_F32, UNIFORM_BF16, NORMAL_F32, NORMAL_BF16, UNIFORM_I32, NORMAL_BF16_OUTLIERS = range(6)


def _count(x: Any, n: Optional[int]) -> int:
    if n is not None:
        return int(n)
    if hasattr(x, "element_count"):
        return int(x.element_count)
    if hasattr(x, "numel"):
        return int(x.numel())
    raise ValueError("element count required for a raw device address")


def _nbytes(buf: Any) -> int:
    """Byte size of a CudaDeviceBuffer, a torch tensor or an object with size_bytes."""
    if hasattr(buf, "size_bytes"):
        return int(buf.size_bytes)
    if hasattr(buf, "numel") and hasattr(buf, "element_size"):
        return int(buf.numel() * buf.element_size())
    raise ValueError("buffer size unknown: pass a CudaDeviceBuffer or a torch tensor")


def argmax_value(dtype: str, record: np.ndarray) -> tuple[float | int, int]:
    """(max value, index) of an argmax record of any OrderedType; (nan, -1)
    when the input was empty."""
    r = np.ascontiguousarray(record).view(np.int64)
    index = int(r[1])
    if index < 0:
        return float("nan"), -1
    if dtype == "f64":
        key = int(r[0])
        bits = key ^ ((key >> 63) & 0x7FFFFFFFFFFFFFFF)
        return float(np.array([bits & 0xFFFFFFFFFFFFFFFF], np.uint64).view(np.float64)[0]), index
    key = int(r[0]) >> 32
    if dtype == "f32":
        return unpack_argmax_key(int(r[0]))[0], index
    if dtype == "i32":
        return key, index
    if dtype == "u32":
        return (key & 0xFFFFFFFF) ^ 0x80000000, index
    bits = (key ^ ((key >> 31) & 0x7FFF)) & 0xFFFF
    if dtype == "f16":
        return float(np.array([bits], np.uint16).view(np.float16)[0]), index
    return float(np.array([bits << 16], np.uint32).view(np.float32)[0]), index


def unpack_argmax_key(packed: int) -> tuple[float, int]:
    """(value, index) of a packed argmax key:
    (signed totalOrder key << 32) | (0xFFFFFFFF - index)."""
    key = packed >> 32                      # arithmetic: signed 32-bit key
    bits = key ^ ((key >> 31) & 0x7FFFFFFF)
    value = float(np.array([bits & 0xFFFFFFFF], np.uint32).view(np.float32)[0])
    return value, 0xFFFFFFFF - (packed & 0xFFFFFFFF)


class Hotpath:
    def __init__(self, context: CudaContext):
        self.context = context
        h = C.c_void_p()
        check(lib.f4s_hotpath_open(context.handle, C.byref(h)), "hot-path module load")
        self._h = h
        self.sm_count = lib.f4s_hotpath_sm_count(h)
        self.module = CudaModule(context, lib.f4s_hotpath_module(h), owned=False)
        self.workspace_bytes = int(lib.f4s_reduce_workspace_bytes(h))
        self._workspace = None
        self._ordered_workspace = None
        self._result = None

    # ------------------------------------------------------------ plumbing
    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def workspace(self):
        """Zeroed reduction workspace owned by this hotpath (one per hotpath:
        reductions issued on different streams concurrently need their own,
        allocated with `new_workspace`)."""
        if self._workspace is None:
            self._workspace = self.new_workspace()
        return self._workspace

    def new_workspace(self):
        ws = self.context.allocate("u8", self.workspace_bytes)
        ws.copy_from(np.zeros(self.workspace_bytes, np.uint8))
        return ws

    def policy_workspace_bytes(self, dtype: str, n: int, policy: str = "fast") -> int:
        """Workspace bytes a ReduceSum of `n` elements needs under `policy`."""
        b = C.c_uint64()
        check(lib.f4s_reduce_policy_workspace_bytes(self._h, SUM_TYPE_CODES[dtype], POLICIES[policy], int(n),
                                                    C.byref(b)), "policy workspace size")
        return int(b.value)

    def ordered_workspace(self, nbytes: int):
        """Zeroed workspace of at least `nbytes` for order-fixed sums, kept and
        grown by this hotpath (same stream rule as `workspace`)."""
        if self._ordered_workspace is None or self._ordered_workspace.size_bytes < nbytes:
            if self._ordered_workspace is not None:
                self._ordered_workspace.close()
            self._ordered_workspace = self.context.allocate("u8", nbytes)
            self._ordered_workspace.copy_from(np.zeros(nbytes, np.uint8))
        return self._ordered_workspace

    @staticmethod
    def ordered_groups(dtype: str, address: int, n: int) -> int:
        """Group partials an order-fixed sum of `n` elements at `address` writes."""
        g = C.c_uint64()
        check(lib.f4s_reduce_ordered_groups(SUM_TYPE_CODES[dtype], int(address), int(n), C.byref(g)),
              "ordered group count")
        return int(g.value)

    def _result_buffer(self):
        if self._result is None:
            self._result = self.context.allocate("u64", 2)
        return self._result

    def wait_timeouts(self, reset: bool = False) -> int:
        """Bounded device waits that gave up since the last reset (0 when
        every staged row arrived); synchronizes the context."""
        n = C.c_uint32()
        check(lib.f4s_hotpath_wait_timeouts(self._h, C.byref(n), int(reset)), "wait-timeout count")
        return int(n.value)

    def check_bounded_wait(self, polls: int) -> None:
        """Run the diagnostic kernel whose wait cannot complete (bounded)."""
        check(lib.f4s_hotpath_check_bounded_wait(self._h, polls), "bounded-wait check")

    def set_reduce_cluster(self, cluster: int) -> None:
        check(lib.f4s_hotpath_set_reduce_cluster(self._h, cluster), "reduction cluster size")

    def set_launch_overlap(self, enable: bool) -> None:
        """Let each device-resident full-array reduction start streaming its
        input while the kernel launched before it on the same stream
        finishes (programmatic dependent launch).  Only for callers that
        never launch a kernel writing a reduction's input immediately before
        that reduction on the same stream."""
        check(lib.f4s_hotpath_set_launch_overlap(self._h, 1 if enable else 0), "launch overlap")

    def close(self) -> None:
        if self._h is not None:
            for b in (self._workspace, self._ordered_workspace, self._result):
                if b is not None:
                    b.close()
            check(lib.f4s_hotpath_close(self._h), "hot-path module unload")
            self._h = None

    # ------------------------------------------------- full-array reductions
    def reduce_into(self, op: int, x: Any, out: Any, n: Optional[int] = None, stream: Any = None,
                    accumulate: bool = False, index_base: int = 0, workspace: Any = None) -> None:
        ws = self.workspace() if workspace is None else workspace
        ws_bytes = _nbytes(ws)
        args = (self._h, stream_handle(stream), device_address(x), _count(x, n), device_address(out),
                device_address(ws), ws_bytes)
        if op == REDUCE_SUM_F32:
            check(lib.f4s_reduce_sum_f32(*args, int(accumulate)), "reduce_sum_f32")
        elif op == REDUCE_SUM_I32:
            check(lib.f4s_reduce_sum_i32(*args, int(accumulate)), "reduce_sum_i32")
        elif op == REDUCE_ARGMAX_F32:
            check(lib.f4s_reduce_argmax_f32(*args, index_base, int(accumulate)), "reduce_argmax_f32")
        else:
            raise ValueError(f"unknown reduction op {op}")

    def _reduce_sync(self, op: int, x: Any, n: Optional[int], stream: Any) -> np.ndarray:
        out = self._result_buffer()
        self.reduce_into(op, x, out, n=n, stream=stream)
        if stream is not None and hasattr(stream, "synchronize"):
            stream.synchronize()
        self.context.synchronize()
        return out.copy_to_array()

    def reduce_sum_f32(self, x: Any, n: Optional[int] = None, stream: Any = None) -> float:
        return float(self._reduce_sync(REDUCE_SUM_F32, x, n, stream).view(np.float64)[0])

    def reduce_sum_i32(self, x: Any, n: Optional[int] = None, stream: Any = None) -> int:
        return int(self._reduce_sync(REDUCE_SUM_I32, x, n, stream).view(np.int32)[0])

    def reduce_argmax_f32(self, x: Any, n: Optional[int] = None, stream: Any = None) -> tuple[float, int]:
        """(max value, index of its first occurrence); (nan, -1) when empty."""
        r = self._reduce_sync(REDUCE_ARGMAX_F32, x, n, stream).view(np.int64)
        index = int(r[1])
        if index < 0:
            return float("nan"), -1
        return unpack_argmax_key(int(r[0]))[0], index

    def reduce_argmax_into(self, dtype: str, x: Any, out: Any, n: Optional[int] = None, stream: Any = None,
                           accumulate: bool = False, index_base: int = 0, workspace: Any = None) -> None:
        """max / argmax over any OrderedType ("i32", "u32", "f16", "bf16",
        "f32", "f64"): the 16-byte record of f4s_reduce_argmax.  Asynchronous."""
        if dtype not in ARGMAX_TYPE_BYTES:
            raise ValueError(f"no max/argmax order for {dtype!r}")
        ws = self.workspace() if workspace is None else workspace
        check(lib.f4s_reduce_argmax(self._h, stream_handle(stream), CONVERT_TYPE_CODES[dtype], device_address(x),
                                    _count(x, n), device_address(out), device_address(ws), _nbytes(ws), index_base,
                                    int(accumulate)), f"reduce_argmax {dtype}")

    def reduce_argmax(self, dtype: str, x: Any, n: Optional[int] = None, stream: Any = None):
        """(max value, index of its first occurrence); (nan, -1) when empty."""
        out = self._result_buffer()
        self.reduce_argmax_into(dtype, x, out, n=n, stream=stream)
        if stream is not None and hasattr(stream, "synchronize"):
            stream.synchronize()
        self.context.synchronize()
        return argmax_value(dtype, out.copy_to_array())

    def reduce_sum_into(self, dtype: str, x: Any, out: Any, n: Optional[int] = None, stream: Any = None,
                        accumulate: bool = False, workspace: Any = None, policy: str = "fast") -> None:
        """ReduceSum of any accumulator input type ("i32", "u32", "f16", "bf16",
        "f32", "f64", "e4m3", "e5m2"): 4-byte wrapping sum for the integer
        types, f64 for the rest.  `policy` "strict" / "deterministic" selects
        the order-fixed kernels for floating-point inputs (the same bits on
        any launch shape, device or GPU count), "fast" the geometry-sized
        ones.  Asynchronous."""
        if dtype not in SUM_TYPE_CODES:
            raise ValueError(f"no ReduceSum accumulator for {dtype!r}")
        if policy not in POLICIES:
            raise ValueError(f"unknown reduction policy {policy!r}")
        count = _count(x, n)
        if workspace is not None:
            ws = workspace
        elif policy != "fast" and dtype in ORDERED_TYPES:
            ws = self.ordered_workspace(self.policy_workspace_bytes(dtype, count, policy))
        else:
            ws = self.workspace()
        check(lib.f4s_reduce_sum_policy(self._h, stream_handle(stream), SUM_TYPE_CODES[dtype], POLICIES[policy],
                                        device_address(x), count, device_address(out), device_address(ws),
                                        _nbytes(ws), int(accumulate)), f"reduce_sum {dtype} ({policy})")

    def reduce_ordered_final_into(self, groups: Any, count: int, out: Any, stream: Any = None,
                                  accumulate: bool = False) -> None:
        """Order-fixed total of `count` f64 group partials (device memory)."""
        check(lib.f4s_reduce_ordered_final(self._h, stream_handle(stream), device_address(groups), int(count),
                                           device_address(out), int(accumulate)), "reduce_ordered_final")

    def reduce_sum(self, dtype: str, x: Any, n: Optional[int] = None, stream: Any = None,
                   policy: str = "fast") -> float | int:
        """Synchronous ReduceSum: int (signed for i32, unsigned for u32) or float."""
        out = self._result_buffer()
        self.reduce_sum_into(dtype, x, out, n=n, stream=stream, policy=policy)
        if stream is not None and hasattr(stream, "synchronize"):
            stream.synchronize()
        self.context.synchronize()
        return self.sum_result(dtype, out.copy_to_array())

    @staticmethod
    def sum_result(dtype: str, raw: np.ndarray) -> float | int:
        """Host value of a sum record (the first 8 bytes of `raw`)."""
        raw = np.ascontiguousarray(raw).view(np.uint8)[:8]
        if dtype == "i32":
            return int(raw[:4].view(np.int32)[0])
        if dtype == "u32":
            return int(raw[:4].view(np.uint32)[0])
        return float(raw.view(np.float64)[0])

    def reduce_host(self, op: int, host: np.ndarray, staging: Any, copy_stream: Any, compute_stream: Any,
                    workspace: Any = None, index_base: int = 0) -> np.ndarray:
        """End-to-end reduction of a host array (pinned for overlap) through
        `staging` device memory; returns the raw 8/4/16-byte result."""
        ws = self.workspace() if workspace is None else workspace
        out = np.zeros(2, np.uint64)
        host = np.ascontiguousarray(host)
        if op not in _HOST_OP_BYTES:
            raise ValueError(f"unknown reduction op {op}")
        if host.itemsize != _HOST_OP_BYTES[op]:
            raise ValueError(f"reduction op {op} reads {_HOST_OP_BYTES[op]}-byte elements, got {host.dtype}")
        check(lib.f4s_reduce_host(self._h, op, host.ctypes.data, host.size, index_base, out.ctypes.data,
                                  device_address(staging), _nbytes(staging), device_address(ws), _nbytes(ws),
                                  stream_handle(copy_stream), stream_handle(compute_stream)), "reduce_host")
        return out

    def reduce_host_sum(self, dtype: str, host: np.ndarray, staging: Any, copy_stream: Any, compute_stream: Any,
                        policy: str = "fast", workspace: Any = None) -> float | int:
        """ReduceSum of a host array (pinned for overlap) under `policy`: the
        order-fixed policies stage whole 256 KiB groups and give the same
        bits as `reduce_sum` of the array at a 16-byte-aligned device
        address, for any staging size."""
        if dtype not in SUM_TYPE_CODES:
            raise ValueError(f"no ReduceSum accumulator for {dtype!r}")
        if policy not in POLICIES:
            raise ValueError(f"unknown reduction policy {policy!r}")
        host = np.ascontiguousarray(host)
        if host.itemsize != SUM_TYPE_BYTES[dtype]:
            raise ValueError(f"{dtype} sums read {SUM_TYPE_BYTES[dtype]}-byte elements, got {host.dtype}")
        if workspace is not None:
            ws = workspace
        elif policy != "fast" and dtype in ORDERED_TYPES:
            ws = self.ordered_workspace(self.policy_workspace_bytes(dtype, host.size, policy))
        else:
            ws = self.workspace()
        out = np.zeros(1, np.uint64)
        check(lib.f4s_reduce_host_sum_policy(self._h, SUM_TYPE_CODES[dtype], POLICIES[policy], host.ctypes.data,
                                             host.size, out.ctypes.data, device_address(staging), _nbytes(staging),
                                             device_address(ws), _nbytes(ws), stream_handle(copy_stream),
                                             stream_handle(compute_stream)), f"reduce_host_sum {dtype} ({policy})")
        return self.sum_result(dtype, out)

    def reduce_host_sum_argmax(self, host: np.ndarray, staging: Any, copy_stream: Any, compute_stream: Any,
                               workspace: Any = None, index_base: int = 0) -> tuple[np.ndarray, np.ndarray]:
        """f32 sum and argmax of a host array from one transfer of each chunk;
        returns (8-byte sum record, 16-byte argmax record)."""
        ws = self.workspace() if workspace is None else workspace
        s = np.zeros(1, np.uint64)
        a = np.zeros(2, np.uint64)
        host = np.ascontiguousarray(host)
        check(lib.f4s_reduce_host_sum_argmax_f32(self._h, host.ctypes.data, host.size, index_base, s.ctypes.data,
                                                 a.ctypes.data, device_address(staging), _nbytes(staging),
                                                 device_address(ws), _nbytes(ws), stream_handle(copy_stream),
                                                 stream_handle(compute_stream)), "reduce_host_sum_argmax")
        return s, a

    # -------------------------------------------------------------- Convert
    def convert_into(self, from_dtype: str, to_dtype: str, x: Any, y: Any, n: Optional[int] = None,
                     rounding: str = "nearest_even", saturation: Optional[str] = None, stream: Any = None) -> None:
        """y[i] = Convert(x[i]) with the reference's rounding / saturation modes
        ("nearest_even" | "toward_zero" | "toward_positive" | "toward_negative";
        "none" | "finite", default "finite" for FP8 targets as in the DSL).
        Asynchronous."""
        if saturation is None:
            saturation = "finite" if to_dtype in ("e4m3", "e5m2") else "none"
        for d in (from_dtype, to_dtype):
            if d not in CONVERT_TYPE_CODES:
                raise ValueError(f"no Convert type {d!r}")
        check(lib.f4s_convert(self._h, stream_handle(stream), CONVERT_TYPE_CODES[from_dtype],
                              CONVERT_TYPE_CODES[to_dtype], ROUNDING[rounding], SATURATION[saturation],
                              device_address(x), device_address(y), _count(x, n)),
              f"convert {from_dtype} -> {to_dtype}")

    # ------------------------------------------------------------ block sum
    @staticmethod
    def block_reduce_workspace_bytes(n: int) -> int:
        return int(lib.f4s_block_reduce_workspace_bytes(n))

    def block_reduce_sum_f32_into(self, x: Any, partials: Any, out: Any, workspace: Any, n: Optional[int] = None,
                                  stream: Any = None) -> None:
        check(lib.f4s_block_reduce_sum_f32(self._h, stream_handle(stream), device_address(x), _count(x, n),
                                           device_address(partials), device_address(out),
                                           device_address(workspace), _nbytes(workspace)),
              "block_reduce_sum_f32")

    # ---------------------------------------------------------- elementwise
    def vector_add_f32(self, a: Any, b: Any, c: Any, n: Optional[int] = None, stream: Any = None) -> None:
        check(lib.f4s_vector_add_f32(self._h, stream_handle(stream), device_address(a), device_address(b),
                                     device_address(c), _count(a, n)), "vectorAdd f32")

    def vector_add_bf16(self, a: Any, b: Any, c: Any, n: Optional[int] = None, stream: Any = None) -> None:
        check(lib.f4s_vector_add_bf16(self._h, stream_handle(stream), device_address(a), device_address(b),
                                      device_address(c), _count(a, n)), "vectorAdd bf16")

    def vector_add(self, dtype: str, a: Any, b: Any, c: Any, n: Optional[int] = None, stream: Any = None) -> None:
        """c = a + b for any AdditiveType: "i32", "u32", "f16", "bf16", "f32", "f64"."""
        if dtype not in ("i32", "u32", "f16", "bf16", "f32", "f64"):
            raise ValueError(f"no addition for {dtype!r}")
        check(lib.f4s_vector_add(self._h, stream_handle(stream), CONVERT_TYPE_CODES[dtype], device_address(a),
                                 device_address(b), device_address(c), _count(a, n)), f"vectorAdd {dtype}")

    # ------------------------------------------------------------- row-wise
    def softmax_rows_bf16(self, x: Any, y: Any, rows: int, cols: int, stream: Any = None) -> None:
        check(lib.f4s_softmax_rows_bf16(self._h, stream_handle(stream), device_address(x), device_address(y),
                                        rows, cols), "softmax rows bf16")

    def rmsnorm_rows_bf16(self, x: Any, w: Any, y: Any, rows: int, cols: int, eps: float = 1e-6,
                          stream: Any = None) -> None:
        check(lib.f4s_rmsnorm_rows_bf16(self._h, stream_handle(stream), device_address(x), device_address(w),
                                        device_address(y), rows, cols, eps), "rmsnorm rows bf16")

    # ------------------------------------------------------------------ fp8
    def fp8_quantize_e4m3(self, x: Any, codes: Any, scales: Any, rows: int, cols: int, stream: Any = None) -> None:
        check(lib.f4s_fp8_quantize_e4m3(self._h, stream_handle(stream), device_address(x), device_address(codes),
                                        device_address(scales), rows, cols), "fp8 e4m3 quantize")

    def fp8_dequantize_e4m3(self, codes: Any, scales: Any, y: Any, rows: int, cols: int, stream: Any = None) -> None:
        check(lib.f4s_fp8_dequantize_e4m3(self._h, stream_handle(stream), device_address(codes),
                                          device_address(scales), device_address(y), rows, cols),
              "fp8 e4m3 dequantize")

    # ------------------------------------------------------------ synthetic
    def fill_synthetic(self, out: Any, n: int, kind: int, seed: int, offset: int = 0, stream_id: int = 0,
                       p0: float = 0.0, p1: float = 1.0, p2: float = 0.0, p3: float = 1.0, ilo: int = 0,
                       ihi: int = 0, stream: Any = None) -> None:
        check(lib.f4s_fill_synthetic(self._h, stream_handle(stream), device_address(out), n, offset, seed, stream_id,
                                     kind, p0, p1, p2, p3, ilo, ihi), "synthetic fill")
