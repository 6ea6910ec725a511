"""Host mirror of the reference's typed runtime API over the C ABI.

Names, argument meaning and error behaviour follow
runtime/src/main/scala/flight4s/runtime/cuda/CudaResources.scala
(CudaContext :122-490, CudaStream :492-639, CudaEvent :641-754,
CudaPinnedBuffer :756-859, CudaDeviceBuffer :861-1255, CudaModule :1290-1399,
CudaFunction.launch :1401-1534), core/src/main/scala/flight4s/core/launch/LaunchConfig.scala
and core/src/main/scala/flight4s/core/abi/NativeArgumentStorage.scala.
Rejected arguments raise ValueError (the reference's `require` /
IllegalArgumentException); driver failures raise CudaDriverFailure.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
from typing import Any, Iterable, Optional, Sequence

import numpy as np

from ._native import CudaDriverFailure, check, lib

# --------------------------------------------------------------- ABI codes
# core/src/main/scala/flight4s/core/abi/CudaAbi.scala:12-21
BOOL8, INT32, UINT32, FLOAT16, BFLOAT16, FLOAT32, FLOAT64, FP8E4M3, FP8E5M2, DEVPTR = range(1, 11)
# Addition: signed 64-bit values (element counts / offsets beyond 2^31 - 1)
INT64 = 11
_ABI = {BOOL8: (1, 1, "?"), INT32: (4, 4, "<i4"), UINT32: (4, 4, "<u4"), FLOAT16: (2, 2, "<u2"),
        BFLOAT16: (2, 2, "<u2"), FLOAT32: (4, 4, "<f4"), FLOAT64: (8, 8, "<f8"), FP8E4M3: (1, 1, "u1"),
        FP8E5M2: (1, 1, "u1"), DEVPTR: (8, 8, "<u8"), INT64: (8, 8, "<i8")}

# element storage types of buffers (bf16 / fp8 are carried as raw bits,
# like runtime/src/main/scala/flight4s/runtime/cuda/CudaHostCodec.scala:98-128)
DTYPES = {"f32": np.float32, "f64": np.float64, "i32": np.int32, "u32": np.uint32,
          "bf16": np.uint16, "f16": np.uint16, "e4m3": np.uint8, "e5m2": np.uint8, "u8": np.uint8, "u64": np.uint64,
          "i64": np.int64}


# --------------------------------------------------------- launch config
@dataclasses.dataclass(frozen=True)
class _Dim3:
    x: int
    y: int = 1
    z: int = 1
    _kind = "grid"

    def __post_init__(self):
        for axis in "xyz":
            v = getattr(self, axis)
            if not (isinstance(v, (int, np.integer)) and v > 0):
                raise ValueError(f"{self._kind} {axis} dimension must be positive: {v}")


class Grid(_Dim3):
    _kind = "grid"


class Block(_Dim3):
    _kind = "block"


class Cluster(_Dim3):
    _kind = "cluster"


@dataclasses.dataclass(frozen=True)
class LaunchConfig:
    """core/src/main/scala/flight4s/core/launch/LaunchConfig.scala:48-74."""
    grid: Grid
    block: Block
    dynamic_shared_memory_bytes: int = 0
    cluster: Optional[Cluster] = None

    def __post_init__(self):
        if self.dynamic_shared_memory_bytes < 0:
            raise ValueError(f"dynamic shared memory must not be negative: {self.dynamic_shared_memory_bytes}")
        if self.cluster is not None:
            for axis in "xyz":
                g, c = getattr(self.grid, axis), getattr(self.cluster, axis)
                if g % c != 0:
                    raise ValueError(f"grid {axis} dimension {g} must be divisible by cluster {axis} dimension {c}")


# ----------------------------------------------------- argument storage
class NativeArgumentStorage:
    """Aligned native argument bytes + offsets + descriptor codes, laid out
    like NativeArgumentStorage.materialize (NativeArgumentStorage.scala:65-133):
    each argument at the next offset aligned to its own alignment."""

    def __init__(self, arguments: Sequence[tuple[int, Any]]):
        offsets, codes, end, widest = [], [], 0, 1
        for code, _ in arguments:
            if code not in _ABI:
                raise ValueError(f"unknown descriptor code {code}")
            size, align, _ = _ABI[code]
            off = (end + align - 1) // align * align
            offsets.append(off)
            codes.append(code)
            end = off + size
            widest = max(widest, align)
        self.size_bytes = end
        self._raw = C.create_string_buffer(end + widest)
        base = C.addressof(self._raw)
        self.address = (base + widest - 1) // widest * widest
        view = (C.c_uint8 * max(end, 1)).from_address(self.address)
        buf = np.frombuffer(view, dtype=np.uint8, count=end) if end else np.zeros(0, np.uint8)
        for (code, value), off in zip(arguments, offsets):
            size, _, fmt = _ABI[code]
            if code == BOOL8:
                buf[off] = 1 if value else 0
            else:
                buf[off:off + size] = np.frombuffer(np.array([value], dtype=fmt).tobytes(), np.uint8)
        self.offsets = (C.c_int32 * max(len(offsets), 1))(*offsets)
        self.codes = (C.c_int8 * max(len(codes), 1))(*codes)
        self.count = len(offsets)


# --------------------------------------------------------------- helpers
def device_address(x: Any) -> int:
    """Device address of a CudaDeviceBuffer, a torch CUDA tensor or an int."""
    if isinstance(x, CudaDeviceBuffer):
        return x.address
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    return int(x)


def stream_handle(s: Any) -> int:
    """Native stream handle of a CudaStream, a torch.cuda.Stream, an int, or 0."""
    if s is None:
        return 0
    if isinstance(s, CudaStream):
        return s.handle
    if hasattr(s, "cuda_stream"):
        return int(s.cuda_stream)
    return int(s)


# ------------------------------------------------------------- resources
class CudaContext:
    """A retained primary context (CudaResources.scala:453-490)."""

    def __init__(self, handle: int, ordinal: int, cc: tuple[int, int]):
        self.handle = handle
        self.device_ordinal = ordinal
        self.compute_capability = cc
        self._open = True
        self._hotpath = None

    @staticmethod
    def open(device_ordinal: int = 0) -> "CudaContext":
        if device_ordinal < 0:
            raise ValueError("CUDA device ordinal must not be negative")
        h, major, minor = C.c_uint64(), C.c_int32(), C.c_int32()
        check(lib.f4s_retain_primary_context(device_ordinal, C.byref(h), C.byref(major), C.byref(minor)),
              "CUDA primary context retain")
        return CudaContext(h.value, device_ordinal, (major.value, minor.value))

    @property
    def is_open(self) -> bool:
        return self._open

    def _require_open(self):
        if not self._open:
            raise ValueError("CUDA context is closed")

    def attribute(self, attribute: int) -> int:
        v = C.c_int32()
        check(lib.f4s_device_attribute(self.handle, attribute, C.byref(v)), "CUDA device attribute")
        return v.value

    def load(self, image: bytes) -> "CudaModule":
        """Load a cubin / fatbin image (addition for sm_100a binaries)."""
        self._require_open()
        m = C.c_uint64()
        check(lib.f4s_load_module_image(self.handle, image, len(image), C.byref(m)), "CUDA module image load")
        return CudaModule(self, m.value)

    def load_ptx(self, ptx: bytes) -> "CudaModule":
        self._require_open()
        m = C.c_uint64()
        arr = (C.c_uint8 * len(ptx)).from_buffer_copy(ptx) if ptx else None
        check(lib.f4s_load_ptx(self.handle, arr, len(ptx), C.byref(m)), "CUDA PTX module load")
        return CudaModule(self, m.value)

    def hotpath(self):
        """The sm_100a hot-path module loaded into this context (cached)."""
        from .hotpath import Hotpath
        self._require_open()
        if self._hotpath is None:
            self._hotpath = Hotpath(self)
        return self._hotpath

    def allocate(self, dtype: str, element_count: int) -> "CudaDeviceBuffer":
        self._require_open()
        if element_count < 0:
            raise ValueError(f"element count must not be negative: {element_count}")
        item = np.dtype(DTYPES[dtype]).itemsize
        addr = C.c_uint64()
        check(lib.f4s_allocate_device_memory(self.handle, max(element_count * item, 1), C.byref(addr)),
              "CUDA device allocation")
        return CudaDeviceBuffer(self, addr.value, dtype, element_count)

    def allocate_pinned(self, dtype: str, element_count: int) -> "CudaPinnedBuffer":
        self._require_open()
        if element_count < 0:
            raise ValueError(f"element count must not be negative: {element_count}")
        item = np.dtype(DTYPES[dtype]).itemsize
        p = C.c_void_p()
        check(lib.f4s_allocate_pinned_memory(self.handle, max(element_count * item, 1), C.byref(p)),
              "CUDA pinned allocation")
        return CudaPinnedBuffer(self, p.value, dtype, element_count)

    def create_stream(self, non_blocking: bool = False) -> "CudaStream":
        self._require_open()
        s = C.c_uint64()
        check(lib.f4s_create_stream(self.handle, 1 if non_blocking else 0, C.byref(s)), "CUDA stream create")
        return CudaStream(self, s.value)

    def create_event(self, timing: bool = True, blocking: bool = False) -> "CudaEvent":
        self._require_open()
        e = C.c_uint64()
        flags = (0 if timing else 2) | (1 if blocking else 0)
        check(lib.f4s_create_event(self.handle, flags, C.byref(e)), "CUDA event create")
        return CudaEvent(self, e.value)

    def synchronize(self) -> None:
        self._require_open()
        check(lib.f4s_synchronize_context(self.handle), "CUDA context synchronize")

    def close(self) -> None:
        if not self._open:
            return
        if self._hotpath is not None:
            self._hotpath.close()
            self._hotpath = None
        check(lib.f4s_release_primary_context(self.device_ordinal), "CUDA primary context release")
        self._open = False

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class CudaStream:
    def __init__(self, context: CudaContext, handle: int):
        self.context, self.handle, self._open = context, handle, True

    def synchronize(self) -> None:
        check(lib.f4s_synchronize_stream(self.context.handle, self.handle), "CUDA stream synchronize")

    def wait_for(self, event: "CudaEvent") -> None:
        check(lib.f4s_wait_for_event(self.context.handle, self.handle, event.handle), "CUDA stream wait")

    def close(self) -> None:
        if self._open:
            self.synchronize()
            check(lib.f4s_destroy_stream(self.context.handle, self.handle), "CUDA stream destroy")
            self._open = False


class CudaEvent:
    def __init__(self, context: CudaContext, handle: int):
        self.context, self.handle, self._open = context, handle, True

    def record(self, stream: Optional[CudaStream] = None) -> None:
        check(lib.f4s_record_event(self.context.handle, self.handle, stream_handle(stream)), "CUDA event record")

    def query(self) -> bool:
        done = C.c_int32()
        check(lib.f4s_query_event(self.context.handle, self.handle, C.byref(done)), "CUDA event query")
        return bool(done.value)

    def synchronize(self) -> None:
        check(lib.f4s_synchronize_event(self.context.handle, self.handle), "CUDA event synchronize")

    def elapsed_ms(self, end: "CudaEvent") -> float:
        ms = C.c_float()
        check(lib.f4s_event_elapsed_ms(self.context.handle, self.handle, end.handle, C.byref(ms)),
              "CUDA event elapsed time")
        return ms.value

    def close(self) -> None:
        if self._open:
            check(lib.f4s_destroy_event(self.context.handle, self.handle), "CUDA event destroy")
            self._open = False


class CudaPinnedBuffer:
    """Page-locked host memory with a numpy view (CudaResources.scala:756-859)."""

    def __init__(self, context: CudaContext, address: int, dtype: str, element_count: int):
        self.context, self.address, self.dtype, self.element_count = context, address, dtype, element_count
        self._open = True
        item = np.dtype(DTYPES[dtype]).itemsize
        raw = (C.c_uint8 * max(element_count * item, 1)).from_address(address)
        self.array = np.frombuffer(raw, dtype=DTYPES[dtype], count=element_count)

    @property
    def size_bytes(self) -> int:
        return self.array.nbytes

    def copy_from(self, values: np.ndarray) -> None:
        values = np.asarray(values, dtype=DTYPES[self.dtype]).reshape(-1)
        if values.size != self.element_count:
            raise ValueError(f"pinned buffer holds {self.element_count} elements, got {values.size}")
        self.array[:] = values

    def to_array(self) -> np.ndarray:
        return self.array.copy()

    def close(self) -> None:
        if self._open:
            check(lib.f4s_free_pinned_memory(self.context.handle, self.address), "CUDA pinned free")
            self._open = False
            self.array = None


class CudaDeviceBuffer:
    """Typed device memory (CudaResources.scala:861-1255)."""

    def __init__(self, context: CudaContext, address: int, dtype: str, element_count: int):
        self.context, self.address, self.dtype, self.element_count = context, address, dtype, element_count
        self._open = True

    @property
    def size_bytes(self) -> int:
        return self.element_count * np.dtype(DTYPES[self.dtype]).itemsize

    @property
    def is_open(self) -> bool:
        return self._open

    def copy_from(self, values: np.ndarray) -> None:
        values = np.ascontiguousarray(np.asarray(values, dtype=DTYPES[self.dtype]).reshape(-1))
        if values.size != self.element_count:
            raise ValueError(f"device buffer holds {self.element_count} elements, got {values.size}")
        if values.size:
            check(lib.f4s_copy_host_to_device(self.context.handle, self.address, 0,
                                              values.ctypes.data, values.nbytes), "CUDA host-to-device copy")

    def copy_to_array(self) -> np.ndarray:
        out = np.empty(self.element_count, dtype=DTYPES[self.dtype])
        if out.size:
            check(lib.f4s_copy_device_to_host(self.context.handle, self.address, 0, out.ctypes.data, out.nbytes),
                  "CUDA device-to-host copy")
        return out

    def copy_from_async(self, source: CudaPinnedBuffer, stream: CudaStream, offset_elements: int = 0,
                        count: Optional[int] = None) -> None:
        item = np.dtype(DTYPES[self.dtype]).itemsize
        count = source.element_count if count is None else count
        check(lib.f4s_copy_host_to_device_async(self.context.handle, self.address, offset_elements * item,
                                                source.address, count * item, stream.handle),
              "CUDA async host-to-device copy")

    def copy_to_async(self, destination: CudaPinnedBuffer, stream: CudaStream) -> None:
        check(lib.f4s_copy_device_to_host_async(self.context.handle, self.address, 0, destination.address,
                                                destination.size_bytes, stream.handle),
              "CUDA async device-to-host copy")

    def close(self) -> None:
        if self._open:
            check(lib.f4s_free_device_memory(self.context.handle, self.address), "CUDA device free")
            self._open = False


@dataclasses.dataclass(frozen=True)
class CudaFunctionAttributes:
    max_threads_per_block: int
    static_shared_memory_bytes: int
    constant_memory_bytes: int
    local_memory_bytes: int
    registers_per_thread: int


class CudaModule:
    def __init__(self, context: CudaContext, handle: int, owned: bool = True):
        self.context, self.handle, self._owned, self._open = context, handle, owned, True

    def function(self, name: str, signature: Optional[Sequence[int]] = None) -> "CudaFunction":
        f = C.c_uint64()
        check(lib.f4s_resolve_function(self.context.handle, self.handle, name.encode(), C.byref(f)),
              "CUDA function resolve")
        a = (C.c_int32 * 5)()
        check(lib.f4s_query_function_attributes(self.context.handle, f.value, a), "CUDA function attributes")
        return CudaFunction(self, name, f.value, CudaFunctionAttributes(*a), signature)

    def close(self) -> None:
        if self._open and self._owned:
            check(lib.f4s_unload_module(self.context.handle, self.handle), "CUDA module unload")
        self._open = False


class KernelInvocation:
    """Typed argument values bound to a kernel (KernelSignature.scala:132-155):
    a sequence of (descriptor code, value)."""

    def __init__(self, kernel_name: str, arguments: Iterable[tuple[int, Any]]):
        self.kernel_name = kernel_name
        self.arguments = [(code, device_address(v) if code == DEVPTR else v) for code, v in arguments]

    def storage(self) -> NativeArgumentStorage:
        return NativeArgumentStorage(self.arguments)


class CudaFunction:
    def __init__(self, module: CudaModule, name: str, handle: int, attributes: CudaFunctionAttributes,
                 signature: Optional[Sequence[int]]):
        self.module, self.name, self.handle, self.attributes, self.signature = (module, name, handle, attributes,
                                                                               signature)

    def bind(self, *values: Any) -> KernelInvocation:
        if self.signature is None:
            raise ValueError(f"{self.name} has no declared signature; pass (code, value) pairs to KernelInvocation")
        if len(values) != len(self.signature):
            raise ValueError(f"{self.name} takes {len(self.signature)} arguments, got {len(values)}")
        return KernelInvocation(self.name, zip(self.signature, values))

    def launch(self, invocation: KernelInvocation, config: LaunchConfig, stream: Optional[CudaStream] = None) -> None:
        """Asynchronous launch (CudaResources.scala:1411-1465): validates the
        invocation's kernel identity and dynamic shared memory, then calls the
        native launcher.  Never synchronizes."""
        if invocation.kernel_name != self.name:
            raise ValueError(f"invocation for {invocation.kernel_name} cannot launch {self.name}")
        storage = invocation.storage()
        g, b, c = config.grid, config.block, config.cluster
        check(lib.f4s_launch_kernel(self.module.context.handle, self.handle, stream_handle(stream), g.x, g.y, g.z,
                                    b.x, b.y, b.z, config.dynamic_shared_memory_bytes, 1 if c else 0,
                                    c.x if c else 0, c.y if c else 0, c.z if c else 0,
                                    storage.address if storage.size_bytes else None, storage.size_bytes,
                                    storage.offsets, storage.codes, storage.count),
              "CUDA kernel launch")
