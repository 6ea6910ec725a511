"""ctypes binding of libflight4s_b200.so (declarations: include/flight4s_b200.h).

Importing this module loads the in-tree native library and fails loudly if
it is missing: there is no Python or CPU fallback for any operator.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libflight4s_b200.so"

STATUS_SUCCESS = 0
STATUS_INVALID_ARGUMENT = -1
STATUS_OVERFLOW = -2
STATUS_DRIVER_UNAVAILABLE = -3
STATUS_INTERNAL = -4

u64, i64, i32, u32, f32 = C.c_uint64, C.c_int64, C.c_int32, C.c_uint32, C.c_float
size_t, vp, cp = C.c_size_t, C.c_void_p, C.c_char_p
P = C.POINTER

# name -> (restype, argtypes); must match include/flight4s_b200.h exactly
# (a CPU test parses the header and checks both directions).
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "f4s_abi_version": (C.c_int, []),
    "f4s_last_status_code": (C.c_int, []),
    "f4s_last_status_name": (cp, []),
    "f4s_last_status_description": (cp, []),
    "f4s_last_info_log": (cp, []),
    "f4s_last_error_log": (cp, []),
    "f4s_driver_available": (C.c_int, []),
    "f4s_validate_launch_geometry": (C.c_int, [i32] * 11),
    "f4s_validate_argument_layout": (C.c_int, [vp, i64, P(i32), size_t, P(C.c_int8), size_t]),
    "f4s_launch_kernel": (C.c_int, [u64, u64, u64] + [i32] * 11 + [vp, i64, P(i32), P(C.c_int8), size_t]),
    "f4s_retain_primary_context": (C.c_int, [i32, P(u64), P(i32), P(i32)]),
    "f4s_release_primary_context": (C.c_int, [i32]),
    "f4s_synchronize_context": (C.c_int, [u64]),
    "f4s_device_attribute": (C.c_int, [u64, i32, P(i32)]),
    "f4s_load_ptx": (C.c_int, [u64, P(C.c_uint8), size_t, P(u64)]),
    "f4s_load_module_image": (C.c_int, [u64, vp, size_t, P(u64)]),
    "f4s_unload_module": (C.c_int, [u64, u64]),
    "f4s_resolve_function": (C.c_int, [u64, u64, cp, P(u64)]),
    "f4s_query_function_attributes": (C.c_int, [u64, u64, P(i32)]),
    "f4s_create_stream": (C.c_int, [u64, i32, P(u64)]),
    "f4s_destroy_stream": (C.c_int, [u64, u64]),
    "f4s_synchronize_stream": (C.c_int, [u64, u64]),
    "f4s_create_event": (C.c_int, [u64, i32, P(u64)]),
    "f4s_destroy_event": (C.c_int, [u64, u64]),
    "f4s_record_event": (C.c_int, [u64, u64, u64]),
    "f4s_query_event": (C.c_int, [u64, u64, P(i32)]),
    "f4s_synchronize_event": (C.c_int, [u64, u64]),
    "f4s_wait_for_event": (C.c_int, [u64, u64, u64]),
    "f4s_event_elapsed_ms": (C.c_int, [u64, u64, u64, P(f32)]),
    "f4s_allocate_pinned_memory": (C.c_int, [u64, u64, P(vp)]),
    "f4s_free_pinned_memory": (C.c_int, [u64, vp]),
    "f4s_allocate_device_memory": (C.c_int, [u64, u64, P(u64)]),
    "f4s_free_device_memory": (C.c_int, [u64, u64]),
    "f4s_copy_host_to_device": (C.c_int, [u64, u64, u64, vp, u64]),
    "f4s_copy_host_to_device_async": (C.c_int, [u64, u64, u64, vp, u64, u64]),
    "f4s_copy_device_to_host": (C.c_int, [u64, u64, u64, vp, u64]),
    "f4s_copy_device_to_host_async": (C.c_int, [u64, u64, u64, vp, u64, u64]),
    "f4s_hotpath_open": (C.c_int, [u64, P(vp)]),
    "f4s_hotpath_close": (C.c_int, [vp]),
    "f4s_hotpath_module": (u64, [vp]),
    "f4s_hotpath_sm_count": (C.c_int, [vp]),
    "f4s_hotpath_set_reduce_cluster": (C.c_int, [vp, i32]),
    "f4s_hotpath_set_launch_overlap": (C.c_int, [vp, i32]),
    "f4s_hotpath_wait_timeouts": (C.c_int, [vp, P(u32), i32]),
    "f4s_hotpath_check_bounded_wait": (C.c_int, [vp, u32]),
    "f4s_reduce_workspace_bytes": (u64, [vp]),
    "f4s_reduce_sum_f32": (C.c_int, [vp, u64, u64, u64, u64, u64, u64, i32]),
    "f4s_reduce_sum_i32": (C.c_int, [vp, u64, u64, u64, u64, u64, u64, i32]),
    "f4s_reduce_argmax_f32": (C.c_int, [vp, u64, u64, u64, u64, u64, u64, u64, i32]),
    "f4s_reduce_sum": (C.c_int, [vp, u64, i32, u64, u64, u64, u64, u64, i32]),
    "f4s_reduce_argmax": (C.c_int, [vp, u64, i32, u64, u64, u64, u64, u64, u64, i32]),
    "f4s_reduce_sum_policy": (C.c_int, [vp, u64, i32, i32, u64, u64, u64, u64, u64, i32]),
    "f4s_reduce_policy_workspace_bytes": (C.c_int, [vp, i32, i32, u64, P(u64)]),
    "f4s_reduce_ordered_groups": (C.c_int, [i32, u64, u64, P(u64)]),
    "f4s_reduce_ordered_final": (C.c_int, [vp, u64, u64, u64, u64, i32]),
    "f4s_convert": (C.c_int, [vp, u64, i32, i32, i32, i32, u64, u64, u64]),
    "f4s_reduce_host": (C.c_int, [vp, i32, vp, u64, u64, vp, u64, u64, u64, u64, u64, u64]),
    "f4s_reduce_host_sum_argmax_f32": (C.c_int, [vp, vp, u64, u64, vp, vp, u64, u64, u64, u64, u64, u64]),
    "f4s_reduce_host_sum_policy": (C.c_int, [vp, i32, i32, vp, u64, vp, u64, u64, u64, u64, u64, u64]),
    "f4s_block_reduce_workspace_bytes": (u64, [i32]),
    "f4s_block_reduce_sum_f32": (C.c_int, [vp, u64, u64, i32, u64, u64, u64, u64]),
    "f4s_block_reduce_sum_f32_noalloc": (C.c_int, [vp, u64, u64, i32, u64, u64]),
    "f4s_vector_add_f32": (C.c_int, [vp, u64, u64, u64, u64, i32]),
    "f4s_vector_add_bf16": (C.c_int, [vp, u64, u64, u64, u64, i32]),
    "f4s_vector_add": (C.c_int, [vp, u64, i32, u64, u64, u64, i32]),
    "f4s_softmax_rows_bf16": (C.c_int, [vp, u64, u64, u64, i32, i32]),
    "f4s_rmsnorm_rows_bf16": (C.c_int, [vp, u64, u64, u64, u64, i32, i32, f32]),
    "f4s_fp8_quantize_e4m3": (C.c_int, [vp, u64, u64, u64, u64, i32, i32]),
    "f4s_fp8_dequantize_e4m3": (C.c_int, [vp, u64, u64, u64, u64, i32, i32]),
    "f4s_fill_synthetic": (C.c_int, [vp, u64, u64, u64, u64, u64, u32, i32, f32, f32, f32, f32, i32, i32]),
}


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(there is no fallback implementation)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = _load()


class CudaDriverFailure(RuntimeError):
    """A failed native call; fields of the reference's CudaDriverFailure
    (runtime/src/main/scala/flight4s/runtime/cuda/CudaResources.scala:16-29)."""

    def __init__(self, operation: str, code: int, name: str, description: str, info_log: str = "",
                 error_log: str = ""):
        self.operation = operation
        self.result_code = code
        self.result_name = name
        self.description = description
        self.info_log = info_log
        self.error_log = error_log
        super().__init__(f"{operation} failed with {name} ({code}): {description}"
                         + (f"\n{error_log}" if error_log else ""))


class DriverUnavailable(CudaDriverFailure):
    pass


def last_status() -> tuple[int, str, str, str, str]:
    return (lib.f4s_last_status_code(), lib.f4s_last_status_name().decode(),
            lib.f4s_last_status_description().decode(), lib.f4s_last_info_log().decode(),
            lib.f4s_last_error_log().decode())


def check(status: int, operation: str) -> None:
    """Raise for a non-zero status: ValueError for rejected arguments (the
    reference's IllegalArgumentException), OverflowError for overflows,
    CudaDriverFailure for driver errors."""
    if status == STATUS_SUCCESS:
        return
    code, name, desc, info, err = last_status()
    if status == STATUS_INVALID_ARGUMENT:
        raise ValueError(f"{operation}: {desc}")
    if status == STATUS_OVERFLOW:
        raise OverflowError(f"{operation}: {desc}")
    if status == STATUS_DRIVER_UNAVAILABLE:
        raise DriverUnavailable(operation, status, name, desc)
    raise CudaDriverFailure(operation, status, name, desc, info, err)
