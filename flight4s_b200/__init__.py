"""flight4s_b200: the flight4s data-parallel hot path on B200 (sm_100a).

Hand-written sm_100a kernels (full-array and block reductions, vectorAdd,
row-wise softmax / RMSNorm, FP8 E4M3 block quantize / dequantize) behind a
C ABI that mirrors the reference's native runtime boundary, plus a Python
mirror of its typed runtime API.  See include/flight4s_b200.h.
"""
from ._native import CudaDriverFailure, DriverUnavailable, lib  # noqa: F401  (loads the native library)
from .hotpath import (ARGMAX_HOST_OPS, argmax_value, NORMAL_BF16, NORMAL_BF16_OUTLIERS, NORMAL_F32, REDUCE_ARGMAX_F32, REDUCE_SUM_BF16,  # noqa: F401
                      REDUCE_SUM_E4M3, REDUCE_SUM_E5M2, REDUCE_SUM_F16, REDUCE_SUM_F32, REDUCE_SUM_F64, REDUCE_SUM_I32,
                      REDUCE_SUM_U32, ROUNDING, SATURATION, CONVERT_TYPE_CODES, SUM_HOST_OPS, SUM_TYPE_CODES, UNIFORM_BF16,
                      UNIFORM_F32, UNIFORM_I32, ORDERED_GROUP_BYTES, ORDERED_TYPES, POLICIES, Hotpath)
from .runtime import (BFLOAT16, BOOL8, DEVPTR, FLOAT16, FLOAT32, FLOAT64, FP8E4M3, FP8E5M2, INT32, INT64, UINT32,  # noqa: F401
                      Block, Cluster, CudaContext, CudaDeviceBuffer, CudaEvent, CudaFunction, CudaModule,
                      CudaPinnedBuffer, CudaStream, Grid, KernelInvocation, LaunchConfig, NativeArgumentStorage)

__all__ = [name for name in dir() if not name.startswith("_")]
