"""ctypes loader of the C oracle (oracle.c) — TEST INFRASTRUCTURE ONLY.

Imported by tests/, by __graft_entry__.smoke() as the checker, and by
bench.py's CPU-baseline leg.  The product package never imports it.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
REF_CONTRACT = HERE / "_ref" / "reference_contract_check"


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _load() -> C.CDLL:
    if not LIB.exists() or LIB.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
        build()
    lib = C.CDLL(str(LIB))
    P = C.POINTER
    sig = {
        "orc_philox4x32_10": (None, [P(C.c_uint32), P(C.c_uint32), P(C.c_uint32)]),
        "orc_fill_uniform_f32": (None, [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint32]),
        "orc_fill_uniform_i32": (None, [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint32, C.c_int32,
                                        C.c_int32]),
        "orc_f32_to_bf16_rn": (C.c_uint16, [C.c_float]),
        "orc_bf16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_f32_to_e4m3_satfinite": (C.c_uint8, [C.c_float]),
        "orc_e4m3_to_f32": (C.c_float, [C.c_uint8]),
        "orc_e5m2_to_f32": (C.c_float, [C.c_uint8]),
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_decode_to_f32": (C.c_int, [C.c_int, C.c_void_p, C.c_int64, C.c_void_p]),
        "orc_sum_typed_exactish": (C.c_double, [C.c_int, C.c_void_p, C.c_int64, P(C.c_double)]),
        "orc_sum_u32": (C.c_uint32, [C.c_void_p, C.c_int64]),
        "orc_ordered_final": (C.c_double, [C.c_void_p, C.c_int64]),
        "orc_f32_to_f16": (C.c_uint16, [C.c_float, C.c_int]),
        "orc_f32_to_bf16": (C.c_uint16, [C.c_float, C.c_int]),
        "orc_f32_to_e4m3": (C.c_uint8, [C.c_float, C.c_int]),
        "orc_f32_to_e5m2": (C.c_uint8, [C.c_float, C.c_int]),
        "orc_convert": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int64]),
        "orc_vector_add_typed": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64]),
        "orc_argmax_typed": (C.c_int64, [C.c_int, C.c_void_p, C.c_int64, P(C.c_int64)]),
        "orc_sum_ordered": (C.c_double, [C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, P(C.c_int64)]),
        "orc_vector_add_f32": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64]),
        "orc_vector_add_bf16": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64]),
        "orc_sum_f32_sequential": (C.c_float, [C.c_void_p, C.c_int64]),
        "orc_sum_f32_sequential_from": (C.c_float, [C.c_void_p, C.c_int64, C.c_float]),
        "orc_sum_f32_exactish": (C.c_double, [C.c_void_p, C.c_int64, P(C.c_double)]),
        "orc_sum_i32": (C.c_int32, [C.c_void_p, C.c_int64]),
        "orc_argmax_f32": (C.c_int64, [C.c_void_p, C.c_int64, P(C.c_float)]),
        "orc_argmax_packed_key": (C.c_int64, [C.c_float, C.c_int64]),
        "orc_block_tree_sum_f32": (C.c_float, [C.c_void_p, C.c_int64, C.c_void_p]),
        "orc_softmax_rows_f64": (None, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64]),
        "orc_rmsnorm_rows_f64": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_double]),
        "orc_fp8_quantize": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64]),
        "orc_fp8_dequantize": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64]),
        "orc_mt_sum_f32": (C.c_double, [C.c_void_p, C.c_int64, C.c_int]),
        "orc_mt_sum_i32": (C.c_int32, [C.c_void_p, C.c_int64, C.c_int]),
        "orc_mt_argmax_f32": (C.c_int64, [C.c_void_p, C.c_int64, C.c_int]),
        "orc_mt_vector_add_f32": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


lib = _load()


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def philox(ctr, key) -> list[int]:
    c = (C.c_uint32 * 4)(*ctr)
    k = (C.c_uint32 * 2)(*key)
    o = (C.c_uint32 * 4)()
    lib.orc_philox4x32_10(c, k, o)
    return list(o)


def uniform_f32(n: int, seed: int, offset: int = 0, stream: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib.orc_fill_uniform_f32(_p(out), n, offset, seed, stream)
    return out


def uniform_i32(n: int, seed: int, lo: int, hi: int, offset: int = 0, stream: int = 0) -> np.ndarray:
    out = np.empty(n, np.int32)
    lib.orc_fill_uniform_i32(_p(out), n, offset, seed, stream, lo, hi)
    return out


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    return np.array([lib.orc_f32_to_bf16_rn(float(v)) for v in x], np.uint16) if x.size < 4096 else \
        _vec_bf16(x)


def _vec_bf16(x: np.ndarray) -> np.ndarray:
    # Same rule as orc_f32_to_bf16_rn, vectorised for large arrays (checked
    # against the C function in the tests).
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    return np.array([lib.orc_f32_to_e4m3_satfinite(float(v)) for v in x], np.uint8)


E4M3_TABLE = np.array([lib.orc_e4m3_to_f32(c) for c in range(256)], np.float32)


def vector_add_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    c = np.empty_like(a, dtype=np.float32)
    lib.orc_vector_add_f32(_p(a), _p(b), _p(c), a.size)
    return c


def vector_add_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    c = np.empty_like(a, dtype=np.uint16)
    lib.orc_vector_add_bf16(_p(a), _p(b), _p(c), a.size)
    return c


def sum_f32_sequential(x: np.ndarray, acc: float = 0.0) -> float:
    """Scala's Array[Float].sum (a Float left fold), continued from `acc`."""
    return float(lib.orc_sum_f32_sequential_from(_p(x), x.size, np.float32(acc)))


def sum_f32_exact(x: np.ndarray) -> tuple[float, float]:
    a = C.c_double()
    s = lib.orc_sum_f32_exactish(_p(x), x.size, C.byref(a))
    return float(s), float(a.value)


# launch-ABI type codes (core/src/main/scala/flight4s/core/abi/CudaAbi.scala:11-20)
TYPE_CODES = {"i32": 2, "u32": 3, "f16": 4, "bf16": 5, "f32": 6, "f64": 7, "e4m3": 8, "e5m2": 9}
STORAGE = {"i32": np.int32, "u32": np.uint32, "f16": np.uint16, "bf16": np.uint16, "f32": np.float32,
           "f64": np.float64, "e4m3": np.uint8, "e5m2": np.uint8}


def decode_to_f32(dtype: str, x: np.ndarray) -> np.ndarray:
    """Exact f32 values of f16 / bf16 / f32 / e4m3 / e5m2 storage bits."""
    x = np.ascontiguousarray(x, STORAGE[dtype])
    out = np.empty(x.size, np.float32)
    if lib.orc_decode_to_f32(TYPE_CODES[dtype], _p(x), x.size, _p(out)) != 0:
        raise ValueError(dtype)
    return out


def sum_typed_exact(dtype: str, x: np.ndarray) -> tuple[float, float]:
    """(exact sum, sum of |x|) of a floating-point ReduceSum input."""
    x = np.ascontiguousarray(x, STORAGE[dtype])
    a = C.c_double()
    s = lib.orc_sum_typed_exactish(TYPE_CODES[dtype], _p(x), x.size, C.byref(a))
    return float(s), float(a.value)


def sum_ordered(dtype: str, x: np.ndarray, head: int = 0) -> tuple[float, np.ndarray]:
    """Order-fixed sum (bit-exact restatement of the device kernels) of x,
    whose first `head` elements lie before the first 16-byte boundary;
    returns (total, group partials)."""
    x = np.ascontiguousarray(x, STORAGE[dtype])
    ng = C.c_int64()
    size = (x.size * x.itemsize + (1 << 18) - 1) >> 18
    groups = np.zeros(max(size, 1), np.float64)
    total = lib.orc_sum_ordered(TYPE_CODES[dtype], _p(x), x.size, head, _p(groups), C.byref(ng))
    return float(total), groups[:ng.value]


def ordered_final(groups: np.ndarray) -> float:
    g = np.ascontiguousarray(groups, np.float64)
    return float(lib.orc_ordered_final(_p(g), g.size))


CONVERT_STORAGE = {"bool": np.uint8, "i32": np.int32, "u32": np.uint32, "f16": np.uint16, "bf16": np.uint16,
                   "f32": np.float32, "f64": np.float64, "e4m3": np.uint8, "e5m2": np.uint8}
CONVERT_CODES = {"bool": 1, **TYPE_CODES}


def convert(from_dtype: str, to_dtype: str, x: np.ndarray, rounding: int = 0, saturation: int = 0) -> np.ndarray:
    """The reference's Convert of each element (raw storage bits for the
    16-bit and 8-bit float types)."""
    x = np.ascontiguousarray(x, CONVERT_STORAGE[from_dtype])
    out = np.empty(x.size, CONVERT_STORAGE[to_dtype])
    rc = lib.orc_convert(CONVERT_CODES[from_dtype], CONVERT_CODES[to_dtype], rounding, saturation, _p(x), _p(out),
                         x.size)
    if rc != 0:
        raise ValueError(f"cannot convert {from_dtype} -> {to_dtype}")
    return out


def vector_add_typed(dtype: str, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """`+` of the reference over any AdditiveType (raw bits for f16 / bf16)."""
    a = np.ascontiguousarray(a, CONVERT_STORAGE[dtype])
    b = np.ascontiguousarray(b, CONVERT_STORAGE[dtype])
    c = np.empty_like(a)
    if lib.orc_vector_add_typed(CONVERT_CODES[dtype], _p(a), _p(b), _p(c), a.size) != 0:
        raise ValueError(f"no addition for {dtype}")
    return c


def argmax_typed(dtype: str, x: np.ndarray) -> tuple[int, int]:
    """(first index of the maximum, its order key) over an OrderedType; (-1, 0) when empty."""
    x = np.ascontiguousarray(x, CONVERT_STORAGE[dtype])
    k = C.c_int64()
    i = lib.orc_argmax_typed(CONVERT_CODES[dtype], _p(x), x.size, C.byref(k))
    return int(i), int(k.value)


def argmax_record(dtype: str, x: np.ndarray, index_base: int = 0) -> list[int]:
    """The 16-byte record the device writes (two signed 64-bit words)."""
    i, k = argmax_typed(dtype, x)
    if i < 0:
        return [-(1 << 63), -1]
    i += index_base
    if dtype == "f64":
        return [k, i]
    low = 0xFFFFFFFF - i if i <= 0xFFFFFFFF else 0
    packed = ((k & 0xFFFFFFFF) << 32) | low
    return [packed - (1 << 64) if packed >= 1 << 63 else packed, i]


def sum_u32(x: np.ndarray) -> int:
    x = np.ascontiguousarray(x, np.uint32)
    return int(lib.orc_sum_u32(_p(x), x.size))


def sum_i32(x: np.ndarray) -> int:
    return int(lib.orc_sum_i32(_p(x), x.size))


def argmax_f32(x: np.ndarray) -> tuple[float, int]:
    v = C.c_float()
    i = lib.orc_argmax_f32(_p(x), x.size, C.byref(v))
    return float(v.value), int(i)


def argmax_packed_key(value: float, index: int) -> int:
    return int(lib.orc_argmax_packed_key(value, index))


def block_tree_sum_f32(x: np.ndarray) -> tuple[float, np.ndarray]:
    tiles = (x.size + 255) // 256
    partials = np.zeros(max(tiles, 1), np.float32)
    r = lib.orc_block_tree_sum_f32(_p(x), x.size, _p(partials))
    return float(np.float32(r)), partials[:tiles]


def softmax_rows(x_bf16: np.ndarray, rows: int, cols: int) -> np.ndarray:
    y = np.empty(rows * cols, np.float64)
    lib.orc_softmax_rows_f64(_p(x_bf16), _p(y), rows, cols)
    return y.reshape(rows, cols)


def rmsnorm_rows(x_bf16: np.ndarray, w_bf16: np.ndarray, rows: int, cols: int, eps: float) -> np.ndarray:
    y = np.empty(rows * cols, np.float64)
    lib.orc_rmsnorm_rows_f64(_p(x_bf16), _p(w_bf16), _p(y), rows, cols, eps)
    return y.reshape(rows, cols)


def fp8_quantize(x_bf16: np.ndarray, rows: int, cols: int) -> tuple[np.ndarray, np.ndarray]:
    bpr = (cols + 127) // 128
    codes = np.empty(rows * cols, np.uint8)
    scales = np.empty(rows * bpr, np.float32)
    lib.orc_fp8_quantize(_p(x_bf16), _p(codes), _p(scales), rows, cols)
    return codes, scales


def fp8_dequantize(codes: np.ndarray, scales: np.ndarray, rows: int, cols: int) -> np.ndarray:
    y = np.empty(rows * cols, np.uint16)
    lib.orc_fp8_dequantize(_p(codes), _p(scales), _p(y), rows, cols)
    return y


def reference_contract_check(cases: list[str]) -> list[str] | None:
    """Verdicts of the reference's own launch contract (oracle/_ref binary,
    one process) for case lines in ref_contract_check.cpp's format, or None
    when it was not built (reference sources absent)."""
    if not REF_CONTRACT.exists():
        return None
    out = subprocess.run([str(REF_CONTRACT)], input="\n".join(cases) + "\n", capture_output=True, text=True,
                         check=True).stdout
    return out.splitlines()
