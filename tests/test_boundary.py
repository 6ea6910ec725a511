"""The C-ABI boundary on CPU: symbols, signatures, launch contract parity
with the reference's own source, host-side argument packing, and clean
failure without a driver."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import flight4s_b200 as f4s
from flight4s_b200 import _native
from oracle import oracle as orc

ROOT = Path(__file__).resolve().parents[1]


def header_functions() -> dict[str, str]:
    text = "\n".join(p.read_text() for p in sorted((ROOT / "include").glob("*.h")))
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = {}
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(f4s_\w+)\s*\(([^;{]*?)\)\s*;", text):
        decls[m.group(2)] = m.group(3)
    return decls


def test_library_exports_every_declared_symbol():
    decls = header_functions()
    assert len(decls) >= 50
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = sorted(set(decls) - exported)
    assert not missing, missing
    for name in decls:
        assert getattr(_native.lib, name) is not None


def test_binding_signatures_cover_the_header_exactly():
    decls = header_functions()
    assert set(_native.SIGNATURES) == set(decls)
    for name, params in decls.items():
        n = 0 if params.strip() in ("", "void") else params.count(",") + 1
        assert len(_native.SIGNATURES[name][1]) == n, name


def test_library_links_no_cuda_library():
    out = subprocess.run(["readelf", "-d", str(_native.LIB_PATH)], capture_output=True, text=True, check=True).stdout
    needed = re.findall(r"\[(.*?)\]", "\n".join(l for l in out.splitlines() if "NEEDED" in l))
    assert not [n for n in needed if "cuda" in n or "nccl" in n], needed


def test_abi_version():
    assert _native.lib.f4s_abi_version() == 1000


def _ours_geometry(*g):
    st = _native.lib.f4s_validate_launch_geometry(*g)
    return st, _native.last_status()[2]


def _ours_layout(storage, size, offsets, codes):
    o = (C.c_int32 * max(len(offsets), 1))(*offsets)
    c = (C.c_int8 * max(len(codes), 1))(*codes)
    st = _native.lib.f4s_validate_argument_layout(storage, size, o, len(offsets), c, len(codes))
    return st, _native.last_status()[2]


GEOMETRIES = [
    (4, 2, 1, 32, 8, 1, 2048, 0, 0, 0, 0),   # launch_contract_test.cpp "ordinary"
    (4, 2, 1, 32, 8, 1, 0, 1, 2, 2, 1),      # "clustered"
    (4, 2, 1, 32, 8, 1, 0, 1, 3, 2, 1),      # not divisible
    (4, 2, 1, 32, 8, 1, 2048, 0, 1, 0, 0),   # cluster dims without clusters
    (0, 1, 1, 1, 1, 1, 0, 0, 0, 0, 0),
    (1, 1, 1, 1, -3, 1, 0, 0, 0, 0, 0),
    (1, 1, 1, 1, 1, 1, -1, 0, 0, 0, 0),
    (8, 1, 1, 1024, 1, 1, 0, 1, 8, 1, 1),
    (8, 1, 1, 1024, 1, 1, 0, 1, 0, 1, 1),
    (8, 4, 2, 1, 1, 1, 0, 1, 2, 2, 3),
]


def _verdict(status, message):
    return "OK" if status == 0 else f"ERR {message}"


def test_launch_geometry_matches_reference_contract():
    ref = orc.reference_contract_check([f"G {' '.join(map(str, g))}" for g in GEOMETRIES])
    if ref is None:
        pytest.skip("oracle/_ref not built (reference sources absent)")
    ours = [_verdict(*_ours_geometry(*g)) for g in GEOMETRIES]
    assert ours == ref


def test_randomised_layouts_match_reference_contract():
    rng = np.random.default_rng(11)
    storage = C.create_string_buffer(512 + 16)
    base = (C.addressof(storage) + 15) // 16 * 16
    cases, ours = [], []
    for _ in range(3000):
        k = int(rng.integers(0, 6))
        if rng.random() < 0.5:
            # a layout packed by the NativeArgumentStorage rules, then maybe one defect
            codes = [int(c) for c in rng.choice([1, 2, 3, 4, 5, 6, 7, 8, 9, 10], size=k)]
            packed = f4s.NativeArgumentStorage([(c, 0) for c in codes])
            offsets, size = list(packed.offsets)[:k], packed.size_bytes
            n_codes, misalign, null = k, 0, 0
            defect = int(rng.integers(0, 8))
            if defect == 1 and k:
                offsets[-1] += 1
            elif defect == 2:
                size += int(rng.choice([-1, 1, 8]))
            elif defect == 3 and k:
                codes[int(rng.integers(0, k))] = int(rng.choice([0, 12, 127, -1]))
            elif defect == 4:
                misalign = int(rng.choice([1, 2, 4]))
        else:
            # code 11 is this library's one addition (signed 64-bit); the
            # reference rejects it, so it is compared separately below
            codes = [int(c) for c in rng.choice([1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 0, 12, 127], size=k)]
            offsets = sorted(int(o) for o in rng.integers(-2, 48, size=k))
            n_codes = k if rng.random() > 0.1 else max(k - 1, 0)
            size = int(rng.integers(-1, 64))
            misalign = int(rng.choice([0, 0, 0, 1, 2, 4]))
            null = int(rng.random() < 0.1)
        cases.append(f"L {size} {misalign} {null} {k} {n_codes} " + " ".join(map(str, offsets + codes[:n_codes])))
        o = (C.c_int32 * max(k, 1))(*offsets)
        c = (C.c_int8 * max(n_codes, 1))(*codes[:n_codes])
        st = _native.lib.f4s_validate_argument_layout(None if null else base + misalign, size, o, k, c, n_codes)
        ours.append(_verdict(st, _native.last_status()[2]))
    ref = orc.reference_contract_check(cases)
    if ref is None:
        pytest.skip("oracle/_ref not built (reference sources absent)")
    mismatches = [(c, a, b) for c, a, b in zip(cases, ours, ref) if a != b]
    assert not mismatches, mismatches[:5]
    assert sum(v == "OK" for v in ref) > 20 and sum(v != "OK" for v in ref) > 1000


def test_signed_int64_code_is_the_one_addition():
    """Code 11 (signed 64-bit, 8 bytes, 8-aligned) validates and packs here;
    the reference's contract rejects it as unknown, and both agree on 12."""
    storage = (C.c_uint64 * 3)()
    assert _ours_layout(C.addressof(storage), 24, [0, 8, 16], [2, 11, 10])[0] == 0
    assert "not aligned to 8 bytes" in _ours_layout(C.addressof(storage), 16, [0, 4], [2, 11])[1]
    assert "unknown descriptor code" in _ours_layout(C.addressof(storage), 16, [0, 8], [2, 12])[1]
    packed = f4s.NativeArgumentStorage([(f4s.INT32, 7), (f4s.INT64, (1 << 40) + 3), (f4s.DEVPTR, 0x1000)])
    assert list(packed.offsets)[:3] == [0, 8, 16] and packed.size_bytes == 24
    raw = (C.c_uint8 * 24).from_address(packed.address)
    assert np.frombuffer(bytes(raw[8:16]), np.int64)[0] == (1 << 40) + 3
    ref = orc.reference_contract_check(["L 24 0 0 3 3 0 8 16 2 11 10", "L 16 0 0 2 2 0 8 2 12"])
    if ref is not None:
        assert ref[0] != "OK" and ref[1] != "OK"


def test_reference_contract_test_cases():
    """native/tests/launch_contract_test.cpp, against our validator."""
    storage = (C.c_uint64 * 3)()
    assert _ours_layout(C.addressof(storage), 24, [0, 8, 16], [2, 7, 10])[0] == 0
    for code, size in [(1, 1), (2, 4), (3, 4), (4, 2), (5, 2), (6, 4), (7, 8), (8, 1), (9, 1), (10, 8)]:
        assert _ours_layout(C.addressof(storage), size, [0], [code])[0] == 0
    assert "unknown descriptor code" in _ours_layout(C.addressof(storage), 24, [0, 8, 16], [2, 127, 10])[1]
    assert "overlaps" in _ours_layout(C.addressof(storage), 24, [0, 4, 16], [7, 2, 10])[1]
    o = (C.c_int32 * 3)(0, 8, 16)
    c = (C.c_int8 * 3)(2, 7, 10)
    assert _native.lib.f4s_validate_argument_layout(C.addressof(storage), 24, o, 3, c, 2) == -1
    assert "count mismatch" in _native.last_status()[2]
    assert "layout ends" in _ours_layout(C.addressof(storage), 32, [0, 8, 16], [2, 7, 10])[1]


def test_native_argument_storage_layout_rules():
    """NativeArgumentStorage.materialize: each argument at the next offset
    aligned to its own size; storage ends at the last argument."""
    s = f4s.NativeArgumentStorage([(f4s.INT32, 7), (f4s.DEVPTR, 0xABC), (f4s.BOOL8, True), (f4s.FLOAT64, 1.5),
                                   (f4s.BFLOAT16, 0x3F80), (f4s.FLOAT32, 2.0)])
    assert list(s.offsets)[:s.count] == [0, 8, 16, 24, 32, 36]
    assert s.size_bytes == 40 and s.address % 8 == 0
    raw = bytes((C.c_uint8 * s.size_bytes).from_address(s.address))
    assert raw[0:4] == (7).to_bytes(4, "little") and raw[8:16] == (0xABC).to_bytes(8, "little")
    assert raw[16] == 1 and np.frombuffer(raw[24:32], np.float64)[0] == 1.5
    st = _native.lib.f4s_validate_argument_layout(s.address, s.size_bytes, s.offsets, s.count, s.codes, s.count)
    assert st == 0
    # the reduction kernels' argument list: (ptr, u32, u32, ptr, ptr, u32, u32, i32) -> 44 bytes
    r = f4s.NativeArgumentStorage([(f4s.DEVPTR, 1), (f4s.UINT32, 2), (f4s.UINT32, 0), (f4s.DEVPTR, 3),
                                   (f4s.DEVPTR, 4), (f4s.UINT32, 0), (f4s.UINT32, 0), (f4s.INT32, 0)])
    assert list(r.offsets)[:r.count] == [0, 8, 12, 16, 24, 32, 36, 40] and r.size_bytes == 44


def test_reference_native_argument_storage_suite_cases():
    """The known answers of core/src/test/scala/flight4s/core/abi/NativeArgumentStorageSuite.scala."""
    # "native ABI codes are explicit and unique" (:11-30)
    codes = [f4s.BOOL8, f4s.INT32, f4s.UINT32, f4s.FLOAT16, f4s.BFLOAT16, f4s.FLOAT32, f4s.FLOAT64, f4s.FP8E4M3,
             f4s.FP8E5M2, f4s.DEVPTR]
    assert codes == list(range(1, 11))
    # "arguments occupy aligned slots in one direct buffer" (:32-67):
    # (Boolean true, Double 0.0001, Int 37, in[Float] at 0x1122334455667788)
    s = f4s.NativeArgumentStorage([(f4s.BOOL8, True), (f4s.FLOAT64, 0.0001), (f4s.INT32, 37),
                                   (f4s.DEVPTR, 0x1122334455667788)])
    assert list(s.offsets)[:s.count] == [0, 8, 16, 24] and s.size_bytes == 32
    assert list(s.codes)[:s.count] == [1, 7, 2, 10] and s.address % 8 == 0
    raw = bytes((C.c_uint8 * 32).from_address(s.address))
    assert raw[0] == 1 and np.frombuffer(raw[8:16], np.float64)[0] == 0.0001
    assert int.from_bytes(raw[16:20], "little") == 37
    assert int.from_bytes(raw[24:32], "little") == 0x1122334455667788
    # "empty signatures produce empty direct storage" (:69-77)
    e = f4s.NativeArgumentStorage([])
    assert e.count == 0 and e.size_bytes == 0
    # "launch buffer views retain native order" (:79-93): (Int 12, Float 1.5f)
    v = f4s.NativeArgumentStorage([(f4s.INT32, 12), (f4s.FLOAT32, 1.5)])
    raw = bytes((C.c_uint8 * 8).from_address(v.address))
    assert int.from_bytes(raw[0:4], "little") == 12 and np.frombuffer(raw[4:8], np.float32)[0] == 1.5


def test_reference_native_launch_request_suite_cases():
    """The known answers of core/src/test/scala/flight4s/core/abi/NativeLaunchRequestSuite.scala,
    against the native contract (the Scala-side contract mirrors the C++ one)."""
    # "flattens geometry and argument metadata" (:17-66): (Int 37, Double 1.25, in[Float])
    r = f4s.NativeArgumentStorage([(f4s.INT32, 37), (f4s.FLOAT64, 1.25), (f4s.DEVPTR, 0x1122334455667788)])
    assert list(r.offsets)[:3] == [0, 8, 16] and r.size_bytes == 24 and list(r.codes)[:3] == [2, 7, 10]
    assert _ours_geometry(18, 4, 2, 32, 8, 1, 2048, 1, 3, 2, 1)[0] == 0
    # "accepts empty argument storage" (:83-94)
    buf = (C.c_uint8 * 8)()
    assert _ours_layout(C.addressof(buf), 0, [], [])[0] == 0
    # "rejects invalid metadata counts and codes" (:96-113)
    o = (C.c_int32 * 1)(0)
    assert _native.lib.f4s_validate_argument_layout(C.addressof(buf), 4, o, 1, None, 0) == -1
    assert "unknown descriptor code" in _ours_layout(C.addressof(buf), 4, [0], [127])[1]
    # "rejects invalid offsets and extents" (:115-140)
    store = (C.c_uint64 * 2)()
    a = C.addressof(store)
    assert "negative" in _ours_layout(a, 4, [-1], [2])[1]
    assert "not aligned to 8 bytes" in _ours_layout(a, 8, [1], [7])[1]
    assert "overlaps" in _ours_layout(a, 8, [0, 4], [7, 2])[1]
    for size, offsets, codes in [(4, [0], [7]), (8, [0], [2])]:
        assert _ours_layout(a, size, offsets, codes)[0] == -1


def test_launch_config_validation_messages():
    with pytest.raises(ValueError, match="grid x dimension must be positive"):
        f4s.Grid(0)
    with pytest.raises(ValueError, match="must be divisible by cluster x dimension 3"):
        f4s.LaunchConfig(f4s.Grid(4), f4s.Block(32), cluster=f4s.Cluster(3))
    with pytest.raises(ValueError, match="dynamic shared memory must not be negative"):
        f4s.LaunchConfig(f4s.Grid(1), f4s.Block(32), dynamic_shared_memory_bytes=-1)


def test_calls_without_driver_fail_cleanly():
    if _native.lib.f4s_driver_available():
        pytest.skip("a CUDA driver is present on this host")
    with pytest.raises(_native.DriverUnavailable):
        f4s.CudaContext.open(0)
    st = _native.lib.f4s_launch_kernel(1, 1, 0, 1, 1, 1, 32, 1, 1, 0, 0, 0, 0, 0, None, 0, None, None, 0)
    assert st == _native.STATUS_DRIVER_UNAVAILABLE


def test_invalid_arguments_rejected_before_the_driver():
    # null context / function are rejected as invalid arguments first
    st = _native.lib.f4s_launch_kernel(0, 1, 0, 1, 1, 1, 32, 1, 1, 0, 0, 0, 0, 0, None, 0, None, None, 0)
    assert st in (_native.STATUS_INVALID_ARGUMENT, _native.STATUS_DRIVER_UNAVAILABLE)
    assert _native.lib.f4s_hotpath_sm_count(None) == 0
    assert _native.lib.f4s_reduce_workspace_bytes(None) == 0
    assert _native.lib.f4s_reduce_sum_f32(None, 0, 0, 0, 0, 0, 0, 0) == _native.STATUS_INVALID_ARGUMENT
    assert "hotpath handle must not be null" in _native.last_status()[2]
    assert _native.lib.f4s_block_reduce_workspace_bytes(1 << 20) == 256 + 4 * 16


def test_block_sum_workspace_at_the_static_workspace_limit():
    # 1,069,547,520 elements is the largest block sum whose workspace fits
    # 64 KiB (the allocation-free entry point's static array); one more
    # element needs another level-2 slot
    assert _native.lib.f4s_block_reduce_workspace_bytes(1_069_547_520) == 64 * 1024
    assert _native.lib.f4s_block_reduce_workspace_bytes(1_069_547_521) == 64 * 1024 + 4
