"""ReduceSum over every accumulator input type (f4s_reduce_sum, keyed by the
launch-ABI type code): parity with the oracle on seeded inputs, the device
decoders on every f16 / bf16 / E4M3 / E5M2 code, host-buffer chunking, and
full-size properties against torch's own reductions of the same device data.

Tolerances (|sum - exact| <= rtol * sum|x|): the 16-bit and 8-bit inputs
and f32 are summed in f32 inside each 16-byte vector and in f64 above, so
the error is a few f32 roundings of each vector's magnitude; f64 inputs are
summed in f64 throughout.  E4M3 sums are exact: sixteen E4M3 values never
need more than 24 significant bits, and the f64 sum of those vector sums
is exact below 2^44 (any n < 2^35).  Integer sums are bit-exact.
"""
import numpy as np
import pytest

import flight4s_b200 as f4s
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

RTOL = {"f16": 1e-6, "bf16": 1e-6, "f32": 1e-5, "f64": 1e-12, "e5m2": 1e-6, "e4m3": 0.0}
FLOAT_TYPES = list(RTOL)
SIZES = [0, 1, 2, 3, 7, 8, 15, 16, 17, 31, 33, 255, 257, 1000, 4097, 65537, (1 << 20) + 3, 3_000_001]


def _finite_codes(dtype, codes):
    return codes[np.isfinite(orc.decode_to_f32(dtype, codes))]


def _values(dtype, n, seed):
    rng = np.random.default_rng(seed)
    if dtype in ("e4m3", "e5m2"):
        x = _finite_codes(dtype, rng.integers(0, 256, n + n // 8 + 8).astype(np.uint8))
    elif dtype == "f16":
        x = (rng.standard_normal(n) * 100).astype(np.float16).view(np.uint16)
    elif dtype == "bf16":
        x = orc.f32_to_bf16((rng.standard_normal(n) * 100).astype(np.float32))
    elif dtype == "f32":
        x = rng.standard_normal(n).astype(np.float32)
    elif dtype == "f64":
        x = rng.standard_normal(n) * 1e6
    elif dtype == "u32":
        x = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    else:
        x = rng.integers(-2**31, 2**31, n, dtype=np.int64).astype(np.int32)
    return np.ascontiguousarray(x[:n])


def _upload(ctx, dtype, values, misalign):
    """`values` placed `misalign` elements past a 256-byte-aligned
    allocation, with non-zero garbage around them."""
    pad = np.full(misalign, 0x11, values.dtype)
    tail = np.full(9, 0x22, values.dtype)
    buf = ctx.allocate(dtype, misalign + values.size + tail.size)
    buf.copy_from(np.concatenate([pad, values, tail]))
    return buf, buf.address + misalign * values.itemsize


@pytest.mark.parametrize("misalign", [0, 1, 3])
@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("dtype", FLOAT_TYPES)
def test_float_sums_match_oracle(ctx, hp, dtype, n, misalign):
    x = _values(dtype, n, seed=n * 7 + misalign)
    buf, addr = _upload(ctx, dtype, x, misalign)
    s = hp.reduce_sum(dtype, addr, n=n)
    exact, abs_sum = orc.sum_typed_exact(dtype, x)
    assert abs(s - exact) <= RTOL[dtype] * abs_sum, (s, exact, abs_sum)
    if n == 0:
        assert s == 0.0
    buf.close()


@pytest.mark.parametrize("misalign", [0, 1, 3])
@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("dtype", ["i32", "u32"])
def test_integer_sums_bit_exact(ctx, hp, dtype, n, misalign):
    x = _values(dtype, n, seed=n + 31 * misalign)
    buf, addr = _upload(ctx, dtype, x, misalign)
    got = hp.reduce_sum(dtype, addr, n=n)
    if dtype == "u32":
        assert got == orc.sum_u32(x)
    else:
        assert got == orc.sum_i32(x)
    buf.close()


def test_code_6_and_2_are_the_f32_and_i32_operators(ctx, hp):
    x = _values("f32", 100_003, seed=5)
    xi = _values("i32", 100_003, seed=6)
    b, a = _upload(ctx, "f32", x, 1)
    bi, ai = _upload(ctx, "i32", xi, 1)
    assert hp.reduce_sum("f32", a, n=x.size) == hp.reduce_sum_f32(a, n=x.size)
    assert hp.reduce_sum("i32", ai, n=xi.size) == hp.reduce_sum_i32(ai, n=xi.size)


@pytest.mark.parametrize("dtype", ["e4m3", "e5m2", "f16", "bf16"])
def test_device_decoders_on_every_code(ctx, hp, dtype):
    """One 16-byte vector of copies of each code: the result is the f32
    pairwise sum of those copies, so it pins the kernel's widening of every
    code (inf and NaN included) against the oracle's decoder, which matches
    CUDA's own conversions on every code."""
    codes = 256 if dtype in ("e4m3", "e5m2") else 65536
    storage = np.uint8 if codes == 256 else np.uint16
    per = 16 // np.dtype(storage).itemsize
    data = np.repeat(np.arange(codes, dtype=storage), per)
    buf = ctx.allocate(dtype, data.size)
    buf.copy_from(data)
    outs = ctx.allocate("f64", codes)
    stream = ctx.create_stream(non_blocking=True)
    for c in range(codes):
        hp.reduce_sum_into(dtype, buf.address + 16 * c, outs.address + 8 * c, n=per, stream=stream)
    stream.synchronize()
    got = outs.copy_to_array()
    v = orc.decode_to_f32(dtype, np.arange(codes, dtype=storage))
    with np.errstate(over="ignore", invalid="ignore"):
        level = v
        for _ in range(per.bit_length() - 1):  # pairwise in f32: 2v, 4v, ...
            level = (level + level).astype(np.float32)
    want = level.astype(np.float64)
    same = (got == want) | (np.isnan(got) & np.isnan(want))
    bad = np.nonzero(~same)[0]
    assert bad.size == 0, [(hex(c), got[c], want[c]) for c in bad[:8]]
    stream.close()


@pytest.mark.parametrize("dtype", ["f16", "e5m2", "f64"])
def test_special_values(ctx, hp, dtype):
    inf = {"f16": 0x7C00, "e5m2": 0x7C, "f64": np.inf}[dtype]
    ninf = {"f16": 0xFC00, "e5m2": 0xFC, "f64": -np.inf}[dtype]
    one = {"f16": 0x3C00, "e5m2": 0x3C, "f64": 1.0}[dtype]
    st = orc.STORAGE[dtype]
    for vals, check in [([one] * 1000 + [inf], np.isposinf), ([ninf] + [one] * 77, np.isneginf),
                        ([inf] + [one] * 500 + [ninf], np.isnan)]:
        x = np.array(vals, st)
        buf, addr = _upload(ctx, dtype, x, 1)
        assert check(hp.reduce_sum(dtype, addr, n=x.size)), (dtype, vals[:2])
        buf.close()


@pytest.mark.parametrize("dtype", ["bf16", "e4m3", "u32"])
def test_accumulate_chunks(ctx, hp, dtype):
    x = _values(dtype, 1_000_003, seed=11)
    buf, addr = _upload(ctx, dtype, x, 0)
    out = ctx.allocate("u64", 1)
    bounds = [0, 17, 400_000, 999_999, x.size]
    for k, (lo, hi) in enumerate(zip(bounds[:-1], bounds[1:])):
        hp.reduce_sum_into(dtype, addr + lo * x.itemsize, out, n=hi - lo, accumulate=k > 0)
    ctx.synchronize()
    got = hp.sum_result(dtype, out.copy_to_array())
    if dtype == "u32":
        assert got == orc.sum_u32(x)
    else:
        exact, abs_sum = orc.sum_typed_exact(dtype, x)
        assert abs(got - exact) <= RTOL[dtype] * abs_sum


@pytest.mark.parametrize("dtype", ["e4m3", "e5m2", "f16", "bf16", "f64", "u32"])
@pytest.mark.parametrize("n", [0, 5, 100_003, 3_000_017])
def test_host_buffer_sums(ctx, hp, dtype, n):
    """f4s_reduce_host with the typed sum ops: 4096-byte chunks through a
    small staging buffer, ragged last chunk."""
    x = _values(dtype, n, seed=n + 3)
    pinned = ctx.allocate_pinned(dtype, n)
    pinned.copy_from(x)
    staging = ctx.allocate("u8", 256 + 2 * 4096)
    s1, s2 = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    raw = hp.reduce_host(f4s.SUM_HOST_OPS[dtype], pinned.array, staging, s1, s2)
    got = hp.sum_result(dtype, raw)
    if dtype == "u32":
        assert got == orc.sum_u32(x)
    else:
        exact, abs_sum = orc.sum_typed_exact(dtype, x)
        assert abs(got - exact) <= RTOL[dtype] * abs_sum
    s1.close()
    s2.close()


def test_host_buffer_rejects_wrong_element_size(ctx, hp):
    staging = ctx.allocate("u8", 1024)
    s1, s2 = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    with pytest.raises(ValueError, match="1-byte elements"):
        hp.reduce_host(f4s.REDUCE_SUM_E4M3, np.zeros(8, np.float32), staging, s1, s2)


def test_full_size_against_torch(ctx, hp, torch_dev):
    """2^32 E4M3 and E5M2 codes, 2^31 f16 and bf16 values, 2^30 f64 values
    and 2^32 u32 values on the device, against torch's f64 / i64 sums of the
    same data (computed in chunks).  E4M3 must match exactly."""
    import torch

    def chunked(x, f):
        return sum(f(x[i:i + (1 << 28)]) for i in range(0, x.numel(), 1 << 28))

    g = torch.Generator(device=torch_dev)
    g.manual_seed(0x5EED)
    for dtype, n in [("e4m3", 1 << 32), ("e5m2", 1 << 32)]:
        x = torch.randint(0, 256, (n,), dtype=torch.uint8, device=torch_dev, generator=g)
        if dtype == "e4m3":
            x[(x & 0x7F) == 0x7F] = 0        # NaN codes
            tdt = torch.float8_e4m3fn
        else:
            x[(x & 0x7C) == 0x7C] = 0x3C     # inf / NaN codes -> 1.0
            tdt = torch.float8_e5m2
        ref = chunked(x, lambda c: c.view(tdt).to(torch.float64).sum().item())
        abs_sum = chunked(x, lambda c: c.view(tdt).to(torch.float64).abs().sum().item())
        got = hp.reduce_sum(dtype, x)
        assert abs(got - ref) <= RTOL[dtype] * abs_sum, (dtype, got, ref)
        if dtype == "e4m3":
            assert got == ref
        del x
        torch.cuda.empty_cache()
    for dtype, tdt in [("f16", torch.float16), ("bf16", torch.bfloat16)]:
        x = (torch.randn(1 << 31, dtype=torch.float32, device=torch_dev, generator=g) * 100).to(tdt)
        ref = chunked(x, lambda c: c.to(torch.float64).sum().item())
        abs_sum = chunked(x, lambda c: c.to(torch.float64).abs().sum().item())
        got = hp.reduce_sum(dtype, x)
        assert abs(got - ref) <= RTOL[dtype] * abs_sum, (dtype, got, ref)
        del x
        torch.cuda.empty_cache()
    x = torch.randn(1 << 30, dtype=torch.float64, device=torch_dev, generator=g)
    got = hp.reduce_sum("f64", x)
    ref, abs_sum = x.sum().item(), x.abs().sum().item()
    assert abs(got - ref) <= RTOL["f64"] * abs_sum
    del x
    torch.cuda.empty_cache()
    x = torch.randint(-2**31, 2**31, (1 << 32,), dtype=torch.int32, device=torch_dev, generator=g)
    ref = chunked(x, lambda c: c.to(torch.int64).sum().item()) % 2**32
    assert hp.reduce_sum("u32", x) == ref
    del x
    torch.cuda.empty_cache()
