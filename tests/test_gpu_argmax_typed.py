"""max / argmax over every OrderedType (f4s_reduce_argmax): the device
record (packed order key, index) bit for bit against the oracle, with ties,
signed zeros, infinities and NaNs, misaligned heads, index bases and
accumulation across chunks, and host-buffer chunking."""
import numpy as np
import pytest

import flight4s_b200 as f4s
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TYPES = ["i32", "u32", "f16", "bf16", "f32", "f64"]
SIZES = [0, 1, 2, 3, 5, 8, 9, 17, 33, 255, 1000, 4097, 65537, 1_000_003]


def _values(dtype, n, seed, few=False):
    """Random values; `few` draws from 13 distinct values so ties abound."""
    rng = np.random.default_rng(seed)
    storage = orc.CONVERT_STORAGE[dtype]
    if dtype in ("i32", "u32"):
        x = rng.integers(-50, 50, n) if few else rng.integers(-2**31, 2**31, n, dtype=np.int64)
        return (x.astype(np.int64) & 0xFFFFFFFF).astype(np.uint32).view(storage)
    v = rng.integers(-6, 7, n).astype(np.float64) if few else rng.standard_normal(n) * 100
    if dtype == "f16":
        return v.astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return orc.f32_to_bf16(v.astype(np.float32))
    return v.astype(storage)


def _upload(ctx, dtype, x, misalign):
    buf = ctx.allocate(dtype, x.size + misalign + 3)
    buf.copy_from(np.concatenate([np.zeros(misalign, x.dtype), x, np.zeros(3, x.dtype)]))
    return buf, buf.address + misalign * x.itemsize


def _record(ctx, hp, dtype, addr, n, **kw):
    out = ctx.allocate("i64", 2)
    hp.reduce_argmax_into(dtype, addr, out, n=n, **kw)
    ctx.synchronize()
    return out.copy_to_array().tolist()


@pytest.mark.parametrize("few", [False, True])
@pytest.mark.parametrize("misalign", [0, 1, 3])
@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("dtype", TYPES)
def test_record_bit_exact(ctx, hp, dtype, n, misalign, few):
    x = _values(dtype, n, seed=n * 5 + misalign + few, few=few)
    buf, addr = _upload(ctx, dtype, x, misalign)
    assert _record(ctx, hp, dtype, addr, n) == orc.argmax_record(dtype, x)
    buf.close()


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32", "f64"])
def test_total_order_special_values(ctx, hp, dtype):
    """+NaN above +inf above everything; -0 below +0; -NaN below -inf."""
    enc = {"f16": lambda v: np.array(v, np.float16).view(np.uint16),
           "bf16": lambda v: orc.f32_to_bf16(np.array(v, np.float32)),
           "f32": lambda v: np.array(v, np.float32), "f64": lambda v: np.array(v, np.float64)}[dtype]
    cases = [[1.0, np.inf, 3.0, np.inf], [-0.0, 0.0, -0.0], [-np.inf, -1.0, -np.inf],
             [2.0, np.nan, np.inf], [-np.inf, -np.nan, -1e3]]
    for vals in cases:
        x = enc(vals)
        buf, addr = _upload(ctx, dtype, x, 1)
        assert _record(ctx, hp, dtype, addr, x.size) == orc.argmax_record(dtype, x), (dtype, vals)
        buf.close()


@pytest.mark.parametrize("dtype", TYPES)
def test_index_base_and_chunks(ctx, hp, dtype):
    """Chunks reduced with accumulate and a running index base give the
    whole array's record (the packed key keeps 32-bit indices)."""
    x = _values(dtype, 300_001, seed=9, few=True)
    buf, addr = _upload(ctx, dtype, x, 0)
    out = ctx.allocate("i64", 2)
    bounds = [0, 1, 70_000, 70_017, 299_999, x.size]
    for k, (lo, hi) in enumerate(zip(bounds[:-1], bounds[1:])):
        hp.reduce_argmax_into(dtype, addr + lo * x.itemsize, out, n=hi - lo, index_base=lo + 1000,
                              accumulate=k > 0)
    ctx.synchronize()
    assert out.copy_to_array().tolist() == orc.argmax_record(dtype, x, index_base=1000)


@pytest.mark.parametrize("dtype", TYPES)
def test_value_unpacking(ctx, hp, dtype):
    x = _values(dtype, 12_345, seed=3)
    buf, addr = _upload(ctx, dtype, x, 0)
    value, index = hp.reduce_argmax(dtype, addr, n=x.size)
    i, _ = orc.argmax_typed(dtype, x)
    assert index == i
    want = x[i] if dtype in ("i32", "u32", "f32", "f64") else orc.decode_to_f32(dtype, x[i:i + 1])[0]
    assert value == want


@pytest.mark.parametrize("dtype", ["f16", "u32", "f64"])
def test_host_buffer(ctx, hp, dtype):
    x = _values(dtype, 1_000_003, seed=21, few=True)
    pinned = ctx.allocate_pinned(dtype, x.size)
    pinned.copy_from(x)
    staging = ctx.allocate("u8", 256 + 2 * 65536)
    s1, s2 = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    raw = hp.reduce_host(f4s.ARGMAX_HOST_OPS[dtype], pinned.array, staging, s1, s2, index_base=7)
    assert raw.view(np.int64).tolist() == orc.argmax_record(dtype, x, index_base=7)
    s1.close()
    s2.close()


def test_unordered_types_rejected(ctx, hp):
    from flight4s_b200 import _native
    d = ctx.allocate("f32", 8)
    ws = hp.workspace()
    for code in (1, 8, 9, 10):
        rc = _native.lib.f4s_reduce_argmax(hp.handle, 0, code, d.address, 8, d.address, ws.address, ws.size_bytes,
                                           0, 0)
        assert rc == _native.STATUS_INVALID_ARGUMENT and "no max/argmax order" in _native.last_status()[2]


def test_full_size_against_torch(ctx, hp, torch_dev):
    """Benchmark-scale arrays: the index and value of torch.argmax (its
    first maximal element) on the same device data, many ties included
    (normal bf16 / f16 repeat their largest values)."""
    import torch
    g = torch.Generator(device=torch_dev)
    g.manual_seed(0xA5)
    cases = [("f16", torch.float16, 1 << 31), ("bf16", torch.bfloat16, 1 << 31), ("i32", torch.int32, 1 << 32),
             ("f64", torch.float64, 1 << 30)]
    for dtype, tdt, n in cases:
        if tdt == torch.int32:
            x = torch.randint(-1000, 1001, (n,), dtype=torch.int32, device=torch_dev, generator=g)
        else:
            x = torch.randn(n, dtype=torch.float32 if tdt != torch.float64 else tdt, device=torch_dev,
                            generator=g).to(tdt)
        value, index = hp.reduce_argmax(dtype, x.view(torch.int16) if tdt in (torch.float16, torch.bfloat16) else x,
                                        n=n)
        want = int(torch.argmax(x).item())
        assert index == want, (dtype, index, want)
        assert value == x[want].item(), dtype
        del x
        torch.cuda.empty_cache()


@pytest.mark.parametrize("misalign", [0, 1])
@pytest.mark.parametrize("n", [1, 7, 64, 4097, 1_000_003])
@pytest.mark.parametrize("dtype", ["i32", "u32", "f32", "f64"])
def test_every_element_holds_the_smallest_key(ctx, hp, dtype, n, misalign):
    """An array whose every element has the smallest order key of its type
    (i32 INT32_MIN, u32 0, f32 / f64 the negative NaN with every payload bit
    set): the maximum is that key and the first index wins."""
    storage = orc.CONVERT_STORAGE[dtype]
    smallest = {"i32": np.array(-2**31, np.int64).astype(np.int32), "u32": np.uint32(0),
                "f32": np.array(0xFFFFFFFF, np.uint32).view(np.float32),
                "f64": np.array(0xFFFFFFFFFFFFFFFF, np.uint64).view(np.float64)}[dtype]
    x = np.full(n, smallest, dtype=storage)
    buf, addr = _upload(ctx, dtype, x, misalign)
    got = _record(ctx, hp, dtype, addr, n)
    assert got == orc.argmax_record(dtype, x)
    assert got[1] == 0
    buf.close()
