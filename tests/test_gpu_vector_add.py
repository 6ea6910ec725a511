"""vectorAdd f32 / bf16 vs the oracle (bit-exact) and at full size vs torch."""
import json
from pathlib import Path

import numpy as np
import pytest

import flight4s_b200 as f4s
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def test_reference_known_answer_through_cuda_function_launch(ctx, hp):
    """The reference's typed vectorAdd test (CudaResourcesJniSuite.scala:108-227):
    n = 1024, grid 4 x block 256 on an explicit stream, pinned async copies."""
    ka = json.loads((GOLDEN / "reference_known_answers.json").read_text())["vector_add"]
    n = ka["n"]
    left = np.arange(n, dtype=np.float32)
    right = (np.arange(n) * 2).astype(np.float32)
    fn = hp.module.function("f4s_vector_add_f32", signature=[f4s.DEVPTR, f4s.DEVPTR, f4s.DEVPTR, f4s.INT32])
    stream = ctx.create_stream()
    done = ctx.create_event(timing=False)
    lh, rh, oh = (ctx.allocate_pinned("f32", n) for _ in range(3))
    lb, rb, ob = (ctx.allocate("f32", n) for _ in range(3))
    lh.copy_from(left)
    rh.copy_from(right)
    lb.copy_from_async(lh, stream)
    rb.copy_from_async(rh, stream)
    fn.launch(fn.bind(lb, rb, ob, n), f4s.LaunchConfig(f4s.Grid(n // 256), f4s.Block(256)), stream)
    ob.copy_to_async(oh, stream)
    done.record(stream)
    done.synchronize()
    assert done.query()
    out = oh.to_array()
    assert out[:8].tolist() == ka["expected_first"]
    assert np.array_equal(out, orc.vector_add_f32(left, right))
    assert float(out.astype(np.float64).sum()) == ka["expected_sum_of_outputs"]


@pytest.mark.parametrize("misalign", [0, 1, 3])
@pytest.mark.parametrize("n", [1, 3, 4, 5, 255, 1024, 4097, 1_000_003])
def test_f32_bit_exact(ctx, hp, n, misalign):
    rng = np.random.default_rng(n)
    a = rng.uniform(-1, 1, n).astype(np.float32)
    b = rng.uniform(-1, 1, n).astype(np.float32)
    da, db, dc = (ctx.allocate("f32", n + 4) for _ in range(3))
    da.copy_from(np.concatenate([np.zeros(misalign, np.float32), a, np.zeros(4 - misalign, np.float32)]))
    db.copy_from(np.concatenate([np.zeros(misalign, np.float32), b, np.zeros(4 - misalign, np.float32)]))
    off = 4 * misalign
    hp.vector_add_f32(da.address + off, db.address + off, dc.address + off, n=n)
    ctx.synchronize()
    c = dc.copy_to_array()[misalign:misalign + n]
    assert np.array_equal(c.view(np.uint32), orc.vector_add_f32(a, b).view(np.uint32))


@pytest.mark.parametrize("misalign", [0, 1, 5])
@pytest.mark.parametrize("n", [1, 7, 8, 9, 1000, 65537, 1_000_003])
def test_bf16_bit_exact(ctx, hp, n, misalign):
    rng = np.random.default_rng(n + 1)
    a = orc.f32_to_bf16(rng.uniform(-1, 1, n).astype(np.float32))
    b = orc.f32_to_bf16(rng.standard_normal(n).astype(np.float32) * 1e-3)
    pad = np.zeros(misalign, np.uint16)
    tail = np.zeros(8 - misalign, np.uint16)
    da, db, dc = (ctx.allocate("bf16", n + 8) for _ in range(3))
    da.copy_from(np.concatenate([pad, a, tail]))
    db.copy_from(np.concatenate([pad, b, tail]))
    off = 2 * misalign
    hp.vector_add_bf16(da.address + off, db.address + off, dc.address + off, n=n)
    ctx.synchronize()
    c = dc.copy_to_array()[misalign:misalign + n]
    assert np.array_equal(c, orc.vector_add_bf16(a, b))


def test_bf16_special_values(ctx, hp):
    vals = np.array([0.0, -0.0, 1.0, -1.0, 3.4e38, -3.4e38, 1e-40, -1e-40, np.inf, -np.inf, 1.0 + 2**-8,
                     2**-133, 65504.0, 1e30], np.float32)
    a = orc.f32_to_bf16(np.repeat(vals, len(vals)))
    b = orc.f32_to_bf16(np.tile(vals, len(vals)))
    n = a.size
    da, db, dc = (ctx.allocate("bf16", n) for _ in range(3))
    da.copy_from(a)
    db.copy_from(b)
    hp.vector_add_bf16(da, db, dc)
    ctx.synchronize()
    got, ref = dc.copy_to_array(), orc.vector_add_bf16(a, b)
    nan_got = (got & 0x7F80) == 0x7F80
    nan_got &= (got & 0x7F) != 0
    nan_ref = ((ref & 0x7F80) == 0x7F80) & ((ref & 0x7F) != 0)
    assert np.array_equal(nan_got, nan_ref)
    assert np.array_equal(got[~nan_ref], ref[~nan_ref])


def test_full_size_2pow28_against_torch(ctx, hp, torch_dev):
    import torch
    n = 1 << 28
    for dtype, kind, fn in [(torch.float32, f4s.UNIFORM_F32, hp.vector_add_f32),
                            (torch.bfloat16, f4s.UNIFORM_BF16, hp.vector_add_bf16)]:
        a = torch.empty(n, dtype=dtype, device=torch_dev)
        b = torch.empty(n, dtype=dtype, device=torch_dev)
        c = torch.empty(n, dtype=dtype, device=torch_dev)
        hp.fill_synthetic(a, n, kind, seed=1)
        hp.fill_synthetic(b, n, kind, seed=2)
        fn(a, b, c)
        torch.cuda.synchronize()
        ref = a + b  # torch: IEEE f32 add; bf16 add computed in f32 and rounded
        assert torch.equal(c.view(torch.int16) if dtype == torch.bfloat16 else c.view(torch.int32),
                           ref.view(torch.int16) if dtype == torch.bfloat16 else ref.view(torch.int32))
        del a, b, c, ref
    torch.cuda.empty_cache()


def _typed_values(dtype, n, seed):
    rng = np.random.default_rng(seed)
    if dtype in ("i32", "u32"):
        return rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32).view(orc.CONVERT_STORAGE[dtype])
    if dtype == "f16":
        return (rng.standard_normal(n) * 1000).astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return orc.f32_to_bf16((rng.standard_normal(n) * 1000).astype(np.float32))
    if dtype == "f32":
        return (rng.standard_normal(n) * 1000).astype(np.float32)
    return rng.standard_normal(n) * 1e100


@pytest.mark.parametrize("misalign", [0, 1])
@pytest.mark.parametrize("n", [1, 15, 16, 17, 1000, 65_537, 1_000_003])
@pytest.mark.parametrize("dtype", ["i32", "u32", "f16", "bf16", "f32", "f64"])
def test_every_additive_type_bit_exact(ctx, hp, dtype, n, misalign):
    """f4s_vector_add over the reference's AdditiveTypes, against the
    oracle's `+` (integers wrap; f16 / bf16 round to nearest-even)."""
    a, b = _typed_values(dtype, n, n), _typed_values(dtype, n, n + 1)
    bufs = []
    for arr in (a, b, np.zeros_like(a)):
        d = ctx.allocate(dtype, n + misalign)
        d.copy_from(np.concatenate([np.zeros(misalign, arr.dtype), arr]))
        bufs.append(d)
    item = a.itemsize
    hp.vector_add(dtype, *(d.address + misalign * item for d in bufs), n=n)
    ctx.synchronize()
    got = bufs[2].copy_to_array()[misalign:]
    assert np.array_equal(got.view(np.uint8), orc.vector_add_typed(dtype, a, b).view(np.uint8))


def test_f16_special_values(ctx, hp):
    """Overflow to inf, inf - inf = NaN, subnormal sums, signed zeros."""
    a = np.array([0x7BFF, 0x7C00, 0x0001, 0x8000, 0x3C00, 0xFC00, 0x03FF], np.uint16)
    b = np.array([0x7BFF, 0xFC00, 0x0001, 0x0000, 0xBC00, 0xFC00, 0x0001], np.uint16)
    da, db, dc = (ctx.allocate("f16", a.size) for _ in range(3))
    da.copy_from(a)
    db.copy_from(b)
    hp.vector_add("f16", da, db, dc)
    ctx.synchronize()
    got = orc.decode_to_f32("f16", dc.copy_to_array())
    want = orc.decode_to_f32("f16", orc.vector_add_typed("f16", a, b))
    assert np.array_equal(got, want, equal_nan=True)
    assert np.isposinf(got[0]) and np.isnan(got[1]) and np.isneginf(got[5])


def test_non_additive_types_are_rejected(ctx, hp):
    from flight4s_b200 import _native
    d = ctx.allocate("f32", 8)
    for code in (1, 8, 9, 10):
        rc = _native.lib.f4s_vector_add(hp.handle, 0, code, d.address, d.address, d.address, 8)
        assert rc == _native.STATUS_INVALID_ARGUMENT and "no addition" in _native.last_status()[2]

