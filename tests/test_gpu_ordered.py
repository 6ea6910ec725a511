"""Order-fixed ("Deterministic" / "Strict") floating-point sums: bit-exact
against the oracle's operation-by-operation restatement, independent of the
launch grid, with readable group partials and a final tree that reproduces
the total from them."""
import numpy as np
import pytest

import flight4s_b200 as f4s
from flight4s_b200 import _native
from flight4s_b200.runtime import DEVPTR, INT32, UINT32, Block, Grid, LaunchConfig
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TYPES = ["f16", "bf16", "f32", "f64", "e4m3", "e5m2"]
SIZES = [0, 1, 2, 5, 17, 255, 4097, 65537, (1 << 18) + 3, (1 << 20) + 7, 3_000_001]


def _values(dtype, n, seed):
    rng = np.random.default_rng(seed)
    if dtype in ("e4m3", "e5m2"):
        x = rng.integers(0, 256, n + n // 8 + 8).astype(np.uint8)
        return np.ascontiguousarray(x[np.isfinite(orc.decode_to_f32(dtype, x))][:n])
    if dtype == "f16":
        return (rng.standard_normal(n) * 100).astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return orc.f32_to_bf16((rng.standard_normal(n) * 100).astype(np.float32))
    if dtype == "f32":
        return rng.standard_normal(n).astype(np.float32)
    return rng.standard_normal(n) * 1e6


def _upload(ctx, dtype, x, misalign):
    pad = np.full(misalign, 0x33, x.dtype)
    buf = ctx.allocate(dtype, misalign + x.size + 7)
    buf.copy_from(np.concatenate([pad, x, np.full(7, 0x44, x.dtype)]))
    return buf, buf.address + misalign * x.itemsize


def _head(addr, itemsize, n):
    return min(((16 - addr % 16) % 16) // itemsize, n)


def _bits(v: float) -> int:
    return int(np.array([v], np.float64).view(np.uint64)[0])


@pytest.mark.parametrize("misalign", [0, 1, 3])
@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("dtype", TYPES)
def test_ordered_sum_bit_exact_against_oracle(ctx, hp, dtype, n, misalign):
    x = _values(dtype, n, seed=n * 3 + misalign)
    buf, addr = _upload(ctx, dtype, x, misalign)
    for policy in ("deterministic", "strict"):
        got = hp.reduce_sum(dtype, addr, n=n, policy=policy)
        want, _ = orc.sum_ordered(dtype, x, head=_head(addr, x.itemsize, n))
        assert _bits(got) == _bits(want), (dtype, n, misalign, policy, got, want)
    exact, abs_sum = orc.sum_typed_exact(dtype, x)
    assert abs(got - exact) <= (1e-12 if dtype == "f64" else 1e-6) * abs_sum
    buf.close()


def test_integer_types_ignore_policy(ctx, hp):
    x = np.random.default_rng(1).integers(-2**31, 2**31, 100_003, dtype=np.int64).astype(np.int32)
    buf, addr = _upload(ctx, "i32", x, 1)
    for policy in ("strict", "deterministic", "fast"):
        assert hp.reduce_sum("i32", addr, n=x.size, policy=policy) == orc.sum_i32(x)
        assert hp.reduce_sum("u32", addr, n=x.size, policy=policy) == orc.sum_u32(x.view(np.uint32))


@pytest.mark.parametrize("dtype", ["f32", "bf16", "e5m2"])
def test_result_independent_of_grid(ctx, hp, dtype):
    """The same bits from grids of 1, 7, 148 and 1000 CTAs (the product picks
    min(groups, resident CTAs))."""
    n = (5 << 20) + 11
    x = _values(dtype, n, seed=77)
    buf, addr = _upload(ctx, dtype, x, 0)
    fn = hp.module.function(f"f4s_reduce_ordered_{dtype}",
                            [DEVPTR, UINT32, UINT32, DEVPTR, DEVPTR, DEVPTR, INT32])
    ws = ctx.allocate("u8", hp.policy_workspace_bytes(dtype, n, "deterministic"))
    ws.copy_from(np.zeros(ws.element_count, np.uint8))
    out = ctx.allocate("f64", 1)
    want, _ = orc.sum_ordered(dtype, x)
    for grid in (1, 7, 148, 1000):
        fn.launch(fn.bind(addr, n & 0xFFFFFFFF, n >> 32, out, ws, ws.address + 256, 0),
                  LaunchConfig(Grid(grid), Block(512)))
        ctx.synchronize()
        assert _bits(out.copy_to_array()[0]) == _bits(want), grid


@pytest.mark.parametrize("dtype", ["f32", "e4m3"])
def test_group_partials_and_final(ctx, hp, dtype):
    n = (3 << 20) + 5
    x = _values(dtype, n, seed=5)
    buf, addr = _upload(ctx, dtype, x, 0)
    ws = ctx.allocate("u8", hp.policy_workspace_bytes(dtype, n, "deterministic"))
    ws.copy_from(np.zeros(ws.element_count, np.uint8))
    out = ctx.allocate("f64", 2)
    hp.reduce_sum_into(dtype, addr, out, n=n, workspace=ws, policy="deterministic")
    ctx.synchronize()
    ng = hp.ordered_groups(dtype, addr, n)
    want, groups = orc.sum_ordered(dtype, x)
    assert ng == groups.size
    got_groups = ws.copy_to_array()[256:256 + 8 * ng].view(np.float64)
    assert np.array_equal(got_groups.view(np.uint64), groups.view(np.uint64))
    # the final tree alone, over the partials (plus zero padding), and accumulate
    pad = ctx.allocate("f64", ng + 9)
    pad.copy_from(np.concatenate([groups, np.zeros(9)]))
    hp.reduce_ordered_final_into(pad, ng + 9, out.address + 8)
    ctx.synchronize()
    r = out.copy_to_array()
    assert _bits(r[0]) == _bits(want) and _bits(r[1]) == _bits(want)
    hp.reduce_sum_into(dtype, addr, out, n=n, workspace=ws, policy="strict", accumulate=True)
    ctx.synchronize()
    assert _bits(out.copy_to_array()[0]) == _bits(want + want)


HOST_SIZES = [0, 1, 5, 65_536, 65_537, (3 << 18) + 1, (1 << 20) + 7, 3_000_001]


@pytest.mark.parametrize("n", HOST_SIZES)
@pytest.mark.parametrize("dtype", TYPES)
def test_host_buffer_bit_identical(ctx, hp, dtype, n):
    """A host array summed through the chunked pipeline gives the bits of
    the device-resident order-fixed sum at an aligned address, for staging
    areas of 2, 3 and 5 groups per half (chunk boundaries anywhere)."""
    x = _values(dtype, n, seed=n + 17)
    buf, addr = _upload(ctx, dtype, x, 0)
    want, _ = orc.sum_ordered(dtype, x)
    assert _bits(hp.reduce_sum(dtype, addr, n=n, policy="deterministic")) == _bits(want)
    pinned = ctx.allocate_pinned(dtype, max(n, 1))
    pinned.copy_from(np.concatenate([x, np.zeros(max(n, 1) - n, x.dtype)]))
    s1, s2 = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    for groups_per_half in (1, 3, 5):
        staging = ctx.allocate("u8", 256 + 2 * groups_per_half * f4s.ORDERED_GROUP_BYTES + 4096)
        for policy in ("deterministic", "strict"):
            got = hp.reduce_host_sum(dtype, pinned.array[:n], staging, s1, s2, policy=policy)
            assert _bits(got) == _bits(want), (dtype, n, groups_per_half, policy, got, want)
        staging.close()
    s1.close()
    s2.close()
    buf.close()


@pytest.mark.parametrize("dtype", ["f32", "bf16", "e5m2", "f64"])
def test_host_buffer_pageable_odd_start(ctx, hp, dtype):
    """Pageable host memory starting one element past an allocation: the
    order fixes on the array, not on its host address."""
    x = _values(dtype, 1_234_567, seed=31)
    backing = np.concatenate([np.zeros(1, x.dtype), x])
    view = backing[1:]
    staging = ctx.allocate("u8", 256 + 2 * 2 * f4s.ORDERED_GROUP_BYTES)
    s1, s2 = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    want, _ = orc.sum_ordered(dtype, x)
    assert _bits(hp.reduce_host_sum(dtype, view, staging, s1, s2, policy="deterministic")) == _bits(want)
    s1.close()
    s2.close()


def test_host_buffer_fast_and_integers(ctx, hp):
    """The fast policy and the integer sums keep the per-chunk pipeline."""
    x = _values("f32", 1_000_003, seed=4)
    xi = np.random.default_rng(2).integers(-2**31, 2**31, 1_000_003, dtype=np.int64).astype(np.int32)
    staging = ctx.allocate("u8", 256 + 2 * 65536)
    s1, s2 = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    exact, abs_sum = orc.sum_f32_exact(x)
    assert abs(hp.reduce_host_sum("f32", x, staging, s1, s2) - exact) <= 1e-6 * abs_sum
    for policy in ("strict", "fast"):
        assert hp.reduce_host_sum("i32", xi, staging, s1, s2, policy=policy) == orc.sum_i32(xi)
    with pytest.raises(ValueError, match="too small for an order-fixed sum"):
        hp.reduce_host_sum("f32", x, staging, s1, s2, policy="deterministic")
    s1.close()
    s2.close()


def test_workspace_checks(ctx, hp):
    n = 1 << 20
    dx, out = ctx.allocate("f32", n), ctx.allocate("f64", 1)
    need = hp.policy_workspace_bytes("f32", n, "deterministic")
    assert need == 256 + 8 * ((4 * n + (1 << 18) - 1) >> 18)
    small = ctx.allocate("u8", need - 8)
    with pytest.raises(ValueError, match="workspace too small"):
        hp.reduce_sum_into("f32", dx, out, workspace=small, policy="deterministic")
    rc = _native.lib.f4s_reduce_sum_policy(hp.handle, 0, f4s.SUM_TYPE_CODES["f32"], 3, dx.address, n, out.address,
                                           small.address, small.size_bytes, 0)
    assert rc == _native.STATUS_INVALID_ARGUMENT and "unknown reduction policy" in _native.last_status()[2]


def test_full_size_against_torch_and_fast(ctx, hp, torch_dev):
    """2^32 f32 values: the order-fixed sum is within the f32-sum tolerance
    of torch's f64 sum and repeats bit for bit."""
    import torch
    n = 1 << 32
    x = torch.empty(n, dtype=torch.float32, device=torch_dev)
    hp.fill_synthetic(x, n, f4s.NORMAL_F32, seed=0x5EED, p0=0.0, p1=1.0)
    a = hp.reduce_sum("f32", x, policy="deterministic")
    b = hp.reduce_sum("f32", x, policy="deterministic")
    ref = torch.sum(x, dtype=torch.float64).item()
    abs_sum = torch.sum(x.abs(), dtype=torch.float64).item()
    assert _bits(a) == _bits(b)
    assert abs(a - ref) <= 1e-6 * abs_sum
    assert abs(hp.reduce_sum("f32", x) - a) <= 1e-6 * abs_sum
    del x
    torch.cuda.empty_cache()
