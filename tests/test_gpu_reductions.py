"""Full-array reductions on the GPU vs the oracle (parity), plus
full-size (2^32-element) properties against independent torch reductions."""
import numpy as np
import pytest

import flight4s_b200 as f4s
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

SUM_F32_RTOL = 1e-5  # |sum - exact| <= 1e-5 * sum|x|  (f32 sums, per the hot-path contract)
SIZES = [0, 1, 2, 3, 4, 5, 7, 31, 32, 33, 255, 256, 257, 1000, 4096, 4097, 65535, 1 << 20, (1 << 20) + 3, 3_000_001]


def _upload(ctx, values, dtype, misalign):
    """Device buffer holding `values` starting `misalign` elements past a
    256-byte-aligned allocation (garbage around it)."""
    pad = np.full(misalign, 7, dtype=values.dtype)
    tail = np.full(5, 9, dtype=values.dtype)
    buf = ctx.allocate(dtype, misalign + values.size + tail.size)
    buf.copy_from(np.concatenate([pad, values, tail]))
    return buf, buf.address + misalign * values.itemsize


@pytest.mark.parametrize("misalign", [0, 1, 3])
@pytest.mark.parametrize("n", SIZES)
def test_sum_f32_matches_oracle(ctx, hp, n, misalign):
    x = np.random.default_rng(n + 17 * misalign).standard_normal(n).astype(np.float32)
    buf, addr = _upload(ctx, x, "f32", misalign)
    s = hp.reduce_sum_f32(addr, n=n)
    exact, abs_sum = orc.sum_f32_exact(x)
    assert abs(s - exact) <= SUM_F32_RTOL * abs_sum
    if n == 0:
        assert s == 0.0
    buf.close()


@pytest.mark.parametrize("misalign", [0, 2])
@pytest.mark.parametrize("n", SIZES)
def test_sum_i32_bit_exact(ctx, hp, n, misalign):
    x = np.random.default_rng(n).integers(-1000, 1001, n).astype(np.int32)
    buf, addr = _upload(ctx, x, "i32", misalign)
    assert hp.reduce_sum_i32(addr, n=n) == orc.sum_i32(x)
    buf.close()


def test_sum_i32_wraps_like_int32(ctx, hp):
    x = np.full(100_000, 2**31 - 7, np.int32)
    buf, addr = _upload(ctx, x, "i32", 0)
    assert hp.reduce_sum_i32(addr, n=x.size) == orc.sum_i32(x)


@pytest.mark.parametrize("misalign", [0, 1, 3])
@pytest.mark.parametrize("n", SIZES)
def test_argmax_bit_exact(ctx, hp, n, misalign):
    x = np.random.default_rng(n + 5).standard_normal(n).astype(np.float32)
    buf, addr = _upload(ctx, x, "f32", misalign)
    v, i = hp.reduce_argmax_f32(addr, n=n)
    rv, ri = orc.argmax_f32(x)
    assert i == ri
    if n:
        assert np.float32(v).view(np.uint32) == np.float32(rv).view(np.uint32)
    buf.close()


@pytest.mark.parametrize("case", ["ties", "zeros", "inf", "nan", "last", "first", "head", "tail", "all_equal",
                                  "negative"])
def test_argmax_special_values(ctx, hp, case):
    n = 100_003
    rng = np.random.default_rng(1)
    x = rng.standard_normal(n).astype(np.float32)
    if case == "ties":
        x[[5000, 77, 99_999, 40_000]] = 9.0
    elif case == "zeros":
        x[:] = -0.0
        x[[600, 900]] = 0.0
    elif case == "inf":
        x[[123, 5]] = np.inf
    elif case == "nan":
        x[[50_000]] = np.nan
        x[[7]] = np.inf
    elif case == "last":
        x[-1] = 100.0
    elif case == "first":
        x[0] = 100.0
    elif case == "head":
        x[1] = 100.0
    elif case == "tail":
        x[-2] = 100.0
        x[-1] = 100.0
    elif case == "all_equal":
        x[:] = 3.5
    elif case == "negative":
        x = -np.abs(x) - 1.0
    for misalign in (0, 1, 2, 3):
        buf, addr = _upload(ctx, x, "f32", misalign)
        v, i = hp.reduce_argmax_f32(addr, n=n)
        rv, ri = orc.argmax_f32(x)
        assert i == ri, (case, misalign)
        assert np.float32(v).view(np.uint32) == np.float32(rv).view(np.uint32)
        buf.close()


def test_packed_key_and_accumulate_chunks(ctx, hp):
    """Chunked reductions with accumulate == whole-array results."""
    n = 1_000_003
    rng = np.random.default_rng(9)
    x = rng.standard_normal(n).astype(np.float32)
    xi = rng.integers(-1000, 1001, n).astype(np.int32)
    dx, dxi = ctx.allocate("f32", n), ctx.allocate("i32", n)
    dx.copy_from(x)
    dxi.copy_from(xi)
    out_f, out_i, out_a = ctx.allocate("f64", 1), ctx.allocate("i32", 1), ctx.allocate("i64", 2)
    cuts = [0, 1, 4099, 500_000, 999_999, n]
    for k in range(len(cuts) - 1):
        a, b = cuts[k], cuts[k + 1]
        hp.reduce_into(f4s.REDUCE_SUM_F32, dx.address + 4 * a, out_f, n=b - a, accumulate=k > 0)
        hp.reduce_into(f4s.REDUCE_SUM_I32, dxi.address + 4 * a, out_i, n=b - a, accumulate=k > 0)
        hp.reduce_into(f4s.REDUCE_ARGMAX_F32, dx.address + 4 * a, out_a, n=b - a, accumulate=k > 0, index_base=a)
    ctx.synchronize()
    exact, abs_sum = orc.sum_f32_exact(x)
    assert abs(out_f.copy_to_array()[0] - exact) <= SUM_F32_RTOL * abs_sum
    assert out_i.copy_to_array()[0] == orc.sum_i32(xi)
    packed, index = out_a.copy_to_array()
    rv, ri = orc.argmax_f32(x)
    assert index == ri and packed == orc.argmax_packed_key(rv, ri)


@pytest.mark.parametrize("cluster", [1, 2, 4, 8])
def test_cluster_sizes(ctx, hp, cluster):
    n = 5_000_011
    rng = np.random.default_rng(cluster)
    x = rng.standard_normal(n).astype(np.float32)
    xi = rng.integers(-1000, 1001, n).astype(np.int32)
    dx, dxi = ctx.allocate("f32", n), ctx.allocate("i32", n)
    dx.copy_from(x)
    dxi.copy_from(xi)
    hp.set_reduce_cluster(cluster)
    try:
        exact, abs_sum = orc.sum_f32_exact(x)
        s1, s2 = hp.reduce_sum_f32(dx), hp.reduce_sum_f32(dx)
        assert s1 == s2  # deterministic
        assert abs(s1 - exact) <= SUM_F32_RTOL * abs_sum
        assert hp.reduce_sum_i32(dxi) == orc.sum_i32(xi)
        assert hp.reduce_argmax_f32(dx)[1] == orc.argmax_f32(x)[1]
    finally:
        hp.set_reduce_cluster(4)


def test_workspace_too_small_is_rejected(ctx, hp):
    dx, out = ctx.allocate("f32", 1 << 20), ctx.allocate("f64", 1)
    small = ctx.allocate("u8", 64)
    with pytest.raises(ValueError, match="workspace too small"):
        hp.reduce_into(f4s.REDUCE_SUM_F32, dx, out, workspace=small)


def test_full_size_2pow32_against_torch(ctx, hp, torch_dev):
    """2^32 elements (16 GiB): f32 N(0,1) sum / argmax and i32 U[-1000,1000]
    sum, checked against torch's own reductions of the same device data."""
    import torch
    n = 1 << 32
    x = torch.empty(n, dtype=torch.float32, device=torch_dev)
    hp.fill_synthetic(x, n, f4s.NORMAL_F32, seed=0x5EED, p0=0.0, p1=1.0)
    torch.cuda.synchronize()
    s = hp.reduce_sum_f32(x)
    ref = torch.sum(x, dtype=torch.float64).item()
    abs_sum = torch.sum(x.abs(), dtype=torch.float64).item()
    assert abs(s - ref) <= SUM_F32_RTOL * abs_sum
    v, i = hp.reduce_argmax_f32(x)
    assert i == int(torch.argmax(x).item()) and v == float(x.max().item())
    del x
    torch.cuda.empty_cache()
    xi = torch.empty(n, dtype=torch.int32, device=torch_dev)
    hp.fill_synthetic(xi, n, f4s.UNIFORM_I32, seed=0x5EED, ilo=-1000, ihi=1000)
    torch.cuda.synchronize()
    ref_i = int(torch.sum(xi, dtype=torch.int64).item())
    wrapped = (ref_i + 2**31) % 2**32 - 2**31
    assert hp.reduce_sum_i32(xi) == wrapped
    del xi
    torch.cuda.empty_cache()
