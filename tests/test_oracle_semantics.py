"""Internal consistency of the oracle's definitions (CPU)."""
import math

import numpy as np
import pytest

from oracle import oracle as orc


@pytest.mark.parametrize("n", [0, 1, 5, 255, 256, 257, 65536, 65537, 200_003])
def test_block_tree_is_exact_on_small_integers(n):
    x = (np.arange(n) % 8).astype(np.float32)
    total, partials = orc.block_tree_sum_f32(x)
    assert total == float(x.astype(np.int64).sum())
    assert partials.size == (n + 255) // 256


def test_block_tree_close_to_exact_sum():
    x = orc.uniform_f32(1 << 20, seed=1)
    total, _ = orc.block_tree_sum_f32(x)
    exact, abs_sum = orc.sum_f32_exact(x)
    assert abs(total - exact) <= 1e-5 * abs_sum


def test_argmax_ties_and_total_order():
    x = np.array([1.0, 3.0, -2.0, 3.0, 3.0], np.float32)
    assert orc.argmax_f32(x) == (3.0, 1)
    z = np.array([-0.0, 0.0, -0.0], np.float32)
    assert orc.argmax_f32(z)[1] == 1  # +0 > -0 under totalOrder
    inf = np.array([1.0, np.inf, 5.0, np.inf], np.float32)
    assert orc.argmax_f32(inf) == (math.inf, 1)
    nan = np.array([1.0, np.nan, np.inf], np.float32)
    assert orc.argmax_f32(nan)[1] == 1  # +NaN sorts above +inf
    assert orc.argmax_f32(np.zeros(0, np.float32))[1] == -1


def test_packed_argmax_key_orders_like_value_then_index():
    keys = [orc.argmax_packed_key(v, i) for v, i in [(1.0, 5), (1.0, 3), (2.0, 9), (-1.0, 0), (np.inf, 2**32 - 1)]]
    assert max(keys[:2]) == keys[1]            # equal value: lower index wins
    assert max(keys[:3]) == keys[2]            # larger value wins
    assert keys[3] < keys[0]
    assert max(keys) == keys[4]


def test_i32_sum_wraps():
    x = np.array([2**31 - 1, 1, 5], np.int32)
    assert orc.sum_i32(x) == -(2**31) + 5


def test_u32_sum_wraps_and_matches_i32_bits():
    x = np.array([2**32 - 1, 7, 2**31], np.uint32)
    assert orc.sum_u32(x) == (2**32 - 1 + 7 + 2**31) % 2**32
    assert orc.sum_u32(x) == orc.sum_i32(x.view(np.int32)) % 2**32


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32", "f64", "e4m3", "e5m2"])
def test_typed_exact_sum_against_fsum(dtype):
    rng = np.random.default_rng(3)
    if dtype in ("e4m3", "e5m2"):
        x = rng.integers(0, 256, 5000).astype(np.uint8)
        x = x[np.isfinite(orc.decode_to_f32(dtype, x))]
    elif dtype in ("f16", "bf16"):
        x = rng.integers(0, 65536, 5000).astype(np.uint16)
        x = x[np.isfinite(orc.decode_to_f32(dtype, x))]
    else:
        x = (rng.standard_normal(5000) * 1e3).astype(orc.STORAGE[dtype])
    vals = x.astype(np.float64) if dtype == "f64" else (
        x.astype(np.float64) if dtype == "f32" else orc.decode_to_f32(dtype, x).astype(np.float64))
    s, a = orc.sum_typed_exact(dtype, x)
    assert s == math.fsum(vals)
    assert a == pytest.approx(float(np.abs(vals).sum()), rel=1e-12)


def test_fp8_quantize_properties():
    rows, cols = 4, 384
    rng = np.random.default_rng(3)
    x = orc.f32_to_bf16((rng.standard_normal(rows * cols) * 2).astype(np.float32))
    x[5] = orc.f32_to_bf16(np.array([100.0], np.float32))[0]
    codes, scales = orc.fp8_quantize(x, rows, cols)
    xf = orc.bf16_to_f32(x).reshape(rows, cols // 128, 128)
    amax = np.abs(xf).max(axis=2).reshape(-1)
    assert np.array_equal(scales, (amax / np.float32(448.0)).astype(np.float32))
    # the block maximum maps to +-448
    deq = orc.bf16_to_f32(orc.fp8_dequantize(codes, scales, rows, cols)).reshape(rows, cols // 128, 128)
    rel = np.abs(deq - xf).max(axis=2).reshape(-1) / amax
    assert rel.max() <= 2.0 ** -3  # half an E4M3 ulp at the top binade, relative to amax
    zero = np.zeros(128, np.uint16)
    c0, s0 = orc.fp8_quantize(zero, 1, 128)
    assert not c0.any() and s0[0] == 0.0


def test_softmax_and_rmsnorm_definitions():
    rows, cols = 3, 100
    rng = np.random.default_rng(5)
    x = orc.f32_to_bf16(rng.standard_normal(rows * cols).astype(np.float32))
    y = orc.softmax_rows(x, rows, cols)
    assert np.allclose(y.sum(axis=1), 1.0)
    w = orc.f32_to_bf16(np.ones(cols, np.float32))
    r = orc.rmsnorm_rows(x, w, rows, cols, 1e-6)
    assert np.allclose((r ** 2).mean(axis=1), 1.0, rtol=1e-4)


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32", "f64", "e4m3", "e5m2"])
def test_ordered_sum_definition(dtype):
    """The order-fixed sum: close to the exact sum, its total is the fixed
    final tree of its group partials, and whole groups of a shard have the
    same partials as in the full array (what makes multi-GPU results equal)."""
    rng = np.random.default_rng(9)
    eb = np.dtype(orc.STORAGE[dtype]).itemsize
    group = (256 * 1024) // eb
    n = 3 * group + 12345
    if dtype in ("e4m3", "e5m2"):
        x = rng.integers(0, 256, n + n // 4).astype(np.uint8)
        x = x[np.isfinite(orc.decode_to_f32(dtype, x))][:n]
    elif dtype == "f16":
        x = (rng.standard_normal(n) * 100).astype(np.float16).view(np.uint16)
    elif dtype == "bf16":
        x = orc.f32_to_bf16((rng.standard_normal(n) * 100).astype(np.float32))
    else:
        x = rng.standard_normal(n).astype(orc.STORAGE[dtype])
    total, groups = orc.sum_ordered(dtype, x)
    exact, abs_sum = orc.sum_typed_exact(dtype, x)
    assert abs(total - exact) <= 1e-6 * abs_sum
    assert groups.size == 4 and orc.ordered_final(groups) == total
    t2, g2 = orc.sum_ordered(dtype, x[group:])
    assert np.array_equal(g2, groups[1:])
    # trailing zero partials (padding of a short last shard) change nothing
    assert orc.ordered_final(np.concatenate([groups, np.zeros(5)])) == total
    # a misaligned start moves the head elements out of the body
    th, gh = orc.sum_ordered(dtype, x, head=min(3, 16 // eb - 1))
    assert abs(th - exact) <= 1e-6 * abs_sum

