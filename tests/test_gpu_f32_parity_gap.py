"""How far the f32 ReduceSum here is from what the reference would return.

The reference accumulates an F32 ReduceSum in F32
(core/src/main/scala/flight4s/core/types/CudaType.scala:216-218), lowered to
a serial loop, and its own check is Scala's Array[Float].sum, a sequential
Float fold (runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala:235-238).
The kernels here return the sum accumulated in f64.  On the same seeded
N(0,1) data this test states, relative to sum|x|:
  * the f64 result's distance from the exact sum (tiny),
  * that result rounded to f32: the f32 nearest the exact sum,
  * the reference-style Float fold's distance from the exact sum, within
    its classic bound (n - 1) * 2^-24 * sum|x|,
so a drop-in caller knows what to expect: an f64 whose f32 rounding is the
correctly rounded sum, differing from the reference's Float fold by that
fold's own rounding error.
"""
import numpy as np
import pytest

import flight4s_b200 as f4s
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

SEED = 0x5EED


def _ulp32(v: float) -> float:
    f = np.float32(v)
    return float(np.spacing(np.abs(f)))


@pytest.mark.parametrize("log2n", [20, 24, 28])
def test_f32_sum_against_the_reference_float_fold(ctx, hp, log2n):
    n = 1 << log2n
    dx = ctx.allocate("f32", n)
    hp.fill_synthetic(dx, n, f4s.NORMAL_F32, seed=SEED)
    x = dx.copy_to_array()
    ours = hp.reduce_sum_f32(dx)
    exact, abs_sum = orc.sum_f32_exact(x)
    fold = orc.sum_f32_sequential(x)
    rounded = float(np.float32(ours))
    # the f64 result: each element passes through at most four f32 additions
    # (pairs, then the tree over a step's four 16-byte vectors) before f64
    # takes over, so the error is at most 4 * 2^-24 * sum|x| (plus f64's own,
    # far smaller); far inside the 1e-5 of sum|x| the f32 sums are held to
    assert abs(ours - exact) <= (4 * 2.0 ** -24 + 1e-12) * abs_sum
    # rounded to the reference's Float: the f32 nearest the exact sum
    assert abs(rounded - exact) <= 0.5 * max(_ulp32(exact), _ulp32(ours)) + abs(ours - exact)
    # the reference's fold: within the textbook bound of a recursive sum
    assert abs(fold - exact) <= (n - 1) * 2.0 ** -24 * abs_sum
    # and no closer to the exact sum than the correctly rounded value
    assert abs(fold - exact) >= abs(rounded - exact) - 2 * abs(ours - exact)
    print(f"n=2^{log2n}: |ours-exact|/S={abs(ours - exact) / abs_sum:.3e} "
          f"|f32(ours)-exact|/S={abs(rounded - exact) / abs_sum:.3e} "
          f"|fold-exact|/S={abs(fold - exact) / abs_sum:.3e} "
          f"|f32(ours)-fold|/S={abs(rounded - fold) / abs_sum:.3e} (S=sum|x|={abs_sum:.6e}, exact={exact:.9e})")
    dx.close()
