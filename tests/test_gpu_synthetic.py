"""Device Philox generator: bit-exact vs the oracle for uniform streams,
shard-consistent, and statistically sane for the normal streams."""
import numpy as np
import pytest

import flight4s_b200 as f4s
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,offset", [(1, 0), (5, 3), (1000, 0), (100_003, 17), (1 << 20, 1 << 33)])
def test_uniform_bit_exact(ctx, hp, n, offset):
    d = ctx.allocate("f32", n)
    hp.fill_synthetic(d, n, f4s.UNIFORM_F32, seed=0x5EED, offset=offset)
    di = ctx.allocate("i32", n)
    hp.fill_synthetic(di, n, f4s.UNIFORM_I32, seed=0x5EED, offset=offset, ilo=-1000, ihi=1000)
    ctx.synchronize()
    assert np.array_equal(d.copy_to_array(), orc.uniform_f32(n, 0x5EED, offset))
    assert np.array_equal(di.copy_to_array(), orc.uniform_i32(n, 0x5EED, -1000, 1000, offset))


def test_normal_statistics_and_sharding(ctx, hp):
    n = 1 << 22
    d = ctx.allocate("f32", n)
    hp.fill_synthetic(d, n, f4s.NORMAL_F32, seed=7)
    a = ctx.allocate("f32", n // 2)
    b = ctx.allocate("f32", n // 2)
    hp.fill_synthetic(a, n // 2, f4s.NORMAL_F32, seed=7)
    hp.fill_synthetic(b, n // 2, f4s.NORMAL_F32, seed=7, offset=n // 2)
    ctx.synchronize()
    x = d.copy_to_array()
    assert np.array_equal(np.concatenate([a.copy_to_array(), b.copy_to_array()]), x)
    assert abs(x.mean()) < 5e-3 and abs(x.std() - 1) < 5e-3
    db = ctx.allocate("bf16", n)
    hp.fill_synthetic(db, n, f4s.NORMAL_BF16_OUTLIERS, seed=7, p1=2.0, p2=1e-3, p3=50.0)
    ctx.synchronize()
    xb = orc.bf16_to_f32(db.copy_to_array())
    assert 5e-4 < np.mean(np.abs(xb) > 20) < 2e-3


def test_rejects_bad_parameters(ctx, hp):
    d = ctx.allocate("i32", 16)
    with pytest.raises(ValueError):
        hp.fill_synthetic(d, 16, f4s.UNIFORM_I32, seed=1, ilo=5, ihi=4)
    with pytest.raises(ValueError):
        hp.fill_synthetic(d, 16, 99, seed=1)
