"""FP8 E4M3 1x128 block quantize / dequantize: codes, scales and
dequantized values bit-exact vs the oracle, including the full
16384 x 16384 configuration with outliers."""
import numpy as np
import pytest

import flight4s_b200 as f4s
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _roundtrip(ctx, hp, x, rows, cols):
    bpr = (cols + 127) // 128
    dx = ctx.allocate("bf16", x.size)
    dx.copy_from(x)
    dq, dsc, dy = ctx.allocate("u8", x.size), ctx.allocate("f32", rows * bpr), ctx.allocate("bf16", x.size)
    hp.fp8_quantize_e4m3(dx, dq, dsc, rows, cols)
    hp.fp8_dequantize_e4m3(dq, dsc, dy, rows, cols)
    ctx.synchronize()
    return dq.copy_to_array(), dsc.copy_to_array(), dy.copy_to_array()


def _check(ctx, hp, x, rows, cols):
    q, s, y = _roundtrip(ctx, hp, x, rows, cols)
    rq, rs = orc.fp8_quantize(x, rows, cols)
    assert np.array_equal(s.view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(q, rq)
    ry = orc.fp8_dequantize(rq, rs, rows, cols)
    nan = ((ry & 0x7F80) == 0x7F80) & ((ry & 0x7F) != 0)
    assert np.array_equal(y[~nan], ry[~nan])
    assert np.all(((y[nan] & 0x7F80) == 0x7F80) & ((y[nan] & 0x7F) != 0))


@pytest.mark.parametrize("rows,cols", [(1, 128), (4, 256), (3, 200), (2, 1000), (5, 8), (16, 16384), (1, 1)])
def test_bit_exact_vs_oracle(ctx, hp, rows, cols):
    rng = np.random.default_rng(rows * cols)
    v = rng.standard_normal(rows * cols).astype(np.float32) * 2
    out = rng.random(rows * cols) < 1e-2
    v[out] *= 50
    _check(ctx, hp, orc.f32_to_bf16(v), rows, cols)


def test_special_blocks(ctx, hp):
    rows, cols = 8, 128
    v = np.random.default_rng(2).standard_normal(rows * cols).astype(np.float32)
    v[0:128] = 0.0                      # all-zero block -> scale 0, codes 0
    v[128:256] *= 1e-38                 # tiny amax (f32 subnormal range after bf16)
    v[256] = np.inf                     # inf -> amax inf, inv 0
    v[384] = np.nan                     # NaN ignored by amax
    v[512:640] = 448.0                  # exact E4M3 max
    v[640:768] = -1e30                  # huge
    v[768:896] = 2.0 ** -133            # bf16 subnormals: 448/amax clamps to FLT_MAX
    v[896:1024] = np.linspace(-1, 1, 128)
    _check(ctx, hp, orc.f32_to_bf16(v), rows, cols)


def test_full_size_16384x16384_with_outliers(ctx, hp, torch_dev):
    import torch
    rows = cols = 16384
    n = rows * cols
    x = torch.empty(n, dtype=torch.bfloat16, device=torch_dev)
    hp.fill_synthetic(x, n, f4s.NORMAL_BF16_OUTLIERS, seed=0x5EED, p0=0.0, p1=2.0, p2=1e-3, p3=50.0)
    q = torch.empty(n, dtype=torch.uint8, device=torch_dev)
    s = torch.empty(rows * cols // 128, dtype=torch.float32, device=torch_dev)
    y = torch.empty_like(x)
    hp.fp8_quantize_e4m3(x, q, s, rows, cols)
    hp.fp8_dequantize_e4m3(q, s, y, rows, cols)
    torch.cuda.synchronize()
    xh = x.view(torch.int16).cpu().numpy().view(np.uint16)
    rq, rs = orc.fp8_quantize(xh, rows, cols)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), rq)
    ry = orc.fp8_dequantize(rq, rs, rows, cols)
    assert np.array_equal(y.view(torch.int16).cpu().numpy().view(np.uint16), ry)
    # outliers present: ~0.1% of elements at 50x
    assert 5e-4 < float((x.float().abs() > 20).float().mean().item()) < 2e-3
