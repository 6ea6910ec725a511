"""Row-wise softmax and RMSNorm (bf16 in/out, f32 math) vs the oracle's f64
definitions, within the bf16 tolerance; at the benchmark shape every row vs
a torch fp32 reference and a spread of 257 rows vs the oracle."""
import numpy as np
import pytest

import flight4s_b200 as f4s
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

RTOL, ATOL_SOFTMAX, ATOL_RMS = 1e-2, 1e-6, 1e-2  # bf16 output tolerance
SHAPES = [(1, 8), (3, 100), (2, 24), (4, 2048), (5, 2056), (3, 8192), (2, 16384), (2, 16392), (7, 1000), (33, 512)]


def _bf16(ctx, values):
    buf = ctx.allocate("bf16", values.size)
    buf.copy_from(values)
    return buf


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_softmax_vs_oracle(ctx, hp, rows, cols):
    x = orc.f32_to_bf16((np.random.default_rng(cols).standard_normal(rows * cols) * 3).astype(np.float32))
    dx, dy = _bf16(ctx, x), ctx.allocate("bf16", x.size)
    hp.softmax_rows_bf16(dx, dy, rows, cols)
    ctx.synchronize()
    y = orc.bf16_to_f32(dy.copy_to_array()).reshape(rows, cols)
    ref = orc.softmax_rows(x, rows, cols)
    assert np.allclose(y, ref, rtol=RTOL, atol=ATOL_SOFTMAX)
    assert np.allclose(y.astype(np.float64).sum(axis=1), 1.0, atol=1e-2)


def test_softmax_extremes(ctx, hp):
    rows, cols = 4, 2048
    x = np.zeros(rows * cols, np.float32)
    x[:cols] = -1e30       # all very negative: uniform
    x[cols + 3] = 80.0     # one dominant element
    x[2 * cols:3 * cols] = 5.0  # constant row
    x[3 * cols:] = np.linspace(-100, 100, cols)
    xb = orc.f32_to_bf16(x)
    dx, dy = _bf16(ctx, xb), ctx.allocate("bf16", xb.size)
    hp.softmax_rows_bf16(dx, dy, rows, cols)
    ctx.synchronize()
    y = orc.bf16_to_f32(dy.copy_to_array()).reshape(rows, cols)
    assert np.all(np.isfinite(y))
    assert np.allclose(y, orc.softmax_rows(xb, rows, cols), rtol=RTOL, atol=ATOL_SOFTMAX)


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_rmsnorm_vs_oracle(ctx, hp, rows, cols):
    rng = np.random.default_rng(cols + 1)
    x = orc.f32_to_bf16(rng.standard_normal(rows * cols).astype(np.float32))
    w = orc.f32_to_bf16((1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32))
    dx, dw, dy = _bf16(ctx, x), _bf16(ctx, w), ctx.allocate("bf16", x.size)
    hp.rmsnorm_rows_bf16(dx, dw, dy, rows, cols, eps=1e-6)
    ctx.synchronize()
    y = orc.bf16_to_f32(dy.copy_to_array()).reshape(rows, cols)
    assert np.allclose(y, orc.rmsnorm_rows(x, w, rows, cols, 1e-6), rtol=RTOL, atol=ATOL_RMS)


def test_rmsnorm_zero_rows_use_eps(ctx, hp):
    rows, cols = 2, 4096
    x = np.zeros(rows * cols, np.uint16)
    w = orc.f32_to_bf16(np.ones(cols, np.float32))
    dx, dw, dy = _bf16(ctx, x), _bf16(ctx, w), ctx.allocate("bf16", x.size)
    hp.rmsnorm_rows_bf16(dx, dw, dy, rows, cols, eps=1e-6)
    ctx.synchronize()
    assert not dy.copy_to_array().any()


def test_row_ops_reject_bad_arguments(ctx, hp):
    dx = ctx.allocate("bf16", 16)
    with pytest.raises(ValueError, match="negative"):
        hp.softmax_rows_bf16(dx, dx, -1, 16)
    with pytest.raises(ValueError, match="eps"):
        hp.rmsnorm_rows_bf16(dx, dx, dx, 1, 16, eps=float("nan"))


def test_full_size_32768x8192_against_torch_fp32(ctx, hp, torch_dev):
    import torch
    rows, cols = 32768, 8192
    x = torch.empty(rows * cols, dtype=torch.bfloat16, device=torch_dev)
    hp.fill_synthetic(x, x.numel(), f4s.NORMAL_BF16, seed=0x5EED)
    w = torch.empty(cols, dtype=torch.bfloat16, device=torch_dev)
    hp.fill_synthetic(w, cols, f4s.NORMAL_BF16, seed=0x5EED + 1, p0=1.0, p1=0.1)
    y = torch.empty_like(x)
    hp.softmax_rows_bf16(x, y, rows, cols)
    torch.cuda.synchronize()
    ref = torch.softmax(x.view(rows, cols).float(), dim=1)
    err = ((y.view(rows, cols).float() - ref).abs() - RTOL * ref.abs()).max().item()
    assert err <= ATOL_SOFTMAX
    del ref
    hp.rmsnorm_rows_bf16(x, w, y, rows, cols, eps=1e-6)
    torch.cuda.synchronize()
    xf = x.view(rows, cols).float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(dim=1, keepdim=True) + 1e-6) * w.float()
    err = ((y.view(rows, cols).float() - ref).abs() - RTOL * ref.abs()).max().item()
    assert err <= ATOL_RMS
    del x, y, ref, xf
    torch.cuda.empty_cache()


@pytest.mark.parametrize("rows,cols", [(1, 8192), (3, 2056 * 2), (300, 4104), (1000, 8192), (5000, 6144)])
def test_rmsnorm_tma_staged_matches_register_kernel_bitwise(ctx, hp, rows, cols):
    """Rows of 2049..8192 go through the TMA-staged kernel; it must equal the
    register-resident kernel bit for bit, and no staged wait may give up."""
    rng = np.random.default_rng(rows + cols)
    x = orc.f32_to_bf16(rng.standard_normal(rows * cols).astype(np.float32))
    w = orc.f32_to_bf16((1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32))
    dx, dw, dy, dr = _bf16(ctx, x), _bf16(ctx, w), ctx.allocate("bf16", x.size), ctx.allocate("bf16", x.size)
    hp.wait_timeouts(reset=True)
    hp.rmsnorm_rows_bf16(dx, dw, dy, rows, cols, eps=1e-6)
    fn = hp.module.function("f4s_rmsnorm_rows_bf16_v4",
                            signature=[f4s.DEVPTR, f4s.DEVPTR, f4s.DEVPTR, f4s.INT32, f4s.INT32, f4s.FLOAT32])
    fn.launch(fn.bind(dx, dw, dr, rows, cols, 1e-6), f4s.LaunchConfig(f4s.Grid(min(rows, 296)), f4s.Block(256)))
    ctx.synchronize()
    assert hp.wait_timeouts() == 0
    assert np.array_equal(dy.copy_to_array(), dr.copy_to_array())
    y = orc.bf16_to_f32(dy.copy_to_array()).reshape(rows, cols)
    assert np.allclose(y, orc.rmsnorm_rows(x, w, rows, cols, 1e-6), rtol=RTOL, atol=ATOL_RMS)


def test_benchmark_shape_rows_against_the_oracle(ctx, hp, torch_dev):
    """At the benchmark shape itself (32768 x 8192, device-seeded N(0,1)
    inputs, weight N(1, 0.1)), 257 rows spread over the whole array (the
    first, the last and every 128th) meet the oracle's f64 softmax and
    RMSNorm within the bf16 tolerance."""
    import torch
    rows, cols = 32768, 8192
    x = torch.empty(rows * cols, dtype=torch.bfloat16, device=torch_dev)
    hp.fill_synthetic(x, x.numel(), f4s.NORMAL_BF16, seed=0x5EED)
    w = torch.empty(cols, dtype=torch.bfloat16, device=torch_dev)
    hp.fill_synthetic(w, cols, f4s.NORMAL_BF16, seed=0x5EED + 1, p0=1.0, p1=0.1)
    y = torch.empty_like(x)
    pick = torch.tensor(sorted(set(range(0, rows, 128)) | {rows - 1}), device=torch_dev)
    k = pick.numel()

    def bits(t):
        return t.view(rows, cols).index_select(0, pick).contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

    xs = bits(x).reshape(-1)
    hp.softmax_rows_bf16(x, y, rows, cols)
    torch.cuda.synchronize()
    got = orc.bf16_to_f32(bits(y).reshape(-1)).reshape(k, cols)
    assert np.allclose(got, orc.softmax_rows(xs, k, cols), rtol=RTOL, atol=ATOL_SOFTMAX)
    hp.rmsnorm_rows_bf16(x, w, y, rows, cols, eps=1e-6)
    torch.cuda.synchronize()
    got = orc.bf16_to_f32(bits(y).reshape(-1)).reshape(k, cols)
    wb = w.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.allclose(got, orc.rmsnorm_rows(xs, wb, k, cols, 1e-6), rtol=RTOL, atol=ATOL_RMS)
    del x, y
    torch.cuda.empty_cache()
