"""include/flight4s_b200_device.cuh on B200: the warp / block / cluster
reductions, compiled by NVRTC as a generated kernel would be, against
restatements of their fixed combine orders (bit-exact), every lane /
thread / CTA checked; exp / rsqrt against CUDA's own expf / rsqrtf."""
from pathlib import Path

import numpy as np
import pytest

from _nvrtc import compile_cubin
from flight4s_b200.runtime import DEVPTR, Block, Cluster, Grid, LaunchConfig
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
KERNELS = Path(__file__).resolve().parent / "device" / "intrinsics_kernels.cu"
F32 = np.float32


@pytest.fixture(scope="module")
def module(ctx):
    return ctx.load(compile_cubin(KERNELS))


def _butterfly(v: np.ndarray, op=np.add) -> np.ndarray:
    """The xor butterfly over offsets 16..1 in the input's precision; every
    lane's value (they are all equal)."""
    s = v.copy()
    lanes = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        s = op(s, s[lanes ^ o]).astype(v.dtype)
    return s


def _run(ctx, module, name, inputs, outputs, grid, block, cluster=None):
    bufs = []
    for a in inputs:
        d = ctx.allocate({np.dtype(F32): "f32", np.dtype(np.float64): "f64", np.dtype(np.int32): "i32",
                          np.dtype(np.int64): "i64"}[a.dtype], a.size)
        d.copy_from(a)
        bufs.append(d)
    outs = [ctx.allocate(kind, n) for kind, n in outputs]
    fn = module.function(name, [DEVPTR] * (len(bufs) + len(outs)))
    cfg = LaunchConfig(Grid(grid), Block(block), cluster=Cluster(cluster) if cluster else None)
    fn.launch(fn.bind(*bufs, *outs), cfg)
    ctx.synchronize()
    return [o.copy_to_array() for o in outs]


def _bits(a):
    return a.view(np.uint32 if a.dtype == F32 else np.uint64)


def test_warp_sums(ctx, module):
    rng = np.random.default_rng(1)
    n = 4 * 128
    x = (rng.standard_normal(n) * 10.0 ** rng.integers(-3, 4, n)).astype(F32)
    (got,) = _run(ctx, module, "warp_sum_f32", [x], [("f32", n)], 4, 128)
    want = np.concatenate([_butterfly(x[w:w + 32]) for w in range(0, n, 32)])
    assert np.array_equal(_bits(got), _bits(want))
    xd = rng.standard_normal(n) * 1e6
    (got,) = _run(ctx, module, "warp_sum_f64", [xd], [("f64", n)], 4, 128)
    want = np.concatenate([_butterfly(xd[w:w + 32]) for w in range(0, n, 32)])
    assert np.array_equal(_bits(got), _bits(want))
    xi = rng.integers(-2**31, 2**31, n, dtype=np.int64).astype(np.int32)
    (got,) = _run(ctx, module, "warp_sum_i32", [xi], [("i32", n)], 4, 128)
    sums = [orc.sum_i32(xi[w:w + 32]) for w in range(0, n, 32)]
    assert got.tolist() == [s for s in sums for _ in range(32)]


def test_warp_max_ignores_nan(ctx, module):
    rng = np.random.default_rng(2)
    x = rng.standard_normal(256).astype(F32)
    x[5] = np.nan
    x[40:72] = np.nan  # a whole warp of NaN: the max is NaN
    (got,) = _run(ctx, module, "warp_max_f32", [x], [("f32", 256)], 2, 128)
    for w in range(0, 256, 32):
        seg = x[w:w + 32]
        want = np.nan if np.isnan(seg).all() else np.nanmax(seg)
        assert np.allclose(got[w:w + 32], want, equal_nan=True), w


@pytest.mark.parametrize("few", [False, True])
def test_warp_argmax(ctx, module, few):
    rng = np.random.default_rng(3 + few)
    n = 8 * 32
    x = (rng.integers(-3, 4, n) if few else rng.standard_normal(n)).astype(F32)
    x[7], x[33], x[70] = -0.0, np.inf, np.nan
    index = np.arange(n, dtype=np.int64) * 3 + 100
    index[64:96] = -1            # an empty warp
    index[[1, 2, 130]] = -1      # empty lanes
    got_v, got_i = _run(ctx, module, "warp_argmax_f32", [x, index], [("f32", n), ("i64", n)], 2, 128)
    for w in range(0, n, 32):
        live = index[w:w + 32] >= 0
        if not live.any():
            assert (got_i[w:w + 32] == -1).all()
            continue
        v, j = orc.argmax_f32(np.ascontiguousarray(x[w:w + 32][live]))
        assert (got_i[w:w + 32] == index[w:w + 32][live][j]).all(), w
        assert (_bits(got_v[w:w + 32]) == np.array([v], F32).view(np.uint32)[0]).all(), w


@pytest.mark.parametrize("block", [96, 256, 1024])
def test_block_sum(ctx, module, block):
    rng = np.random.default_rng(block)
    grid = 3
    n = grid * block
    x = (rng.standard_normal(n) * 10.0 ** rng.integers(-2, 3, n)).astype(F32)
    (got,) = _run(ctx, module, "block_sum_f32", [x], [("f32", n)], grid, block)
    for b in range(grid):
        seg = x[b * block:(b + 1) * block]
        slots = np.zeros(32, F32)
        for w in range(block // 32):
            slots[w] = _butterfly(seg[w * 32:(w + 1) * 32])[0]
        want = _butterfly(slots)[0]
        assert np.array_equal(_bits(got[b * block:(b + 1) * block]), np.full(block, np.array([want]).view(np.uint32)[0]))


@pytest.mark.parametrize("block", [128, 512])
def test_block_argmax(ctx, module, block):
    rng = np.random.default_rng(block + 1)
    n = 2 * block
    x = rng.integers(-5, 6, n).astype(F32)  # many ties: the lowest index must win
    got_v, got_i = _run(ctx, module, "block_argmax_f32", [x], [("f32", n), ("i64", n)], 2, block)
    for b in range(2):
        v, j = orc.argmax_f32(np.ascontiguousarray(x[b * block:(b + 1) * block]))
        assert (got_i[b * block:(b + 1) * block] == b * block + j).all()
        assert (got_v[b * block:(b + 1) * block] == v).all()


@pytest.mark.parametrize("cluster", [2, 4, 8])
def test_cluster_sum(ctx, module, cluster):
    rng = np.random.default_rng(cluster)
    block, clusters = 128, 3
    n = block * cluster * clusters
    x = (rng.standard_normal(n) * 10.0 ** rng.integers(-2, 3, n)).astype(F32)
    (got,) = _run(ctx, module, "cluster_sum_f32", [x], [("f32", n)], cluster * clusters, block, cluster)
    for c in range(clusters):
        total = F32(0.0)
        for r in range(cluster):
            b = c * cluster + r
            seg = x[b * block:(b + 1) * block]
            slots = np.zeros(32, F32)
            for w in range(block // 32):
                slots[w] = _butterfly(seg[w * 32:(w + 1) * 32])[0]
            total = F32(total + _butterfly(slots)[0])
        part = got[c * cluster * block:(c + 1) * cluster * block]
        assert np.array_equal(_bits(part), np.full(part.size, np.array([total], F32).view(np.uint32)[0])), c


def test_math_matches_cuda(ctx, module):
    rng = np.random.default_rng(9)
    x = np.concatenate([rng.uniform(-80, 80, 1000), rng.uniform(1e-30, 1e30, 1000)]).astype(F32)
    e, r = _run(ctx, module, "math_f32", [x], [("f32", x.size), ("f32", x.size)], x.size // 250, 250)
    ce, cr = _run(ctx, module, "math_f32_cuda", [x], [("f32", x.size), ("f32", x.size)], x.size // 250, 250)
    assert np.array_equal(_bits(e), _bits(ce)) and np.array_equal(_bits(r), _bits(cr))
    with np.errstate(over="ignore"):
        assert np.allclose(e[:1000], np.exp(x[:1000].astype(np.float64)), rtol=1e-6)
    assert np.allclose(r[1000:], 1 / np.sqrt(x[1000:].astype(np.float64)), rtol=1e-6)
