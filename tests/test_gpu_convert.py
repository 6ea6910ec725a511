"""Elementwise Convert on the GPU (f4s_convert): every pair and mode of the
reference's Convert node bit-exact against the oracle (itself pinned to
CUDA's conversion functions on all 2^32 fp32 patterns), the decodes on every
code, ragged and misaligned buffers, the reference's error for pairs it
cannot emit, and the nearest-even conversions on all 2^32 fp32 patterns
against torch's own conversions of the same device data."""
import numpy as np
import pytest

import flight4s_b200 as f4s
from flight4s_b200 import _native
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

ROUNDINGS = ["nearest_even", "toward_zero", "toward_positive", "toward_negative"]
ENCODES = ([("f16", r, None) for r in ROUNDINGS] + [("bf16", r, None) for r in ROUNDINGS]
           + [(t, "nearest_even", s) for t in ("e4m3", "e5m2") for s in ("none", "finite")])


def _inputs(n_random=200_000):
    """The moded-conversion fixture's inputs (every boundary class, NaN and
    inf) plus random bit patterns."""
    import lzma
    from pathlib import Path
    raw = lzma.decompress((Path(__file__).resolve().parent / "golden" / "conversions_modes.bin.xz").read_bytes())
    n = int(np.frombuffer(raw[:4], np.uint32)[0])
    fixed = np.frombuffer(raw[4:4 + 4 * n], np.uint32)
    rnd = np.random.default_rng(17).integers(0, 2**32, n_random, dtype=np.uint64).astype(np.uint32)
    return np.concatenate([fixed, rnd]).view(np.float32)


def _alloc_dtype(dtype):
    return "u8" if dtype == "bool" else dtype


def _run(ctx, hp, src, dst, x, misalign=0, **modes):
    """Convert x (host array) on the device, `misalign` elements into the
    buffers, with sentinel bytes around the output that must survive."""
    n = x.size
    out_storage = orc.CONVERT_STORAGE[dst]
    ib, ob = x.itemsize, np.dtype(out_storage).itemsize
    total = n + misalign + 3
    din = ctx.allocate(_alloc_dtype(src), total)
    din.copy_from(np.concatenate([np.zeros(misalign, x.dtype), x, np.zeros(3, x.dtype)]))
    sentinel = np.full(total * ob, 0x5A, np.uint8).view(out_storage)
    dout = ctx.allocate(_alloc_dtype(dst), total)
    dout.copy_from(sentinel)
    hp.convert_into(src, dst, din.address + misalign * ib, dout.address + misalign * ob, n=n, **modes)
    ctx.synchronize()
    got = dout.copy_to_array().view(out_storage)
    assert np.array_equal(got[:misalign].view(np.uint8), sentinel[:misalign].view(np.uint8))
    assert np.array_equal(got[misalign + n:].view(np.uint8), sentinel[misalign + n:].view(np.uint8))
    din.close()
    dout.close()
    return got[misalign:misalign + n]


@pytest.mark.parametrize("misalign", [0, 1])
@pytest.mark.parametrize("target,rounding,saturation", ENCODES)
def test_encode_bit_exact_against_oracle(ctx, hp, target, rounding, saturation, misalign):
    x = _inputs()
    got = _run(ctx, hp, "f32", target, x, misalign, rounding=rounding, saturation=saturation)
    want = orc.convert("f32", target, x, f4s.ROUNDING[rounding], f4s.SATURATION[saturation or "none"])
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, [(hex(x.view(np.uint32)[i]), hex(got[i]), hex(want[i])) for i in bad[:8]]


@pytest.mark.parametrize("misalign", [0, 3])
@pytest.mark.parametrize("source", ["f16", "bf16", "e4m3", "e5m2"])
def test_decode_every_code(ctx, hp, source, misalign):
    storage = orc.CONVERT_STORAGE[source]
    codes = np.arange(1 << (8 * np.dtype(storage).itemsize), dtype=storage)
    codes = np.concatenate([codes, codes[::-1], codes[:37]])  # ragged tail
    got = _run(ctx, hp, source, "f32", codes, misalign)
    want = orc.convert(source, "f32", codes)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all(), [(hex(int(codes[i])), got[i], want[i]) for i in np.nonzero(~same)[0][:8]]


@pytest.mark.parametrize("dtype", ["bool", "i32", "u32", "f16", "bf16", "f32", "f64", "e4m3", "e5m2"])
def test_same_type_is_a_copy(ctx, hp, dtype):
    storage = orc.CONVERT_STORAGE[dtype]
    x = np.random.default_rng(3).integers(0, 256, 100_003 * np.dtype(storage).itemsize, dtype=np.uint8)
    x = x.view(storage)
    for misalign in (0, 1):
        assert np.array_equal(_run(ctx, hp, dtype, dtype, x, misalign).view(np.uint8), x.view(np.uint8))


@pytest.mark.parametrize("n", [0, 1, 15, 16, 17, 4095, 4097, 1_000_003])
def test_ragged_lengths(ctx, hp, n):
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32) * 1000
    assert np.array_equal(_run(ctx, hp, "f32", "bf16", x, rounding="toward_zero"),
                          orc.convert("f32", "bf16", x, 1))
    assert np.array_equal(_run(ctx, hp, "f32", "e5m2", x, 1, saturation="none"), orc.convert("f32", "e5m2", x, 0, 0))


def test_reference_errors(ctx, hp):
    d = ctx.allocate("f32", 16)
    codes = f4s.CONVERT_TYPE_CODES
    for src, dst in [("f32", "f64"), ("f16", "bf16"), ("i32", "f32"), ("e4m3", "e5m2"), ("f64", "f32")]:
        rc = _native.lib.f4s_convert(hp.handle, 0, codes[src], codes[dst], 0, 0, d.address, d.address, 4)
        assert rc == _native.STATUS_INVALID_ARGUMENT
    rc = _native.lib.f4s_convert(hp.handle, 0, codes["f32"], codes["f64"], 0, 0, d.address, d.address, 4)
    assert _native.last_status()[2] == "cannot emit a conversion from float to double"
    rc = _native.lib.f4s_convert(hp.handle, 0, codes["f32"], codes["f16"], 4, 0, d.address, d.address, 4)
    assert rc == _native.STATUS_INVALID_ARGUMENT and "rounding mode" in _native.last_status()[2]
    rc = _native.lib.f4s_convert(hp.handle, 0, 10, 10, 0, 0, d.address, d.address, 4)
    assert rc == _native.STATUS_INVALID_ARGUMENT


def test_nearest_even_on_every_fp32_pattern_against_torch(ctx, hp, torch_dev):
    """All 2^32 fp32 bit patterns (in four 2^30 chunks): f32 -> f16 and
    f32 -> bf16 nearest-even equal torch's conversions (NaN to NaN)."""
    import torch
    for lo in (-(1 << 31), -(1 << 30), 0, 1 << 30):
        bits = torch.arange(1 << 30, dtype=torch.int32, device=torch_dev) + lo
        x = bits.view(torch.float32)
        for dst, tdt in (("f16", torch.float16), ("bf16", torch.bfloat16)):
            y = torch.empty(1 << 30, dtype=tdt, device=torch_dev)
            hp.convert_into("f32", dst, x, y)
            torch.cuda.synchronize()
            ref = x.to(tdt)
            same = (y.view(torch.int16) == ref.view(torch.int16)) | (torch.isnan(y) & torch.isnan(ref))
            assert bool(same.all()), (dst, lo, int((~same).sum()))
            del y, ref, same
        del bits, x
        torch.cuda.empty_cache()
