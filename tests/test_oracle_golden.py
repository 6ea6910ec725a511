"""The oracle against the reference's golden vectors and known answers."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


def _conversions():
    raw = (GOLDEN / "conversions.bin").read_bytes()
    n = int(np.frombuffer(raw[:4], np.uint32)[0])
    inputs = np.frombuffer(raw[4:4 + 4 * n], np.uint32)
    e4m3 = np.frombuffer(raw[4 + 4 * n:4 + 5 * n], np.uint8)
    bf16 = np.frombuffer(raw[4 + 5 * n:4 + 7 * n], np.uint16)
    return inputs.view(np.float32), e4m3, bf16


def test_e4m3_encoder_matches_cuda_conversion_golden():
    """Golden codes from __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3),
    the call the reference's codegen emits (CudaCodegen.scala:525-538)."""
    x, codes, _ = _conversions()
    ours = np.array([orc.lib.orc_f32_to_e4m3_satfinite(float(v)) for v in x], np.uint8)
    bad = np.nonzero(ours != codes)[0]
    assert bad.size == 0, [(hex(x.view(np.uint32)[i]), hex(ours[i]), hex(codes[i])) for i in bad[:10]]


def test_bf16_encoder_matches_cuda_conversion_golden():
    """Golden bits from __float2bfloat16_rn (CudaCodegen.scala:518-523)."""
    x, _, bf16 = _conversions()
    ours = np.array([orc.lib.orc_f32_to_bf16_rn(float(v)) for v in x], np.uint16)
    assert np.array_equal(ours, bf16)
    assert np.array_equal(orc._vec_bf16(np.ascontiguousarray(x)), bf16)


def test_exhaustive_conversion_check_recorded_zero_mismatches():
    text = (GOLDEN / "conversions_exhaustive.txt").read_text()
    assert "fp32 patterns checked: 4294967296" in text
    assert "e4m3 satfinite rn mismatches: 0" in text
    assert "bf16 rn mismatches (non-NaN): 0" in text


def test_e4m3_decode_table():
    t = orc.E4M3_TABLE
    assert t[0x00] == 0.0 and t[0x7E] == 448.0 and t[0xFE] == -448.0
    assert t[0x01] == 2.0 ** -9 and t[0x08] == 2.0 ** -6
    assert np.isnan(t[0x7F]) and np.isnan(t[0xFF])
    finite = t[np.isfinite(t)]
    # every finite code round-trips through the encoder
    for c in range(256):
        if np.isfinite(t[c]) and not (c == 0x80):
            assert orc.lib.orc_f32_to_e4m3_satfinite(float(t[c])) == c
    assert finite.size == 254


def _decoder_tables():
    """Every code widened by CUDA's host conversions (__half2float and
    static_cast<float> of the FP8 types, as the reference's ReduceSum widens
    its inputs, CudaCodegen.scala:451-466); NaN canonicalised to 0x7fc00000."""
    import lzma
    raw = np.frombuffer(lzma.decompress((GOLDEN / "decoders.bin.xz").read_bytes()), np.uint32)
    assert raw.size == 256 + 256 + 65536
    return {"e4m3": raw[:256], "e5m2": raw[256:512], "f16": raw[512:]}


def _canonical_bits(f: np.ndarray) -> np.ndarray:
    bits = f.view(np.uint32).copy()
    bits[np.isnan(f)] = 0x7FC00000
    return bits


@pytest.mark.parametrize("dtype,codes", [("e4m3", 256), ("e5m2", 256), ("f16", 65536)])
def test_decoders_match_cuda_conversions_on_every_code(dtype, codes):
    storage = np.uint8 if codes == 256 else np.uint16
    ours = orc.decode_to_f32(dtype, np.arange(codes, dtype=storage))
    golden = _decoder_tables()[dtype]
    bad = np.nonzero(_canonical_bits(ours) != golden)[0]
    assert bad.size == 0, [(hex(c), hex(_canonical_bits(ours)[c]), hex(golden[c])) for c in bad[:10]]


def test_decoder_tables_known_values():
    t = {k: v.view(np.float32) for k, v in _decoder_tables().items()}
    assert t["e5m2"][0x7B] == 57344.0 and t["e5m2"][0x01] == 2.0 ** -16
    assert np.isinf(t["e5m2"][0x7C]) and np.isnan(t["e5m2"][0x7D])
    assert t["f16"][0x3C00] == 1.0 and t["f16"][0x7BFF] == 65504.0 and t["f16"][0x0001] == 2.0 ** -24
    assert np.array_equal(t["e4m3"], orc.E4M3_TABLE, equal_nan=True)


MODED = [("f16", 0), ("f16", 1), ("f16", 2), ("f16", 3), ("bf16", 0), ("bf16", 1), ("bf16", 2), ("bf16", 3),
         ("e4m3", 0), ("e5m2", 0), ("e5m2", 1)]  # (target, rounding for f16/bf16 | saturation for FP8)


def moded_fixture():
    """Inputs and CUDA's outputs of the Convert node's moded conversions
    (__float2half_{rn,rz,ru,rd}, __float2bfloat16_{rn,rz,ru,rd},
    __nv_cvt_float_to_fp8 without / with saturation)."""
    import lzma
    raw = lzma.decompress((GOLDEN / "conversions_modes.bin.xz").read_bytes())
    n = int(np.frombuffer(raw[:4], np.uint32)[0])
    x = np.frombuffer(raw[4:4 + 4 * n], np.uint32).view(np.float32)
    outs, off = [], 4 + 4 * n
    for target, _ in MODED:
        size = 2 if target in ("f16", "bf16") else 1
        outs.append(np.frombuffer(raw[off:off + size * n], np.uint16 if size == 2 else np.uint8))
        off += size * n
    return x, outs


@pytest.mark.parametrize("k", range(len(MODED)))
def test_moded_conversions_match_cuda_golden(k):
    target, mode = MODED[k]
    x, outs = moded_fixture()
    rounding, saturation = (mode, 0) if target in ("f16", "bf16") else (0, mode)
    ours = orc.convert("f32", target, x, rounding, saturation)
    bad = np.nonzero(ours != outs[k])[0]
    assert bad.size == 0, [(hex(x.view(np.uint32)[i]), hex(ours[i]), hex(outs[k][i])) for i in bad[:8]]


def test_exhaustive_moded_check_recorded_zero_mismatches():
    text = (GOLDEN / "conversions_modes_exhaustive.txt").read_text()
    assert "fp32 patterns checked: 4294967296" in text
    lines = [ln for ln in text.splitlines() if "mismatches" in ln]
    assert len(lines) == 11 and all("mismatches (non-NaN): 0; NaN payload differences: 0" in ln for ln in lines)


def test_convert_pairs_and_identity():
    x = np.array([1.5, -2.25, 65504.0, 1e-8], np.float32)
    assert np.array_equal(orc.convert("f32", "f32", x), x)
    assert np.array_equal(orc.convert("f16", "f32", orc.convert("f32", "f16", x)), x[:3].tolist() + [0.0])
    with pytest.raises(ValueError):
        orc.convert("f32", "f64", x)
    with pytest.raises(ValueError):
        orc.convert("f16", "bf16", np.zeros(2, np.uint16))


def test_philox_known_answer_vectors():
    """Random123 Philox4x32-10 known-answer tests."""
    assert orc.philox([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert orc.philox([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert orc.philox([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_uniform_streams_are_shardable():
    whole = orc.uniform_f32(1000, seed=0x5EED)
    parts = np.concatenate([orc.uniform_f32(333, 0x5EED, 0), orc.uniform_f32(667, 0x5EED, 333)])
    assert np.array_equal(whole, parts)
    assert whole.min() >= -1.0 and whole.max() < 1.0
    ints = orc.uniform_i32(10000, 0x5EED, -1000, 1000)
    assert ints.min() >= -1000 and ints.max() <= 1000


def test_reference_known_answers():
    """CudaResourcesJniSuite.scala: vectorAdd (:114-122) and block sum (:235-238, :310)."""
    ka = json.loads((GOLDEN / "reference_known_answers.json").read_text())
    n = ka["vector_add"]["n"]
    a = np.arange(n, dtype=np.float32)
    b = (np.arange(n) * 2).astype(np.float32)
    c = orc.vector_add_f32(a, b)
    assert c[:8].tolist() == ka["vector_add"]["expected_first"]
    assert float(c.astype(np.float64).sum()) == ka["vector_add"]["expected_sum_of_outputs"]
    x = (np.arange(ka["block_reduce_sum"]["n"]) % 8).astype(np.float32)
    assert orc.sum_f32_sequential(x) == ka["block_reduce_sum"]["expected"]
    total, partials = orc.block_tree_sum_f32(x)
    assert total == ka["block_reduce_sum"]["expected"] and partials.tolist() == [896.0]
