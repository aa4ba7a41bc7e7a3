"""The oracle against the reference's own known answers (no GPU)."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def kat_cases():
    return json.loads((GOLDEN / "mxfp4_kat.json").read_text())["cases"]


@pytest.mark.parametrize("case", kat_cases(), ids=lambda c: c["name"])
def test_quantiser_matches_swift_known_answers(case):
    """MXFP4.swift quantiser restatement reproduces DeepSeekRepackTests.swift:336-415."""
    if case["kind"] == "bf16":
        src = np.array(case["source_bf16"], np.uint16).reshape(case["rows"], case["cols"])
        w, s = oracle.quantize_bf16_mxfp4(src)
    else:
        src = np.array(case["source_u8"], np.uint8).reshape(case["rows"], case["cols"])
        inv = np.array(case["inverse_scale_bytes"], np.uint8).view(np.uint16)
        w, s = oracle.quantize_fp8_mxfp4(src, inv)
    if "expect" in case:
        for e in case["expect"]:
            got = (w if e["field"] == "weights" else s).reshape(-1)[: len(e["bytes"])]
            assert got.tolist() == e["bytes"], e["field"]
    else:
        assert hashlib.sha256(w.tobytes()).hexdigest() == case["expect_sha256"]["weights"]
        assert hashlib.sha256(s.tobytes()).hexdigest() == case["expect_sha256"]["scales"]


def test_e2m1_table_and_conventions():
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    for code in range(16):
        v = oracle.e2m1(code, oracle.CONV_MLX)
        expect = (-1.0 if code & 8 else 1.0) * mags[code & 7]
        assert v == expect
    assert np.signbit(oracle.e2m1(8, oracle.CONV_METAL)) and not np.signbit(oracle.e2m1(8, oracle.CONV_MLX))


def test_e8m0_conventions():
    for b in range(1, 255):
        assert oracle.e8m0(b, oracle.CONV_MLX) == 2.0 ** (b - 127) == oracle.e8m0(b, oracle.CONV_METAL)
    assert oracle.e8m0(0, oracle.CONV_MLX) == np.float32(2.0 ** -127)
    assert oracle.e8m0(0, oracle.CONV_METAL) == 0.0
    assert np.isinf(oracle.e8m0(255, oracle.CONV_MLX))


def test_e4m3_matches_torch_float8_for_every_code():
    codes = torch.arange(256, dtype=torch.uint8)
    ref = codes.view(torch.float8_e4m3fn).float().numpy()
    for b in range(256):
        v = oracle.e4m3(b)
        if np.isnan(ref[b]):
            assert np.isnan(v)
        else:
            assert v == ref[b], b


def test_dequant_mxfp4_matches_product_definition():
    rng = np.random.default_rng(1)
    w = rng.integers(0, 256, (7, 64), dtype=np.uint8)
    s = rng.integers(100, 150, (7, 4), dtype=np.uint8)
    out = oracle.bf16_to_f32(oracle.dequant_mxfp4(w, s))
    lo, hi = w & 15, w >> 4
    codes = np.stack([lo, hi], -1).reshape(7, 128)
    mags = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float32)
    vals = np.where(codes & 8, -1, 1) * mags[codes & 7] * np.exp2(s.astype(np.float32) - 127).repeat(32, 1)
    np.testing.assert_array_equal(out, vals.astype(np.float32))


def test_quantise_then_dequantise_is_a_fixed_point():
    """Requantising dequantised MXFP4 values reproduces the same bytes."""
    rng = np.random.default_rng(2)
    w = rng.integers(0, 256, (16, 64), dtype=np.uint8)
    s = rng.integers(110, 140, (16, 4), dtype=np.uint8)
    # groups whose largest magnitude code is 6.0 keep their scale exactly
    w[:, ::16] = (w[:, ::16] & 0xF0) | 0x07
    deq = oracle.dequant_mxfp4(w, s)
    w2, s2 = oracle.quantize_bf16_mxfp4(deq)
    np.testing.assert_array_equal(oracle.dequant_mxfp4(w2, s2), deq)
    np.testing.assert_array_equal(s2, s)


def test_fp8_block_decode_rejects_reserved_codes_and_rounds_once():
    w = np.full((128, 128), 0x38, np.uint8)  # 1.0
    s = np.array([[0.1]], np.float32)
    out = oracle.bf16_to_f32(oracle.dequant_fp8_b128(w, s))
    assert out[0, 0] == oracle.bf16_to_f32(oracle.f32_to_bf16(np.float32(0.1)))
    w[3, 5] = 0x7F
    with pytest.raises(ValueError):
        oracle.dequant_fp8_b128(w, s)


def test_rms_norm_matches_the_reference_known_answer():
    """[3, 4] normalises to [3, 4] / sqrt(12.5 + 1e-6) (the RMS part of
    test_gated_delta_norm_uses_sigmoid, runtime/tests/test_qwen.py:715-727),
    then multiplies by the weight (rms_norm_tg, kernels.metal:443-465)."""
    x = oracle.f32_to_bf16(np.array([[3.0, 4.0]], np.float32))
    one = oracle.f32_to_bf16(np.ones(2, np.float32))
    expected = np.array([[3.0, 4.0]], np.float64) / np.sqrt(12.5 + 1e-6)
    got = oracle.bf16_to_f32(oracle.rms_norm(x, one, 1e-6))
    np.testing.assert_array_equal(got, oracle.bf16_to_f32(oracle.f32_to_bf16(expected.astype(np.float32))))
    w = oracle.f32_to_bf16(np.array([0.5, -2.0], np.float32))
    got = oracle.bf16_to_f32(oracle.rms_norm(x, w, 1e-6))
    np.testing.assert_allclose(got, expected * [0.5, -2.0], rtol=2 ** -8)


def test_rms_norm_is_scale_invariant_and_follows_eps():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((4, 256)).astype(np.float32)
    w = oracle.f32_to_bf16(rng.standard_normal(256).astype(np.float32))
    a = oracle.rms_norm(oracle.f32_to_bf16(x), w, 0.0)
    b = oracle.rms_norm(oracle.f32_to_bf16(x * 4.0), w, 0.0)  # powers of two scale bf16 exactly
    np.testing.assert_array_equal(a, b)
    zero = np.zeros((1, 256), np.uint16)
    assert not oracle.bf16_to_f32(oracle.rms_norm(zero, w, 1e-6)).any()  # zero rows stay zero (signed)


def test_fp8_b32_layer_weights_are_the_dequantised_blocks():
    """The layer restatement of the FP8 32x32 layout multiplies by exactly the
    weights dequant.py:45-50 produces (wmo_dequant_fp8_b32)."""
    rng = np.random.default_rng(7)
    O, I = 96, 128
    codes = rng.integers(0, 254, (O, I))
    w = np.where(codes < 127, codes, codes + 1).astype(np.uint8)
    s = (127 + rng.integers(-10, -3, (O // 32, I // 32))).astype(np.uint8)
    x = oracle.f32_to_bf16(rng.standard_normal((3, I)).astype(np.float32))
    y = oracle.linear(oracle.LAYOUT_W13_FP8_B32, w, s, x)
    deq = oracle.bf16_to_f32(oracle.dequant_fp8_b32(w, s)).astype(np.float64)
    want = oracle.bf16_to_f32(x).astype(np.float64) @ deq.T
    np.testing.assert_allclose(y, want, rtol=1e-6, atol=1e-6)
