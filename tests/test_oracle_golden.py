"""Pins the CPU oracle against the known-answer vectors of the reference's own
tests (tests/golden/golden.json).  CPU only."""

import math

import numpy as np
import pytest


def _hex(h, dtype):
    return np.frombuffer(bytes.fromhex(h), dtype=dtype).copy()


def test_q4k_gemv_kats(golden, orc):
    # src/metal_ops.rs:1154-1235: rel < 1e-3 against dequantize + f32 dot.
    for case in golden["q4k_gemv"]:
        blocks = _hex(case["blocks_hex"], np.uint8)
        x = np.array(case["x"], dtype=np.float32)
        y = orc.q4k_gemv(blocks, case["rows"], case["cols"], x)
        exp = np.array(case["expected"], dtype=np.float32)
        rel = np.abs(y - exp) / (np.abs(exp) + 1e-6)
        assert rel.max() < case["rel_tol"], (case["name"], rel.max())


def test_q4k_dequant_matches_gemv_order(golden, orc):
    # dot_row's factorised sum and dequantize+dot agree closely on the KAT block.
    case = golden["q4k_gemv"][1]
    blocks = _hex(case["blocks_hex"], np.uint8)
    w = orc.q4k_dequantize(blocks, case["rows"], case["cols"])
    x = np.array(case["x"], dtype=np.float32)
    np.testing.assert_allclose(orc.q4k_gemv(blocks, case["rows"], case["cols"], x), w @ x, rtol=1e-5, atol=1e-5)


def test_bf16_gemv_kats(golden, orc):
    # src/metal_ops.rs:1239-1305: |diff| < 1e-2.
    for case in golden["bf16_gemv"]:
        w = _hex(case["w_hex"], np.uint16)
        x = np.array(case["x"], dtype=np.float32)
        y = orc.bf16_gemv(w, case["rows"], case["cols"], x)
        exp = np.array(case["expected"], dtype=np.float32)
        # same sequential order as the restatement: bit-identical
        np.testing.assert_array_equal(y, exp)


def test_rms_norm_kat(golden, orc):
    c = golden["rms_norm"]
    y = orc.rms_norm_gemma3(np.array(c["x"], np.float32), np.array(c["gamma"], np.float32), c["eps"])
    assert np.abs(y - np.array(c["expected"])).max() < c["abs_tol"]


def test_per_head_norm_kat(golden, orc):
    c = golden["per_head_norm"]
    y = orc.per_head_norm(np.array(c["x"], np.float32), np.array(c["gamma"], np.float32), c["n_heads"],
                          c["head_dim"], c["eps"])
    assert np.abs(y - np.array(c["expected"])).max() < c["abs_tol"]


def test_rope_kat(golden, orc):
    c = golden["rope"]
    y = orc.rope(np.array(c["x"], np.float32), c["n_heads"], c["head_dim"], c["theta"], c["pos"], c["freq_scale"])
    assert np.abs(y - np.array(c["expected"])).max() < c["abs_tol"]


def test_gelu_kat(golden, orc):
    c = golden["gelu"]
    y = orc.gelu_tanh(np.array(c["x"], np.float32))
    assert np.all(np.isfinite(y))
    assert np.abs(y - np.array(c["expected"])).max() < c["abs_tol"] * max(1.0, 1.0)


def test_attention_kat(golden, orc):
    c = golden["attention"]
    y = orc.gqa_attention_decode(np.array(c["q"], np.float32), np.array(c["k_cache"], np.float32),
                                 np.array(c["v_cache"], np.float32), c["k_start"], c["k_end"], c["n_q_heads"],
                                 c["n_kv_heads"], c["head_dim"], c["scale"])
    assert np.abs(y - np.array(c["expected"])).max() < c["abs_tol"]


def test_q4k_quantize_bytes_and_roundtrip(golden, orc):
    # src/autograd2.rs:5658-5729 (max abs error < 0.15) and byte equality with
    # the independent restatement in make_golden.py.
    for case in golden["q4k_quantize"]:
        m = np.array(case["input"], np.float32).reshape(case["rows"], case["cols"])
        blocks = orc.q4k_quantize(m)
        assert blocks.tobytes().hex() == case["blocks_hex"], case["name"]
        back = orc.q4k_dequantize(blocks, case["rows"], case["cols"])
        assert np.abs(back - m).max() < case["max_err_bound"]
        assert math.isclose(float(np.abs(back - m).max()), case["max_err"], rel_tol=0, abs_tol=0)


def test_f16_truncating_conversion(golden, orc):
    c = golden["f16"]
    for v, bits, back in zip(c["values"], c["bits"], c["back"]):
        assert orc.lib.or_f32_to_f16(v) == bits, v
        assert orc.lib.or_f16_to_f32(bits) == back or (math.isinf(back) and math.isinf(orc.lib.or_f16_to_f32(bits)))
    # src/autograd2.rs:5732-5746 round-trip tolerance on its own values
    for v in [0.0, 1.0, -1.0, 0.5, 65504.0, -65504.0, 0.001, 100.0]:
        back = orc.lib.or_f16_to_f32(orc.lib.or_f32_to_f16(v))
        assert abs(back - v) < abs(v) * 0.002 + 1e-6


def test_bf16_conversion(golden, orc):
    c = golden["bf16"]
    for v, bits in zip(c["values"], c["bits"]):
        assert orc.lib.or_f32_to_bf16(float(v)) == bits, v
    assert orc.lib.or_bf16_to_f32(orc.lib.or_f32_to_bf16(float("inf"))) == float("inf")
    assert orc.lib.or_bf16_to_f32(orc.lib.or_f32_to_bf16(float("-inf"))) == float("-inf")


def test_q6k_decode(golden, orc):
    c = golden["q6k"]
    data = _hex(c["bytes_hex"], np.uint8)
    f = orc.q6k_to_f32(data, c["n_elem"])
    np.testing.assert_array_equal(f, np.array(c["f32"], np.float32))
    b = orc.q6k_to_bf16(data, c["n_elem"])
    np.testing.assert_array_equal(b, np.array(c["bf16"], np.uint16))


def test_q4_0_to_q4k(golden, orc):
    c = golden["q4_0_to_q4k"]
    out = orc.q4_0_to_q4k(_hex(c["q4_0_hex"], np.uint8), c["rows"], c["cols"])
    assert out.tobytes().hex() == c["q4k_hex"]


def test_sample_greedy_last_max_wins(orc):
    # Iterator::max_by keeps the last of equal maxima (src/transformer4.rs:3084-3091).
    assert orc.sample_greedy(np.array([0.0, 3.0, 1.0, 3.0, 2.0], np.float32)) == 3
    assert orc.sample_greedy(np.array([5.0, 1.0], np.float32)) == 0


def test_gemv_thread_count_invariance(orc):
    rng = np.random.default_rng(3)
    blocks = rng.integers(0, 256, size=300 * 2 * 144, dtype=np.uint8)
    blocks.reshape(-1, 144)[:, 1] &= 0x1F  # keep d finite and small
    blocks.reshape(-1, 144)[:, 3] &= 0x1F
    x = rng.standard_normal(512).astype(np.float32)
    y1 = orc.q4k_gemv(blocks, 300, 512, x, nthreads=1)
    y8 = orc.q4k_gemv(blocks, 300, 512, x, nthreads=8)
    np.testing.assert_array_equal(y1, y8)
