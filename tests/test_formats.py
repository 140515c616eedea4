"""GGUF block formats pinned against gguf-py fixtures (tests/golden/formats.npz).

gguf-py is what the reference converter quantizes with
(models/convert-bert-to-gguf.py:68-77); these pins hold for the numpy encoders in
crispembed_b200.quant, the C oracle's dequantizers and the library's repack.
"""
import os

import numpy as np
import pytest

from crispembed_b200 import quant

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "formats.npz"))


def test_q8_0_encoder_matches_gguf_py_bytes():
    assert np.array_equal(quant.quantize_q8_0(GOLD["q8_x"]), GOLD["q8_blocks"])


def test_q8_0_decoders_match_gguf_py(oracle):
    k = GOLD["q8_x"].shape[1]
    assert np.array_equal(quant.dequantize_q8_0(GOLD["q8_blocks"], k), GOLD["q8_deq"])
    assert np.array_equal(oracle.dequant(oracle.T_Q8_0, GOLD["q8_blocks"], k), GOLD["q8_deq"])


def test_q4_k_decoders_match_gguf_py(oracle):
    k = GOLD["q8_x"].shape[1]
    assert np.array_equal(quant.dequantize_q4_k(GOLD["q4_blocks"], k), GOLD["q4_deq"])
    assert np.array_equal(oracle.dequant(oracle.T_Q4_K, GOLD["q4_blocks"], k), GOLD["q4_deq"])


def test_q4_k_encoder_is_stable():
    """Our Q4_K encoder is deterministic: the committed blocks are reproduced."""
    assert np.array_equal(quant.quantize_q4_k(GOLD["q8_x"]), GOLD["q4_blocks"])


def test_q4_k_error_bound():
    x = GOLD["q8_x"]
    err = np.abs(quant.dequantize_q4_k(quant.quantize_q4_k(x), x.shape[1]) - x)
    # per 32-value sub-block the step is (max-min)/15 (rounded scales): error <= ~1 step
    assert err.max() <= (x.max() - x.min()) / 15.0


@pytest.mark.parametrize("k", [32, 256])
def test_zero_rows(oracle, k):
    z = np.zeros((2, k), np.float32)
    assert np.array_equal(quant.dequantize_q8_0(quant.quantize_q8_0(z), k), z)
    if k % 256 == 0:
        assert np.array_equal(quant.dequantize_q4_k(quant.quantize_q4_k(z), k), z)


def test_f16_conversion_matches_numpy(oracle):
    L = oracle.lib()
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10,
                           np.array([0.0, -0.0, 65504.0, 65520.0, 1e-8, 6e-8, 5.96e-8, 3e-5, -3e-5, 1e5], np.float32)])
    for v in vals:
        h = np.float32(v).astype(np.float16)
        assert L.ceo_f32_to_f16(float(v)) == int(h.view(np.uint16)), v
        assert L.ceo_f16_to_f32(int(h.view(np.uint16))) == np.float32(h)
