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


# ---------------------------------------------------------------------------
# formats of llama.cpp community exports and the registry's IQ4_XS files
# ---------------------------------------------------------------------------
VAR = np.load(os.path.join(os.path.dirname(__file__), "golden", "gguf_variants.npz"))
VARIANTS = ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q5_K", "Q6_K", "IQ4_NL", "IQ4_XS", "BF16"]


@pytest.mark.parametrize("name", VARIANTS)
def test_variant_decoders_match_gguf_py(oracle, name):
    """The library's host decoder (ceb_gguf_dequantize) and the oracle's decode the
    committed blocks to gguf-py's values bit for bit."""
    from crispembed_b200 import binding
    from crispembed_b200 import gguf_io as G
    t = getattr(G, "GGML_" + name)
    blocks, want = VAR[name + "_blocks"], VAR[name + "_deq"]
    rows, k = want.shape
    assert np.array_equal(binding.gguf_dequantize(t, blocks, rows, k), want)
    assert np.array_equal(oracle.dequant(t, blocks, k), want)


@pytest.mark.parametrize("name", VARIANTS)
def test_variant_encoders_are_stable_and_close(name):
    """crispembed_b200.quant reproduces the committed blocks, and they decode close
    to the source matrix (an all-zero super-block decodes to zeros)."""
    from crispembed_b200 import gguf_io as G
    t = getattr(G, "GGML_" + name)
    x = VAR["x"]
    assert np.array_equal(quant.quantize(x, t).view(np.uint8).reshape(x.shape[0], -1), VAR[name + "_blocks"])
    deq = VAR[name + "_deq"]
    assert np.abs(deq[0, :256]).max() == 0.0
    rel = np.abs(deq[2:] - x[2:]).max() / np.abs(x[2:]).max()
    assert rel < (0.01 if name == "BF16" else 0.2), rel


def test_dequantize_rejects_unsupported():
    from crispembed_b200 import binding
    with pytest.raises(binding.CrispEmbedError):
        binding.gguf_dequantize(10, np.zeros(84, np.uint8), 1, 256)  # Q2_K is not read by this library
    with pytest.raises(binding.CrispEmbedError):
        binding.gguf_dequantize(2, np.zeros(18, np.uint8), 1, 40)    # not a whole Q4_0 block
