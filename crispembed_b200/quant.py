"""numpy encoders for the two GGUF block formats on the MoE path.

Q8_0 (34 B per 32 values): fp16 ``d`` then 32 int8 ``qs``; value = d * q.
  The encoder follows the reference converter, which quantizes weights with
  gguf-py (models/convert-bert-to-gguf.py:68-77): d = amax/127, q = roundf(x/d)
  with ties away from zero.  Bit-equality with gguf-py is checked by
  tests/test_formats.py.

Q4_K (144 B per 256 values): fp16 ``d``, fp16 ``dmin``, 12 bytes of packed
  6-bit sub-block scales/mins (8 sub-blocks of 32), 128 bytes of 4-bit quants.
  value = d*sc[j]*q - dmin*m[j].  Within each 64-value chunk, byte l holds value
  l in its low nibble and value 32+l in its high nibble.  gguf-py can decode but
  not encode Q4_K, and the reference quantizer (tools/quantize.cpp) needs ggml,
  so this is our own min/max encoder; any block that gguf-py decodes to the
  same values as our decoder is a valid Q4_K block for the path.
"""
from __future__ import annotations

import numpy as np

QK8_0 = 32
QK_K = 256


def _roundf(v: np.ndarray) -> np.ndarray:
    """C roundf: nearest integer, ties away from zero."""
    a = np.abs(v)
    f = np.floor(a)
    return np.sign(v) * (f + np.floor(2.0 * (a - f)))


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """float array [..., K] (K % 32 == 0) -> uint8 blocks [..., K/32*34]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    shape = x.shape
    if shape[-1] % QK8_0:
        raise ValueError("Q8_0 needs the last dimension to be a multiple of 32")
    blocks = x.reshape(-1, QK8_0)
    d = np.abs(blocks).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = _roundf(blocks * inv).astype(np.int8)
    out = np.empty((blocks.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(*shape[:-1], shape[-1] // QK8_0 * 34)


def dequantize_q8_0(b: np.ndarray, k: int) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8).reshape(-1, 34)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(-1, k)


def _pack_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """sc, mn: [nb, 8] uint8 in [0,63] -> [nb, 12] packed bytes."""
    nb = sc.shape[0]
    s = np.zeros((nb, 12), dtype=np.uint8)
    for i in range(4):
        s[:, i] = (sc[:, i] & 63) | ((sc[:, i + 4] >> 4) << 6)
        s[:, i + 4] = (mn[:, i] & 63) | ((mn[:, i + 4] >> 4) << 6)
        s[:, i + 8] = (sc[:, i + 4] & 15) | ((mn[:, i + 4] & 15) << 4)
    return s


def _unpack_scales(s: np.ndarray):
    nb = s.shape[0]
    sc = np.zeros((nb, 8), dtype=np.uint8)
    mn = np.zeros((nb, 8), dtype=np.uint8)
    for j in range(4):
        sc[:, j] = s[:, j] & 63
        mn[:, j] = s[:, j + 4] & 63
    for j in range(4, 8):
        sc[:, j] = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
        mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    return sc, mn


def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    """float array [..., K] (K % 256 == 0) -> uint8 blocks [..., K/256*144]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    shape = x.shape
    if shape[-1] % QK_K:
        raise ValueError("Q4_K needs the last dimension to be a multiple of 256")
    blk = x.reshape(-1, 8, 32)
    nb = blk.shape[0]
    lo = np.minimum(blk.min(axis=2), 0.0)            # [nb, 8]
    hi = blk.max(axis=2)
    scale = (hi - lo) / 15.0                          # per sub-block step
    off = -lo                                         # >= 0
    d = (scale.max(axis=1) / 63.0).astype(np.float16)
    dmin = (off.max(axis=1) / 63.0).astype(np.float16)
    d32 = d.astype(np.float32)
    dm32 = dmin.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32[:, None] > 0, np.rint(scale / d32[:, None]), 0)
        mn = np.where(dm32[:, None] > 0, np.rint(off / dm32[:, None]), 0)
    sc = np.clip(sc, 0, 63).astype(np.uint8)
    mn = np.clip(mn, 0, 63).astype(np.uint8)
    step = d32[:, None] * sc.astype(np.float32)      # [nb, 8]
    base = dm32[:, None] * mn.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(step[:, :, None] > 0, np.rint((blk + base[:, :, None]) / step[:, :, None]), 0)
    q = np.clip(q, 0, 15).astype(np.uint8).reshape(nb, 4, 2, 32)  # chunk, half, lane
    qs = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(nb, 128)
    out = np.empty((nb, 144), dtype=np.uint8)
    out[:, 0:2] = d.reshape(nb, 1).view(np.uint8)
    out[:, 2:4] = dmin.reshape(nb, 1).view(np.uint8)
    out[:, 4:16] = _pack_scales(sc, mn)
    out[:, 16:] = qs
    return out.reshape(*shape[:-1], shape[-1] // QK_K * 144)


def dequantize_q4_k(b: np.ndarray, k: int) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8).reshape(-1, 144)
    nb = b.shape[0]
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(nb)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(nb)
    sc, mn = _unpack_scales(b[:, 4:16])
    qs = b[:, 16:].reshape(nb, 4, 32)
    q = np.stack([qs & 0xF, qs >> 4], axis=2).reshape(nb, 8, 32).astype(np.float32)
    d1 = (d[:, None] * sc.astype(np.float32)).astype(np.float32)
    m1 = (dmin[:, None] * mn.astype(np.float32)).astype(np.float32)
    return (d1[:, :, None] * q - m1[:, :, None]).astype(np.float32).reshape(-1, k)


def quantize(x: np.ndarray, ggml_type: int) -> np.ndarray:
    from .gguf_io import GGML_F16, GGML_F32, GGML_Q4_K, GGML_Q8_0
    if ggml_type == GGML_F32:
        return np.ascontiguousarray(x, dtype=np.float32)
    if ggml_type == GGML_F16:
        return np.ascontiguousarray(x, dtype=np.float16)
    if ggml_type == GGML_Q8_0:
        return quantize_q8_0(x)
    if ggml_type == GGML_Q4_K:
        return quantize_q4_k(x)
    raise ValueError(f"unsupported ggml type {ggml_type}")


def dequantize(raw: np.ndarray, ggml_type: int, k: int) -> np.ndarray:
    from .gguf_io import GGML_F16, GGML_F32, GGML_Q4_K, GGML_Q8_0
    raw = np.ascontiguousarray(raw).view(np.uint8)
    if ggml_type == GGML_F32:
        return raw.view(np.float32).reshape(-1, k)
    if ggml_type == GGML_F16:
        return raw.view(np.float16).astype(np.float32).reshape(-1, k)
    if ggml_type == GGML_Q8_0:
        return dequantize_q8_0(raw, k)
    if ggml_type == GGML_Q4_K:
        return dequantize_q4_k(raw, k)
    raise ValueError(f"unsupported ggml type {ggml_type}")
