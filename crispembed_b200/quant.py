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


# ---------------------------------------------------------------------------
# encoders for the GGUF formats of llama.cpp community exports and the
# registry's IQ4_XS files.  Block layouts are ggml's published formats; the
# encoders are plain min/max (or abs-max) quantizers of our own, good enough for
# synthetic weights.  tests/test_formats.py checks every block they produce
# against gguf-py's decoder.
# ---------------------------------------------------------------------------

IQ4_CODEBOOK = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.float32)


def _f16(v: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(v, dtype=np.float32).astype(np.float16)


def _nibbles_32(q: np.ndarray) -> np.ndarray:
    """[nb, 32] values in 0..15 -> [nb, 16] bytes: element j low nibble, j+16 high nibble of byte j."""
    q = q.astype(np.uint8)
    return (q[:, :16] | (q[:, 16:] << 4)).astype(np.uint8)


def _blocks(x: np.ndarray, n: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.shape[-1] % n:
        raise ValueError(f"last dimension must be a multiple of {n}")
    return x.reshape(-1, n)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    b = _blocks(x, 32)
    d = (np.abs(b).max(axis=1) / 7.0).astype(np.float32)
    d16 = _f16(d)
    df = d16.astype(np.float32)
    inv = np.where(df == 0, 0.0, 1.0 / np.where(df == 0, 1.0, df)).astype(np.float32)
    q = np.clip(np.rint(b * inv[:, None]) + 8, 0, 15)
    out = np.empty((b.shape[0], 18), dtype=np.uint8)
    out[:, :2] = d16.reshape(-1, 1).view(np.uint8)
    out[:, 2:] = _nibbles_32(q)
    return out.reshape(*x.shape[:-1], -1)


def quantize_q4_1(x: np.ndarray) -> np.ndarray:
    b = _blocks(x, 32)
    lo, hi = b.min(axis=1), b.max(axis=1)
    d16, m16 = _f16((hi - lo) / 15.0), _f16(lo)
    df, mf = d16.astype(np.float32), m16.astype(np.float32)
    inv = np.where(df == 0, 0.0, 1.0 / np.where(df == 0, 1.0, df)).astype(np.float32)
    q = np.clip(np.rint((b - mf[:, None]) * inv[:, None]), 0, 15)
    out = np.empty((b.shape[0], 20), dtype=np.uint8)
    out[:, 0:2] = d16.reshape(-1, 1).view(np.uint8)
    out[:, 2:4] = m16.reshape(-1, 1).view(np.uint8)
    out[:, 4:] = _nibbles_32(q)
    return out.reshape(*x.shape[:-1], -1)


def _qh_32(q5: np.ndarray) -> np.ndarray:
    """fifth bits of 32 five-bit values -> little-endian uint32 bytes (bit j = value j)."""
    bits = ((q5.astype(np.uint32) >> 4) & 1) << np.arange(32, dtype=np.uint32)
    return bits.sum(axis=1).astype(np.uint32).reshape(-1, 1).view(np.uint8)


def quantize_q5_0(x: np.ndarray) -> np.ndarray:
    b = _blocks(x, 32)
    d16 = _f16(np.abs(b).max(axis=1) / 15.0)
    df = d16.astype(np.float32)
    inv = np.where(df == 0, 0.0, 1.0 / np.where(df == 0, 1.0, df)).astype(np.float32)
    q = np.clip(np.rint(b * inv[:, None]) + 16, 0, 31).astype(np.uint8)
    out = np.empty((b.shape[0], 22), dtype=np.uint8)
    out[:, 0:2] = d16.reshape(-1, 1).view(np.uint8)
    out[:, 2:6] = _qh_32(q)
    out[:, 6:] = _nibbles_32(q & 0xF)
    return out.reshape(*x.shape[:-1], -1)


def quantize_q5_1(x: np.ndarray) -> np.ndarray:
    b = _blocks(x, 32)
    lo, hi = b.min(axis=1), b.max(axis=1)
    d16, m16 = _f16((hi - lo) / 31.0), _f16(lo)
    df, mf = d16.astype(np.float32), m16.astype(np.float32)
    inv = np.where(df == 0, 0.0, 1.0 / np.where(df == 0, 1.0, df)).astype(np.float32)
    q = np.clip(np.rint((b - mf[:, None]) * inv[:, None]), 0, 31).astype(np.uint8)
    out = np.empty((b.shape[0], 24), dtype=np.uint8)
    out[:, 0:2] = d16.reshape(-1, 1).view(np.uint8)
    out[:, 2:4] = m16.reshape(-1, 1).view(np.uint8)
    out[:, 4:8] = _qh_32(q)
    out[:, 8:] = _nibbles_32(q & 0xF)
    return out.reshape(*x.shape[:-1], -1)


def _iq4_index(v: np.ndarray) -> np.ndarray:
    """nearest codebook entry of each value (in codebook units)."""
    return np.abs(v[..., None] - IQ4_CODEBOOK).argmin(axis=-1).astype(np.uint8)


def quantize_iq4_nl(x: np.ndarray) -> np.ndarray:
    b = _blocks(x, 32)
    d16 = _f16(np.abs(b).max(axis=1) / 127.0)
    df = d16.astype(np.float32)
    inv = np.where(df == 0, 0.0, 1.0 / np.where(df == 0, 1.0, df)).astype(np.float32)
    q = _iq4_index(b * inv[:, None])
    out = np.empty((b.shape[0], 18), dtype=np.uint8)
    out[:, :2] = d16.reshape(-1, 1).view(np.uint8)
    out[:, 2:] = _nibbles_32(q)
    return out.reshape(*x.shape[:-1], -1)


def quantize_iq4_xs(x: np.ndarray) -> np.ndarray:
    """fp16 d, scales_h (2 high bits of 8 six-bit ls), scales_l[4] (4 low bits), qs[128];
    sub-block scale d * (ls - 32)."""
    b = _blocks(x, 256)
    nb = b.shape[0]
    sub = b.reshape(nb, 8, 32)
    s = np.abs(sub).max(axis=2) / 127.0                      # wanted sub-block scales (>= 0)
    d16 = _f16(s.max(axis=1) / 31.0)
    df = d16.astype(np.float32)
    inv = np.where(df == 0, 0.0, 1.0 / np.where(df == 0, 1.0, df)).astype(np.float32)
    ls = np.clip(np.rint(s * inv[:, None]) + 32, 0, 63).astype(np.uint16)
    dl = df[:, None] * (ls.astype(np.float32) - 32)
    invl = np.where(dl == 0, 0.0, 1.0 / np.where(dl == 0, 1.0, dl)).astype(np.float32)
    q = _iq4_index(sub * invl[:, :, None])
    out = np.zeros((nb, 136), dtype=np.uint8)
    out[:, 0:2] = d16.reshape(-1, 1).view(np.uint8)
    sh = np.zeros(nb, dtype=np.uint16)
    for ib in range(8):
        sh |= ((ls[:, ib] >> 4) & 3) << (2 * ib)
        out[:, 4 + ib // 2] |= ((ls[:, ib] & 0xF) << (4 * (ib % 2))).astype(np.uint8)
    out[:, 2:4] = sh.reshape(-1, 1).view(np.uint8)
    out[:, 8:] = _nibbles_32(q.reshape(-1, 32)).reshape(nb, 128)
    return out.reshape(*x.shape[:-1], -1)


def quantize_q5_k(x: np.ndarray) -> np.ndarray:
    """Q4_K's scales/mins layout with a fifth bit per value: fp16 d, fp16 dmin,
    scales[12], qh[32] (bit 2c / 2c+1 of byte l: value l of chunk c's low / high
    half), qs[128] (chunk c: byte l = value l low nibble, value 32+l high nibble)."""
    b = _blocks(x, 256)
    nb = b.shape[0]
    sub = b.reshape(nb, 8, 32)
    mn = np.maximum(-sub.min(axis=2), 0.0)                    # offsets (value = d*sc*q - dmin*m)
    sc = (sub.max(axis=2) + mn) / 31.0
    d16, dm16 = _f16(sc.max(axis=1) / 63.0), _f16(mn.max(axis=1) / 63.0)
    df, dmf = d16.astype(np.float32), dm16.astype(np.float32)
    inv = np.where(df == 0, 0.0, 1.0 / np.where(df == 0, 1.0, df)).astype(np.float32)
    invm = np.where(dmf == 0, 0.0, 1.0 / np.where(dmf == 0, 1.0, dmf)).astype(np.float32)
    isc = np.clip(np.rint(sc * inv[:, None]), 0, 63).astype(np.uint8)
    imn = np.clip(np.rint(mn * invm[:, None]), 0, 63).astype(np.uint8)
    d1 = df[:, None] * isc.astype(np.float32)
    m1 = dmf[:, None] * imn.astype(np.float32)
    invd1 = np.where(d1 == 0, 0.0, 1.0 / np.where(d1 == 0, 1.0, d1)).astype(np.float32)
    q = np.clip(np.rint((sub + m1[:, :, None]) * invd1[:, :, None]), 0, 31).astype(np.uint8)  # [nb, 8, 32]
    out = np.zeros((nb, 176), dtype=np.uint8)
    out[:, 0:2] = d16.reshape(-1, 1).view(np.uint8)
    out[:, 2:4] = dm16.reshape(-1, 1).view(np.uint8)
    out[:, 4:16] = _pack_scales(isc, imn)
    qh = np.zeros((nb, 32), dtype=np.uint8)
    for c in range(4):
        lo, hi = q[:, 2 * c], q[:, 2 * c + 1]
        out[:, 48 + 32 * c:48 + 32 * (c + 1)] = (lo & 0xF) | ((hi & 0xF) << 4)
        qh |= ((lo >> 4) & 1) << (2 * c)
        qh |= ((hi >> 4) & 1) << (2 * c + 1)
    out[:, 16:48] = qh
    return out.reshape(*x.shape[:-1], -1)


def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    """ql[128] (low 4 bits), qh[64] (high 2 bits), int8 scales[16] (one per 16
    values), fp16 d; value = d * sc * (q - 32).  Per 128-value half n, value
    l + 32 t (t = 0..3, l = 0..31) takes ql[64 n + l + 32 (t & 1)]'s low (t < 2)
    or high (t >= 2) nibble and bits 2t..2t+1 of qh[32 n + l]."""
    b = _blocks(x, 256)
    nb = b.shape[0]
    sub = b.reshape(nb, 16, 16)
    s = np.abs(sub).max(axis=2) / 31.0
    d16 = _f16(s.max(axis=1) / 127.0)
    df = d16.astype(np.float32)
    inv = np.where(df == 0, 0.0, 1.0 / np.where(df == 0, 1.0, df)).astype(np.float32)
    isc = np.clip(np.rint(s * inv[:, None]), -128, 127).astype(np.int8)
    dl = df[:, None] * isc.astype(np.float32)
    invl = np.where(dl == 0, 0.0, 1.0 / np.where(dl == 0, 1.0, dl)).astype(np.float32)
    q = np.clip(np.rint(sub * invl[:, :, None]) + 32, 0, 63).astype(np.uint8).reshape(nb, 256)
    out = np.zeros((nb, 210), dtype=np.uint8)
    for n in range(2):
        for t in range(4):
            v = q[:, 128 * n + 32 * t:128 * n + 32 * (t + 1)]   # values l + 32 t of half n
            lo = v & 0xF
            ql0 = 64 * n + 32 * (t & 1)
            if t < 2:
                out[:, ql0:ql0 + 32] |= lo
            else:
                out[:, ql0:ql0 + 32] |= lo << 4
            out[:, 128 + 32 * n:128 + 32 * (n + 1)] |= ((v >> 4) & 3) << (2 * t)
    out[:, 192:208] = isc.view(np.uint8)
    out[:, 208:210] = d16.reshape(-1, 1).view(np.uint8)
    return out.reshape(*x.shape[:-1], -1)


def quantize(x: np.ndarray, ggml_type: int) -> np.ndarray:
    from . import gguf_io as G
    if ggml_type == G.GGML_F32:
        return np.ascontiguousarray(x, dtype=np.float32)
    if ggml_type == G.GGML_F16:
        return np.ascontiguousarray(x, dtype=np.float16)
    if ggml_type == G.GGML_BF16:
        u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even
        return r
    enc = {G.GGML_Q8_0: quantize_q8_0, G.GGML_Q4_K: quantize_q4_k, G.GGML_Q4_0: quantize_q4_0,
           G.GGML_Q4_1: quantize_q4_1, G.GGML_Q5_0: quantize_q5_0, G.GGML_Q5_1: quantize_q5_1,
           G.GGML_Q5_K: quantize_q5_k, G.GGML_Q6_K: quantize_q6_k, G.GGML_IQ4_NL: quantize_iq4_nl,
           G.GGML_IQ4_XS: quantize_iq4_xs}
    if ggml_type not in enc:
        raise ValueError(f"unsupported ggml type {ggml_type}")
    return enc[ggml_type](x)


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
