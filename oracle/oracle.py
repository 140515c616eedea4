"""Python driver of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module.  It loads oracle/libceb_oracle.so (built from ceb_oracle.c by
oracle/Makefile) and strings the C ops together in the order of the
reference's encoder graph, build_encoder_graph (src/crispembed.cpp:1043-1466),
followed by the host pooling of encode_tokens (src/crispembed.cpp:1794-1846).

Parity status: block formats pinned against gguf-py; graph semantics restated
from the reference call sites and ggml's published CPU algorithms, with no
reference-produced vector to pin them ("parity unpinned", see ceb_oracle.c).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libceb_oracle.so")
# the timing build (C library expf / erff, as the reference's CPU path calls them):
# select it with use_timing_build() before the first call, for CPU-baseline timings only
TIMING_LIB_PATH = os.path.join(HERE, "libceb_oracle_timing.so")
_lib_path = LIB_PATH

EXACT, GGML, F16 = 0, 1, 2
T_F32, T_F16, T_Q8_0, T_Q4_K = 0, 1, 8, 12
T_Q4_0, T_Q4_1, T_Q5_0, T_Q5_1, T_Q5_K, T_Q6_K, T_IQ4_NL, T_IQ4_XS, T_BF16 = 2, 3, 6, 7, 13, 14, 20, 23, 30
_BLOCK = {T_F32: (1, 4), T_F16: (1, 2), T_BF16: (1, 2), T_Q4_0: (32, 18), T_Q4_1: (32, 20), T_Q5_0: (32, 22),
          T_Q5_1: (32, 24), T_Q8_0: (32, 34), T_Q4_K: (256, 144), T_Q5_K: (256, 176), T_Q6_K: (256, 210),
          T_IQ4_NL: (32, 18), T_IQ4_XS: (256, 136)}

_lib = None

_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int32)
_up = ctypes.POINTER(ctypes.c_uint8)


_SOURCES = [os.path.join(HERE, "ceb_oracle.c"),
            os.path.join(os.path.dirname(HERE), "crispembed_b200", "csrc", "ceb_portable_math.h")]


def build(force: bool = False) -> str:
    if force or any(not os.path.exists(t) or any(os.path.exists(p) and os.path.getmtime(t) < os.path.getmtime(p)
                                                 for p in _SOURCES) for t in (LIB_PATH, TIMING_LIB_PATH)):
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return _lib_path


def use_timing_build():
    """Load the timing build (the C library's expf / erff) instead of the parity build;
    call before any other function of this module (CPU-baseline timings only)."""
    global _lib_path
    if _lib is not None and _lib_path != TIMING_LIB_PATH:
        raise RuntimeError("the parity build is already loaded in this process")
    _lib_path = TIMING_LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_lib_path)
        L.ceo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.ceo_f16_to_f32.restype = ctypes.c_float
        L.ceo_f32_to_f16.argtypes = [ctypes.c_float]
        L.ceo_f32_to_f16.restype = ctypes.c_uint16
        L.ceo_dequant_row.argtypes = [ctypes.c_int, _up, ctypes.c_int64, _fp]
        L.ceo_quant_act_q8_0.argtypes = [_fp, ctypes.c_int64, _up]
        L.ceo_quant_act_q8_k.argtypes = [_fp, ctypes.c_int64, _up]
        L.ceo_dot_q8_0.argtypes = [ctypes.c_int64, _up, _up]
        L.ceo_dot_q8_0.restype = ctypes.c_float
        L.ceo_dot_q8_0_scalar.argtypes = [ctypes.c_int64, _up, _up]
        L.ceo_dot_q8_0_scalar.restype = ctypes.c_float
        L.ceo_dot_q4_k.argtypes = [ctypes.c_int64, _up, _up]
        L.ceo_dot_q4_k.restype = ctypes.c_float
        L.ceo_dot_q4_k_scalar.argtypes = [ctypes.c_int64, _up, _up]
        L.ceo_dot_q4_k_scalar.restype = ctypes.c_float
        L.ceo_matmul.argtypes = [ctypes.c_int, _up, ctypes.c_int64, ctypes.c_int64, _fp, ctypes.c_int64, _fp, _fp,
                                 ctypes.c_int]
        L.ceo_gelu_erf.argtypes = [_fp, ctypes.c_int64]
        L.ceo_layernorm.argtypes = [_fp, ctypes.c_int64, ctypes.c_int64, _fp, _fp, ctypes.c_float, _fp]
        L.ceo_attention.argtypes = [_fp, _fp, _fp, ctypes.c_int64, _ip, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_float, _fp, ctypes.c_int64]
        L.ceo_route.argtypes = [_fp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _ip, _fp, _fp]
        L.ceo_moe_ffn.argtypes = [_fp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, _up, ctypes.c_int, _up, _up, _fp, ctypes.c_int, _ip, _fp, _fp, _ip,
                                  _fp, _fp]
        L.ceo_moe_ffn2.argtypes = [_fp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int, _up, ctypes.c_int, _up, ctypes.c_int, _up, _fp, ctypes.c_int, _ip,
                                   _fp, _fp, _ip, _fp, _fp]
        L.ceo_moe_permutation.argtypes = [_ip, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _ip, _ip]
        L.ceo_pool_l2.argtypes = [_fp, _ip, ctypes.c_int, ctypes.c_int, _fp]
        L.ceo_truncate_renorm.argtypes = [_fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _fp]
        L.ceo_expf.argtypes = [ctypes.c_float]
        L.ceo_expf.restype = ctypes.c_float
        L.ceo_erff.argtypes = [ctypes.c_float]
        L.ceo_erff.restype = ctypes.c_float
        L.ceo_set_threads.argtypes = [ctypes.c_int]
        L.ceo_set_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _f(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def _i(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_ip)


def _u(a: np.ndarray):
    a = np.ascontiguousarray(a).view(np.uint8)
    return a.ctypes.data_as(_up), a


def set_threads(n: int) -> int:
    return lib().ceo_set_threads(int(n))


def f16_round(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def row_bytes(t: int, k: int) -> int:
    be, bb = _BLOCK[t]
    return k // be * bb


def dequant(t: int, raw: np.ndarray, k: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
    rows = raw.size // row_bytes(t, k)
    out = np.empty((rows, k), dtype=np.float32)
    rb = row_bytes(t, k)
    L = lib()
    for r in range(rows):
        p, _keep = _u(raw[r * rb:(r + 1) * rb])
        L.ceo_dequant_row(t, p, k, _f(out[r]))
    return out


def quant_act_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.zeros(x.size // 32 * 34, dtype=np.uint8)
    lib().ceo_quant_act_q8_0(_f(x), x.size, out.ctypes.data_as(_up))
    return out


def matmul(t: int, w_raw: np.ndarray, n_out: int, k: int, x: np.ndarray, mode: int,
           bias: Optional[np.ndarray] = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    out = np.empty((x.shape[0], n_out), dtype=np.float32)
    p, _keep = _u(w_raw)
    lib().ceo_matmul(t, p, n_out, k, _f(x), x.shape[0], _f(bias), _f(out), mode)
    return out


def gelu_erf(x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().ceo_gelu_erf(_f(y), y.size)
    return y


def layernorm(x: np.ndarray, gamma, beta, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().ceo_layernorm(_f(x), x.shape[0], x.shape[1], _f(gamma), _f(beta), eps, _f(out))
    return out


def route(logits: np.ndarray, k: int):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    ids = np.empty((T, k), dtype=np.int32)
    w = np.empty((T, k), dtype=np.float32)
    probs = np.empty((T, E), dtype=np.float32)
    lib().ceo_route(_f(logits), T, E, k, _i(ids), _f(w), _f(probs))
    return ids, w, probs


def moe_ffn(x: np.ndarray, E: int, k: int, F: int, router_type: int, router_raw: np.ndarray, wtype: int,
            fc1_raw: np.ndarray, fc2_raw: np.ndarray, bias: Optional[np.ndarray], mode: int,
            ids_in: Optional[np.ndarray] = None, wts_in: Optional[np.ndarray] = None,
            wtype2: Optional[int] = None):
    """Returns (y [T,d], ids [T,k], gate weights [T,k], router logits [T,E]).
    wtype2: fc2's block format when it differs from fc1's."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, d = x.shape
    y = np.empty((T, d), dtype=np.float32)
    ids = np.empty((T, k), dtype=np.int32)
    w = np.empty((T, k), dtype=np.float32)
    logits = np.empty((T, E), dtype=np.float32)
    pr, kr = _u(router_raw)
    p1, k1 = _u(fc1_raw)
    p2, k2 = _u(fc2_raw)
    ids_in = None if ids_in is None else np.ascontiguousarray(ids_in, dtype=np.int32)
    wts_in = None if wts_in is None else np.ascontiguousarray(wts_in, dtype=np.float32)
    lib().ceo_moe_ffn2(_f(x), T, d, E, k, F, router_type, pr, wtype, p1, wtype if wtype2 is None else wtype2, p2,
                       _f(bias), mode, _i(ids_in), _f(wts_in), _f(y), _i(ids), _f(w), _f(logits))
    return y, ids, w, logits


def moe_permutation(ids: np.ndarray, n_experts: int):
    """(slot_pos [T, k], offsets [E+1]) of the expert grouping of ids [T, k]: rows in
    (expert, token, slot) order, as ggml_mul_mat_id groups them."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, k = ids.shape
    slot_pos = np.empty((T, k), dtype=np.int32)
    offsets = np.empty(n_experts + 1, dtype=np.int32)
    lib().ceo_moe_permutation(_i(ids), T, k, n_experts, _i(slot_pos), _i(offsets))
    return slot_pos, offsets


def attention(qkv: np.ndarray, cu: np.ndarray, n_head: int, d: int) -> np.ndarray:
    qkv = np.ascontiguousarray(qkv, dtype=np.float32)
    M = qkv.shape[0]
    out = np.empty((M, d), dtype=np.float32)
    hd = d // n_head
    base = qkv.ctypes.data
    fsz = 4
    q = ctypes.cast(base, _fp)
    k = ctypes.cast(base + d * fsz, _fp)
    v = ctypes.cast(base + 2 * d * fsz, _fp)
    cu = np.ascontiguousarray(cu, dtype=np.int32)
    lib().ceo_attention(q, k, v, 3 * d, _i(cu), len(cu) - 1, n_head, hd, 1.0 / np.sqrt(hd), _f(out), d)
    return out


def pool_l2(hidden: np.ndarray, cu: np.ndarray) -> np.ndarray:
    hidden = np.ascontiguousarray(hidden, dtype=np.float32)
    cu = np.ascontiguousarray(cu, dtype=np.int32)
    n = len(cu) - 1
    out = np.empty((n, hidden.shape[1]), dtype=np.float32)
    lib().ceo_pool_l2(_f(hidden), _i(cu), n, hidden.shape[1], _f(out))
    return out


def truncate_renorm(emb: np.ndarray, dim: int) -> np.ndarray:
    emb = np.ascontiguousarray(emb, dtype=np.float32)
    out = np.empty((emb.shape[0], dim), dtype=np.float32)
    lib().ceo_truncate_renorm(_f(emb), emb.shape[0], emb.shape[1], dim, _f(out))
    return out


# ---------------------------------------------------------------------------
# encoder
# ---------------------------------------------------------------------------

@dataclass
class OracleModel:
    hp: Dict[str, float]
    t: Dict[str, np.ndarray]           # raw tensor bytes (views)
    types: Dict[str, int]
    shapes: Dict[str, tuple]           # ggml ne
    moe_layers: List[int] = field(default_factory=list)

    def f32(self, name: str) -> Optional[np.ndarray]:
        """A float table; block-format tables (llama.cpp exports quantize the token
        embeddings) are decoded row by row."""
        if name not in self.t:
            return None
        if self.types[name] == T_F32:
            return np.ascontiguousarray(self.t[name]).view(np.float32)
        k = int(self.shapes[name][0])
        return dequant(self.types[name], self.t[name], k).reshape(-1)


def load_model(path: str) -> OracleModel:
    """Read the GGUF (metadata keys and tensor names as load_model resolves them,
    src/crispembed.cpp:437-526 and :748-845, CrispEmbed-native enc.N.* names)."""
    import sys
    sys.path.insert(0, os.path.dirname(HERE))
    from crispembed_b200.gguf_io import read_gguf
    g = read_gguf(path)
    kv = g.kv
    arch = kv.get("general.architecture", "")

    def first(keys, default):
        for k in keys:
            if k in kv:
                return kv[k]
        return default

    hp = dict(
        n_embd=int(first(["bert.hidden_size", "bert.embedding_length", f"{arch}.embedding_length"], 384)),
        n_head=int(first(["bert.num_attention_heads", "bert.attention.head_count", f"{arch}.attention.head_count"], 12)),
        n_layer=int(first(["bert.num_hidden_layers", "bert.block_count", f"{arch}.block_count"], 6)),
        eps=float(first(["bert.layer_norm_eps", "bert.attention.layer_norm_epsilon",
                         f"{arch}.attention.layer_norm_epsilon"], 1e-12)),
        n_experts=int(first(["bert.num_experts", f"{arch}.expert_count"], 0)),
        top_k=int(first(["bert.num_experts_per_tok", f"{arch}.expert_used_count"], 0)),
        pos_offset=int(first(["bert.position_offset"], 0)),
        rope_theta=float(first(["bert.rope_theta", f"{arch}.rope.freq_base"], 10000.0)),
    )
    t, types, shapes = {}, {}, {}
    for name, info in g.tensors.items():
        t[name] = g.raw(name)
        types[name] = info.ggml_type
        shapes[name] = info.ne
    m = OracleModel(hp=hp, t=t, types=types, shapes=shapes)
    m.moe_layers = [il for il in range(hp["n_layer"]) if f"enc.{il}.ffn.moe_gate.weight" in t]
    return m


def rope_neox(x: np.ndarray, pos: np.ndarray, n_head: int, theta: float) -> np.ndarray:
    """ggml_rope_ext, NEOX pairing, n_dims = head_dim, no scaling (src/crispembed.cpp:1182-1195):
    dims i and i + hd/2 of each head rotate by pos * theta^(-2i/hd); the angle is
    built as ggml's rope cache builds it, multiplying by theta^(-2/hd) once per pair
    in float32, and cos/sin are taken in float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, d = x.shape
    hd = d // n_head
    half = hd // 2
    xs = x.reshape(M, n_head, hd)
    scale = np.float32(np.power(np.float32(theta), np.float32(-2.0 / hd), dtype=np.float32))
    th = pos.astype(np.float32)
    out = xs.copy()
    for i in range(half):
        c = np.cos(th).astype(np.float32)[:, None]
        s = np.sin(th).astype(np.float32)[:, None]
        x0, x1 = xs[:, :, i], xs[:, :, i + half]
        out[:, :, i] = x0 * c - x1 * s
        out[:, :, i + half] = x0 * s + x1 * c
        th = (th * scale).astype(np.float32)
    return out.reshape(M, d)


def encode(model: OracleModel, ids: np.ndarray, lens: np.ndarray, mode: int = GGML,
           dump: Optional[Dict[str, np.ndarray]] = None) -> np.ndarray:
    """Embeddings [n_seqs, d] for packed token ids (sequences concatenated).

    Every sequence is an independent graph in the reference (encode_tokens per
    sequence, src/crispembed.cpp:2222-2226, pos ids t + pos_offset per sequence,
    :1587-1588); row-wise ops are identical when sequences are packed, and
    attention is restricted to each sequence's own rows.
    """
    hp = model.hp
    d, nh, eps = hp["n_embd"], hp["n_head"], hp["eps"]
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    lens = np.asarray(lens, dtype=np.int64)
    cu = np.zeros(len(lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    M = int(cu[-1])
    pos = np.concatenate([np.arange(n, dtype=np.int64) for n in lens]) + hp["pos_offset"]

    tok = model.f32("token_embd.weight").reshape(-1, d)
    x = tok[ids].astype(np.float32)
    pe = model.f32("position_embd.weight")
    if pe is not None:
        x = x + pe.reshape(-1, d)[pos]
    te = model.f32("token_type_embd.weight")
    if te is None:
        te = model.f32("token_types.weight")
    if te is not None:
        x = x + te.reshape(-1, d)[0][None, :]
    x = np.ascontiguousarray(x, dtype=np.float32)
    if "embd_ln.weight" in model.t:
        x = layernorm(x, model.f32("embd_ln.weight"), model.f32("embd_ln.bias"), eps)
    if dump is not None:
        dump["emb_ln_out"] = x.copy()

    use_rope = "position_embd.weight" not in model.t  # src/crispembed.cpp:790-795

    def lin(name_w, name_b, inp, k_in):
        ne = model.shapes[name_w]
        n_out = int(ne[1])
        return matmul(model.types[name_w], model.t[name_w], n_out, k_in, inp, mode, model.f32(name_b))

    for il in range(hp["n_layer"]):
        p = f"enc.{il}."
        inp = x
        q = lin(p + "attn.q.weight", p + "attn.q.bias", x, d)
        k = lin(p + "attn.k.weight", p + "attn.k.bias", x, d)
        v = lin(p + "attn.v.weight", p + "attn.v.bias", x, d)
        if use_rope:
            q = rope_neox(q, pos, nh, hp["rope_theta"])
            k = rope_neox(k, pos, nh, hp["rope_theta"])
        qkv = np.concatenate([q, k, v], axis=1)
        attn = attention(qkv, cu, nh, d)
        attn = lin(p + "attn.o.weight", p + "attn.o.bias", attn, d)
        cur = layernorm(np.ascontiguousarray(inp + attn), model.f32(p + "ln1.weight"), model.f32(p + "ln1.bias"), eps)
        if il in model.moe_layers:
            E, K = hp["n_experts"], hp["top_k"]
            gname = p + "ffn.moe_gate.weight"
            f1 = p + "ffn.expert_fc1.weight"
            F = int(model.shapes[f1][1])
            ffn, rid, rw, logits = moe_ffn(cur, E, K, F, model.types[gname], model.t[gname], model.types[f1],
                                           model.t[f1], model.t[p + "ffn.expert_fc2.weight"],
                                           model.f32(p + "ffn.moe_bias"), mode,
                                           wtype2=model.types[p + "ffn.expert_fc2.weight"])
            if dump is not None:
                dump[f"router_in_{il}"] = cur.copy()
                dump[f"ids_{il}"] = rid
                dump[f"logits_{il}"] = logits
        else:
            F = int(model.shapes[p + "ffn.fc1.weight"][1])
            h = lin(p + "ffn.fc1.weight", p + "ffn.fc1.bias", cur, d)
            h = gelu_erf(h)
            ffn = lin(p + "ffn.fc2.weight", p + "ffn.fc2.bias", h, F)
        x = layernorm(np.ascontiguousarray(cur + ffn), model.f32(p + "ln2.weight"), model.f32(p + "ln2.bias"), eps)
        if dump is not None:
            dump[f"layer_{il}"] = x.copy()
    return pool_l2(x, cu)
