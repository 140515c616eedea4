"""Seeded synthetic NomicBERT-MoE models and inputs for the benchmark configs.

There is no network in this environment, so the real nomic-embed-text-v2-moe
checkpoint cannot be fetched.  This module writes a random-init model with the
same architecture and the same GGUF layout as the reference converter
(models/convert-bert-to-gguf.py, CrispEmbed-native ``enc.N.*`` names,
``bert.*`` keys, experts stacked as numpy [E, F, d] / [E, d, F] per
models/convert-bert-to-gguf.py:1056-1081):

* token/position/type embeddings and all norms stay F32 (the converter writes
  them with ``f32``), every linear weight uses the chosen block type (the
  converter's ``wt``), biases stay F32;
* linear weights and biases ~ N(0, 0.02); LayerNorm gamma ~ 1 + N(0, 0.02),
  beta ~ N(0, 0.02), so the affine parts of every norm are exercised;
* one ``numpy.random.default_rng(seed)`` stream, tensors drawn in file order
  (recorded in ``general.fixture_order``).

The vocabulary is a synthetic WordPiece list: ids 0-4 are [PAD] [CLS] [SEP]
[UNK] [MASK], id i >= 5 is the 4-letter lowercase word spelling i-5 in base 26,
so any id sequence can also be driven through the text ABI 1:1.
"""
from __future__ import annotations

from dataclasses import dataclass, field, asdict
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import gguf_io as G
from .quant import quantize

SPECIAL_TOKENS = ["[PAD]", "[CLS]", "[SEP]", "[UNK]", "[MASK]"]


def vocab_word(i: int) -> str:
    if i < len(SPECIAL_TOKENS):
        return SPECIAL_TOKENS[i]
    v = i - len(SPECIAL_TOKENS)
    s = []
    for _ in range(4):
        s.append(chr(ord("a") + v % 26))
        v //= 26
    return "".join(reversed(s))


@dataclass
class ModelSpec:
    n_vocab: int = 250048
    n_ctx: int = 512
    d: int = 768
    n_head: int = 12
    n_layer: int = 12
    ffn: int = 3072          # dense FFN width
    n_experts: int = 8
    top_k: int = 2
    expert_ffn: int = 3072
    moe_every: int = 2       # MoE on layers il % moe_every == moe_every - 1 (1, 3, 5, ...)
    type_vocab: int = 2
    ln_eps: float = 1e-5
    wtype: int = G.GGML_Q8_0  # linear-weight block type
    router_wtype: Optional[int] = None  # None = same as wtype (the converter quantizes the router too)
    moe_bias: bool = True
    seed: int = 0
    # per-tensor block types by name suffix ("attn.o.weight", "ffn.expert_fc2.weight",
    # "token_embd.weight", ...), for mixed-format files such as llama.cpp's Q4_K_M
    type_overrides: Dict[str, int] = field(default_factory=dict)
    rope_theta: float = 0.0  # > 0: no position table, RoPE (NEOX) with this base, as NomicBERT v1 GGUFs
    qk_scale: float = 0.02   # std of the q/k projection weights (larger: sharper attention)

    def is_moe(self, il: int) -> bool:
        return self.n_experts > 0 and self.moe_every > 0 and il % self.moe_every == self.moe_every - 1


def nomic_moe_spec(wtype: int = G.GGML_Q8_0) -> ModelSpec:
    """BASELINE configs 1/2/4: shape of nomic-embed-text-v2-moe with learned positions."""
    return ModelSpec(wtype=wtype)


def tiny_spec(wtype: int = G.GGML_Q8_0, **kw) -> ModelSpec:
    """Small model with the same structure, for tests that must finish in seconds."""
    base = dict(n_vocab=1000, n_ctx=128, d=256, n_head=4, n_layer=4, ffn=512, n_experts=4, top_k=2,
                expert_ffn=512, wtype=wtype)
    base.update(kw)
    return ModelSpec(**base)


LLAMA_NAMES = {  # CrispEmbed-native suffix -> llama.cpp nomic-bert-moe name (src/crispembed.cpp:800-845)
    "attn.o.weight": "attn_output.weight", "attn.o.bias": "attn_output.bias",
    "ln1.weight": "attn_output_norm.weight", "ln1.bias": "attn_output_norm.bias",
    "ln2.weight": "layer_output_norm.weight", "ln2.bias": "layer_output_norm.bias",
    "ffn.fc1.weight": "ffn_up.weight", "ffn.fc1.bias": "ffn_up.bias",
    "ffn.fc2.weight": "ffn_down.weight", "ffn.fc2.bias": "ffn_down.bias",
    "ffn.moe_gate.weight": "ffn_gate_inp.weight", "ffn.expert_fc1.weight": "ffn_up_exps.weight",
    "ffn.expert_fc2.weight": "ffn_down_exps.weight",
}


def write_model(path: str, spec: ModelSpec, tokenizer=None, naming: str = "crisp") -> List[str]:
    """Write the synthetic GGUF; returns the tensor order.

    `tokenizer(writer)` replaces the default synthetic WordPiece keys (it must
    write spec.n_vocab tokens).  naming="llama" writes the same weights under
    llama.cpp's nomic-bert-moe names (blk.N.*, a fused attn_qkv with rows q|k|v,
    token_embd_norm, nomic-bert-moe.* keys) as community exports do."""
    if naming == "llama":
        return _write_llama_naming(path, spec, tokenizer)
    rng = np.random.default_rng(spec.seed)
    w = G.GGUFWriter(path)
    w.add_str("general.architecture", "nomic-bert-moe")
    w.add_str("general.name", "crispembed-b200 synthetic nomic-bert-moe")
    w.add_u32("bert.vocab_size", spec.n_vocab)
    w.add_u32("bert.max_position_embeddings", spec.n_ctx)
    w.add_u32("bert.hidden_size", spec.d)
    w.add_u32("bert.num_attention_heads", spec.n_head)
    w.add_u32("bert.num_hidden_layers", spec.n_layer)
    w.add_u32("bert.intermediate_size", spec.ffn)
    w.add_f32("bert.layer_norm_eps", spec.ln_eps)
    w.add_u32("bert.pooling_method", 0)
    if spec.n_experts > 0:
        w.add_u32("bert.num_experts", spec.n_experts)
        w.add_u32("bert.num_experts_per_tok", spec.top_k)
    if tokenizer is not None:
        tokenizer(w)
    else:
        w.add_u32("tokenizer.ggml.type", 0)
        w.add_str_array("tokenizer.ggml.tokens", [vocab_word(i) for i in range(spec.n_vocab)])
        w.add_u32("tokenizer.ggml.padding_token_id", 0)
        w.add_u32("tokenizer.ggml.cls_token_id", 1)
        w.add_u32("tokenizer.ggml.sep_token_id", 2)
        w.add_u32("tokenizer.ggml.unknown_token_id", 3)

    order: List[str] = []
    d, wt = spec.d, spec.wtype
    rwt = spec.router_wtype if spec.router_wtype is not None else wt

    def normal(shape, scale=0.02, loc=0.0):
        a = rng.standard_normal(size=shape, dtype=np.float32)
        a *= np.float32(scale)
        if loc:
            a += np.float32(loc)
        return a

    def add(name, np_shape, gtype, gen):
        ne = tuple(reversed(np_shape))
        order.append(name)
        for suffix, t in spec.type_overrides.items():
            if name.endswith(suffix):
                gtype = t
        w.add_tensor(name, ne, gtype, lambda: quantize(gen(), gtype))

    add("token_embd.weight", (spec.n_vocab, d), G.GGML_F32, lambda: normal((spec.n_vocab, d)))
    if spec.rope_theta > 0:
        w.add_f32("bert.rope_theta", spec.rope_theta)
    else:
        add("position_embd.weight", (spec.n_ctx, d), G.GGML_F32, lambda: normal((spec.n_ctx, d)))
    if spec.type_vocab > 0:
        add("token_type_embd.weight", (spec.type_vocab, d), G.GGML_F32, lambda: normal((spec.type_vocab, d)))
    add("embd_ln.weight", (d,), G.GGML_F32, lambda: normal((d,), loc=1.0))
    add("embd_ln.bias", (d,), G.GGML_F32, lambda: normal((d,)))
    for il in range(spec.n_layer):
        p = f"enc.{il}."
        for nm in ("q", "k", "v"):
            sc = spec.qk_scale if nm != "v" else 0.02
            add(p + f"attn.{nm}.weight", (d, d), wt, lambda sc=sc: normal((d, d), scale=sc))
            add(p + f"attn.{nm}.bias", (d,), G.GGML_F32, lambda: normal((d,)))
        add(p + "attn.o.weight", (d, d), wt, lambda: normal((d, d)))
        add(p + "attn.o.bias", (d,), G.GGML_F32, lambda: normal((d,)))
        add(p + "ln1.weight", (d,), G.GGML_F32, lambda: normal((d,), loc=1.0))
        add(p + "ln1.bias", (d,), G.GGML_F32, lambda: normal((d,)))
        if spec.is_moe(il):
            E, Fm = spec.n_experts, spec.expert_ffn
            add(p + "ffn.moe_gate.weight", (E, d), rwt, lambda: normal((E, d)))
            add(p + "ffn.expert_fc1.weight", (E, Fm, d), wt, lambda: normal((E, Fm, d)))
            add(p + "ffn.expert_fc2.weight", (E, d, Fm), wt, lambda: normal((E, d, Fm)))
            if spec.moe_bias:
                add(p + "ffn.moe_bias", (d,), G.GGML_F32, lambda: normal((d,)))
        else:
            F = spec.ffn
            add(p + "ffn.fc1.weight", (F, d), wt, lambda: normal((F, d)))
            add(p + "ffn.fc1.bias", (F,), G.GGML_F32, lambda: normal((F,)))
            add(p + "ffn.fc2.weight", (d, F), wt, lambda: normal((d, F)))
            add(p + "ffn.fc2.bias", (d,), G.GGML_F32, lambda: normal((d,)))
        add(p + "ln2.weight", (d,), G.GGML_F32, lambda: normal((d,), loc=1.0))
        add(p + "ln2.bias", (d,), G.GGML_F32, lambda: normal((d,)))
    w.add_str("general.fixture_order", ",".join(order))
    w.add_str("general.fixture_init", f"numpy default_rng({spec.seed}); N(0,0.02); LN gamma 1+N(0,0.02), beta N(0,0.02)")
    w.write()
    return order


def _write_llama_naming(path: str, spec: ModelSpec, tokenizer=None) -> List[str]:
    """The tensors of write_model(spec) (same draws, same bytes per row) under
    llama.cpp's names and keys."""
    import os
    import tempfile
    with tempfile.TemporaryDirectory() as td:
        tmp = os.path.join(td, "crisp.gguf")
        write_model(tmp, spec, tokenizer)
        src = G.read_gguf(tmp)
        arch = "nomic-bert-moe"
        w = G.GGUFWriter(path)
        w.add_str("general.architecture", arch)
        w.add_str("general.name", "crispembed-b200 synthetic nomic-bert-moe (llama.cpp naming)")
        keys = {"bert.vocab_size": None, "bert.max_position_embeddings": "context_length",
                "bert.hidden_size": "embedding_length", "bert.num_attention_heads": "attention.head_count",
                "bert.num_hidden_layers": "block_count", "bert.intermediate_size": "feed_forward_length",
                "bert.layer_norm_eps": "attention.layer_norm_epsilon", "bert.num_experts": "expert_count",
                "bert.num_experts_per_tok": "expert_used_count", "bert.rope_theta": "rope.freq_base"}
        for k, v in src.kv.items():
            if k in keys:
                if keys[k] is None:
                    continue
                val = v
                if isinstance(val, float):
                    w.add_f32(f"{arch}.{keys[k]}", val)
                else:
                    w.add_u32(f"{arch}.{keys[k]}", int(val))
            elif k.startswith("tokenizer."):
                if isinstance(v, list):
                    if v and isinstance(v[0], str):
                        w.add_str_array(k, v)
                    else:
                        w.add_f32_array(k, v)
                elif isinstance(v, str):
                    w.add_str(k, v)
                elif isinstance(v, bool):
                    w.add_bool(k, v)
                else:
                    w.add_u32(k, int(v))
        w.add_u32(f"{arch}.pooling_type", 1)  # llama.cpp's MEAN
        order: List[str] = []

        def put(name, info_name, data=None, ne=None, gtype=None):
            info = src.tensors[info_name]
            raw = src.raw(info_name) if data is None else data
            w.add_tensor(name, info.ne if ne is None else ne, info.ggml_type if gtype is None else gtype,
                         lambda raw=raw: raw)
            order.append(name)

        renames = {"embd_ln.weight": "token_embd_norm.weight", "embd_ln.bias": "token_embd_norm.bias",
                   "token_type_embd.weight": "token_types.weight"}
        for name in src.tensors:
            if not name.startswith("enc."):
                put(renames.get(name, name), name)
                continue
            il, rest = name[4:].split(".", 1)
            b = f"blk.{il}."
            if rest in ("attn.q.weight", "attn.q.bias"):
                part = rest.split(".")[2]
                names = [f"enc.{il}.attn.{x}.{part}" for x in "qkv"]
                raws = [np.ascontiguousarray(src.raw(n)).view(np.uint8).reshape(-1) for n in names]
                ne = src.tensors[names[0]].ne
                fused_ne = (ne[0], 3 * ne[1]) if len(ne) == 2 else (3 * ne[0],)
                put(b + "attn_qkv." + part, names[0], data=np.concatenate(raws), ne=fused_ne)
            elif rest.startswith("attn.k.") or rest.startswith("attn.v."):
                continue
            elif rest == "ffn.moe_bias":  # the reference reads the expert bias under its native name only
                put(name, name)
            else:
                put(b + LLAMA_NAMES[rest], name)
        w.write()
        return order


# ---------------------------------------------------------------------------
# token-id batches (2, 4)
# ---------------------------------------------------------------------------

def ids_fixed(n_seqs: int, seq_len: int, seed: int, lo: int = 5, hi: int = 250000) -> Tuple[np.ndarray, np.ndarray]:
    rng = np.random.default_rng(seed)
    ids = rng.integers(lo, hi, size=(n_seqs * seq_len,), dtype=np.int64).astype(np.int32)
    lens = np.full((n_seqs,), seq_len, dtype=np.int32)
    return ids, lens


def ids_ragged(n_seqs: int, min_len: int, max_len: int, seed: int, lo: int = 5, hi: int = 250000):
    rng = np.random.default_rng(seed)
    lens = rng.integers(min_len, max_len + 1, size=(n_seqs,), dtype=np.int64).astype(np.int32)
    ids = rng.integers(lo, hi, size=(int(lens.sum()),), dtype=np.int64).astype(np.int32)
    return ids, lens


def config_ids(cfg: int, n_vocab: int = 250048):
    """cfg 1: 8x128 seed 1; cfg 2: 256 seqs len U[32,512] seed 2; cfg 4: 512x512 seed 3."""
    hi = min(250000, n_vocab)
    if cfg == 1:
        return ids_fixed(8, 128, seed=1, hi=hi)
    if cfg == 2:
        return ids_ragged(256, 32, 512, seed=2, hi=hi)
    if cfg == 4:
        return ids_fixed(512, 512, seed=3, hi=hi)
    raise ValueError(cfg)


# ---------------------------------------------------------------------------
# isolated MoE operator inputs (BASELINE configs 3 and 5)
# ---------------------------------------------------------------------------

@dataclass
class MoEOpInputs:
    d: int
    n_experts: int
    top_k: int
    ffn: int
    wtype: int
    router_wtype: int
    x: np.ndarray              # [T, d] float32 values exactly representable in bf16
    router_raw: np.ndarray     # router weight blocks [E, row_bytes]
    fc1_raw: np.ndarray        # [E, F, row_bytes(d)]
    fc2_raw: np.ndarray        # [E, d, row_bytes(F)]
    bias: Optional[np.ndarray]  # [d] or None
    router_bias_logits: np.ndarray  # the logit shift b realised through x (see make_moe_op_inputs)
    meta: Dict[str, object] = field(default_factory=dict)


def _round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even) and return as float32."""
    u = x.astype(np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) & np.uint32(0xFFFF0000)).view(np.float32)


def zipf_shift(router_w: np.ndarray, top_k: int, s: float, rng: np.random.Generator, n_cal: int = 8192,
               iters: int = 60) -> np.ndarray:
    """Find logit offsets b so that top-k selection frequencies follow Zipf(s).

    The reference router has no bias term (src/crispembed.cpp:1333), so the skew
    is realised through the input: x = z + W^+ b gives W x = W z + b.
    """
    E, d = router_w.shape
    target = 1.0 / np.arange(1, E + 1, dtype=np.float64) ** s
    target = target / target.sum() * top_k
    z = rng.standard_normal((n_cal, d)).astype(np.float32)
    base = z @ router_w.T  # [n, E]
    b = np.zeros(E, dtype=np.float64)
    for _ in range(iters):
        lg = base + b
        top = np.argpartition(-lg, top_k - 1, axis=1)[:, :top_k]
        cnt = np.bincount(top.reshape(-1), minlength=E) / n_cal
        b += 0.5 * (np.log(target) - np.log(np.maximum(cnt, 1e-6)))
        b -= b.mean()
    return b.astype(np.float32)


_OP_WEIGHTS: Dict[tuple, tuple] = {}  # quantized operator weights of the last few parameter sets


def make_moe_op_inputs(T: int, d: int = 768, n_experts: int = 8, top_k: int = 2, ffn: int = 3072,
                       wtype: int = G.GGML_Q4_K, router_wtype: int = G.GGML_F32, zipf_s: Optional[float] = 1.2,
                       seed: int = 0, with_bias: bool = False) -> MoEOpInputs:
    """Seeded operator inputs: router / expert weights N(0, 0.02) drawn first from
    default_rng(seed), then the activations z ~ N(0, 1) from the same stream.  The
    quantized weights of a parameter set are kept for the next call with the same
    weights (the balanced and Zipf variants of a config share them); the stream is
    resumed from its state after the weights, so every call returns the same
    arrays as a fresh draw."""
    key = (d, n_experts, ffn, wtype, router_wtype, seed, with_bias)
    if key in _OP_WEIGHTS:
        router, router_raw, fc1_raw, fc2_raw, bias, state = _OP_WEIGHTS[key]
        rng = np.random.default_rng(seed)
        rng.bit_generator.state = state
    else:
        rng = np.random.default_rng(seed)
        router = (rng.standard_normal((n_experts, d), dtype=np.float32) * np.float32(0.02))
        fc1 = (rng.standard_normal((n_experts, ffn, d), dtype=np.float32) * np.float32(0.02))
        fc2 = (rng.standard_normal((n_experts, d, ffn), dtype=np.float32) * np.float32(0.02))
        bias = (rng.standard_normal((d,), dtype=np.float32) * np.float32(0.02)) if with_bias else None
        router_raw = quantize(router, router_wtype).view(np.uint8).reshape(n_experts, -1)
        fc1_raw = quantize(fc1, wtype).view(np.uint8).reshape(n_experts, ffn, -1)
        fc2_raw = quantize(fc2, wtype).view(np.uint8).reshape(n_experts, d, -1)
        del fc1, fc2
        if len(_OP_WEIGHTS) >= 2:
            _OP_WEIGHTS.pop(next(iter(_OP_WEIGHTS)))
        _OP_WEIGHTS[key] = (router, router_raw, fc1_raw, fc2_raw, bias, rng.bit_generator.state)
    z = rng.standard_normal((T, d), dtype=np.float32)
    if zipf_s:
        b = zipf_shift(router, top_k, zipf_s, np.random.default_rng(seed + 1))
        m = np.linalg.pinv(router.astype(np.float64)) @ b.astype(np.float64)
        x = z + m.astype(np.float32)[None, :]
    else:
        b = np.zeros(n_experts, dtype=np.float32)
        x = z
    x = _round_bf16(x)
    return MoEOpInputs(d=d, n_experts=n_experts, top_k=top_k, ffn=ffn, wtype=wtype, router_wtype=router_wtype,
                       x=x, router_raw=router_raw, fc1_raw=fc1_raw, fc2_raw=fc2_raw,
                       bias=bias, router_bias_logits=b,
                       meta=dict(T=T, seed=seed, zipf_s=zipf_s, init="N(0,0.02) weights, x=bf16(N(0,1)+W^+ b)"))
