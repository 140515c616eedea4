"""ctypes binding of libcrispembed.so (include/crispembed.h, include/ceb_ops.h).

``CrispEmbed`` mirrors the reference's Python class (python/crispembed/_binding.py:
``CrispEmbed(model_path, n_threads).encode(texts)``) for the embedding entry
points this library implements, plus ``encode_ids`` for token-id input.  The
operator-level wrappers (``MoELayer``, ``matmul``, ``pool_l2``) take torch CUDA
tensors purely as device buffers.

There is no CPU fallback: if the CUDA library is missing this module raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional, Sequence, Union

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcrispembed.so")

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K = 0, 1, 8, 12
ACT_F32, ACT_BF16, ACT_F16 = 0, 1, 2

_lib = None


class CrispEmbedError(RuntimeError):
    pass


class _Hparams(ctypes.Structure):
    _fields_ = [
        ("n_vocab", ctypes.c_int32), ("n_max_tokens", ctypes.c_int32), ("n_embd", ctypes.c_int32),
        ("n_head", ctypes.c_int32), ("n_layer", ctypes.c_int32), ("n_intermediate", ctypes.c_int32),
        ("n_output", ctypes.c_int32), ("layer_norm_eps", ctypes.c_float), ("n_experts", ctypes.c_int32),
        ("n_experts_per_tok", ctypes.c_int32),
    ]


def load_library(path: Optional[str] = None):
    """Load (never build) the shared library; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("CRISPEMBED_LIB") or LIB_PATH
    if not os.path.exists(path):
        raise CrispEmbedError(f"{path} not found: build it with `python -m crispembed_b200.build`")
    L = ctypes.CDLL(path)
    vp, cp, ip, fp = ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_float)
    i32p = ctypes.POINTER(ctypes.c_int32)
    sig = {
        "crispembed_init": ([cp, ctypes.c_int], vp),
        "ceb_init_ex": ([cp, ctypes.c_int, ctypes.c_int], vp),
        "crispembed_free": ([vp], None),
        "crispembed_set_dim": ([vp, ctypes.c_int], None),
        "crispembed_set_prefix": ([vp, cp], None),
        "crispembed_get_prefix": ([vp], cp),
        "crispembed_set_gpu_backend": ([cp], None),
        "crispembed_get_hparams": ([vp], ctypes.POINTER(_Hparams)),
        "crispembed_encode": ([vp, cp, ip], fp),
        "crispembed_encode_batch": ([vp, ctypes.POINTER(cp), ctypes.c_int, ip], fp),
        "crispembed_encode_ids_batch": ([vp, i32p, i32p, ctypes.c_int, ip], fp),
        "crispembed_encode_ids_device": ([vp, vp, i32p, ctypes.c_int, vp, ip, vp], ctypes.c_int),
        "crispembed_stream": ([vp], vp),
        "ceb_encode_ids_routes": ([vp, i32p, i32p, ctypes.c_int, vp, vp, vp], ctypes.c_int),
        "ceb_moe_block_count": ([vp], ctypes.c_int),
        "crispembed_has_sparse": ([vp], ctypes.c_int),
        "crispembed_has_colbert": ([vp], ctypes.c_int),
        "crispembed_is_reranker": ([vp], ctypes.c_int),
        "ceb_moe_layer_create": ([ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp,
                                  ctypes.c_int, vp, vp, vp], vp),
        "ceb_moe_layer_free": ([vp], None),
        "ceb_moe_workspace_size": ([vp, ctypes.c_int], ctypes.c_size_t),
        "ceb_moe_ffn": ([vp, vp, ctypes.c_int, ctypes.c_int, vp, vp, vp, vp, vp, vp, ctypes.c_size_t, vp],
                        ctypes.c_int),
        "ceb_moe_ffn_static": ([vp, vp, ctypes.c_int, ctypes.c_int, vp, vp], ctypes.c_int),
        "ceb_moe_workspace_routing": ([vp, ctypes.c_int, vp, ctypes.POINTER(vp), ctypes.POINTER(vp),
                                       ctypes.POINTER(vp), ctypes.POINTER(vp)], ctypes.c_int),
        "ceb_gguf_dequantize": ([ctypes.c_int, vp, ctypes.c_int64, ctypes.c_int64, vp], ctypes.c_int),
        "ceb_ep_create": ([ctypes.c_int] * 7, vp),
        "ceb_ep_ipc_handle": ([vp, vp], ctypes.c_int),
        "ceb_ep_connect": ([vp, vp], ctypes.c_int),
        "ceb_ep_set_timeout_ms": ([vp, ctypes.c_int], None),
        "ceb_ep_free": ([vp], None),
        "ceb_ep_attach": ([vp, vp], ctypes.c_int),
        "ceb_moe_ffn_ep": ([vp, vp, vp, ctypes.c_int, ctypes.c_int, vp, vp, ctypes.c_size_t, vp], ctypes.c_int),
        "ceb_moe_route_ln": ([vp, vp, vp, ctypes.c_int, vp, vp, ctypes.c_float, vp, vp, vp, vp, vp, vp,
                              ctypes.c_size_t, vp], ctypes.c_int),
        "ceb_pool_l2": ([vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, vp], ctypes.c_int),
        "ceb_tokenizer_load": ([ctypes.c_char_p, ctypes.c_int], vp),
        "ceb_tokenizer_encode": ([vp, ctypes.c_char_p, vp, ctypes.c_int], ctypes.c_int),
        "ceb_tokenizer_kind_of": ([vp], ctypes.c_int),
        "ceb_tokenizer_free": ([vp], None),
        "crispembed_encode_tokens": ([vp, ctypes.c_char_p, vp, vp], vp),
        "crispembed_encode_tokens_raw": ([vp, ctypes.c_char_p, vp, vp], vp),
        "crispembed_last_token_ids": ([vp], vp),
        "crispembed_token_str": ([vp, ctypes.c_int32], ctypes.c_char_p),
        "crispembed_tokenizer_kind": ([vp], ctypes.c_int),
        "ceb_attention_forward": ([vp, ctypes.c_int, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, vp],
                                  ctypes.c_int),
        "ceb_matmul": ([ctypes.c_int, vp, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int, vp, ctypes.c_int,
                        ctypes.c_int, vp, vp], ctypes.c_int),
        "ceb_linear_create": ([ctypes.c_int, vp, ctypes.c_int, ctypes.c_int], vp),
        "ceb_linear_forward": ([vp, vp, ctypes.c_int, vp, ctypes.c_int, ctypes.c_int, vp, vp], ctypes.c_int),
        "ceb_linear_free": ([vp], None),
        "ceb_launch_count": ([], ctypes.c_longlong),
        "ceb_profile_enable": ([ctypes.c_int], None),
        "ceb_profile_read": ([ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_double),
                              ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double), ctypes.c_int],
                             ctypes.c_int),
        "ceb_last_error": ([], cp),
        "ceb_sync_check": ([vp], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def last_error() -> str:
    m = load_library().ceb_last_error()
    return m.decode() if m else ""


def _check(rc: int, what: str):
    if rc != 0:
        raise CrispEmbedError(f"{what} failed ({rc}): {last_error()}")


def _stream_ptr(stream) -> Optional[int]:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return int(stream)


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


class CrispEmbed:
    """Text/ids -> L2-normalised embeddings through libcrispembed.so."""

    def __init__(self, model_path: str, n_threads: int = 4, lib_path: Optional[str] = None,
                 reference_arithmetic: bool = False):
        """reference_arithmetic: encode in the reference's CPU arithmetic bit for bit
        (ceb_init_ex with CEB_INIT_REFERENCE_ARITHMETIC; CUDA cores, slow)."""
        self._lib = load_library(lib_path)
        if reference_arithmetic:
            self._ctx = self._lib.ceb_init_ex(model_path.encode(), n_threads, 1)
        else:
            self._ctx = self._lib.crispembed_init(model_path.encode(), n_threads)
        if not self._ctx:
            raise CrispEmbedError(f"Failed to load model: {model_path}: {last_error()}")

    def close(self):
        if getattr(self, "_ctx", None):
            self._lib.crispembed_free(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def hparams(self) -> _Hparams:
        return self._lib.crispembed_get_hparams(self._ctx).contents

    @property
    def n_moe_blocks(self) -> int:
        return int(self._lib.ceb_moe_block_count(self._ctx))

    @property
    def dim(self) -> int:
        h = self.hparams
        return h.n_output if h.n_output > 0 else h.n_embd

    def set_prefix(self, prefix: Optional[str]):
        self._lib.crispembed_set_prefix(self._ctx, (prefix or "").encode())

    def set_dim(self, dim: int):
        self._lib.crispembed_set_dim(self._ctx, int(dim))

    def encode(self, texts: Union[str, List[str]], matryoshka_dim: Optional[int] = None) -> np.ndarray:
        if matryoshka_dim is not None:
            self.set_dim(matryoshka_dim)
        single = isinstance(texts, str)
        if single:
            texts = [texts]
        try:
            dim = ctypes.c_int(0)
            if len(texts) == 1:
                ptr = self._lib.crispembed_encode(self._ctx, texts[0].encode(), ctypes.byref(dim))
            else:
                arr = (ctypes.c_char_p * len(texts))(*(t.encode() for t in texts))
                ptr = self._lib.crispembed_encode_batch(self._ctx, arr, len(texts), ctypes.byref(dim))
            if not ptr:
                raise CrispEmbedError(f"encoding failed: {last_error()}")
            out = np.ctypeslib.as_array(ptr, shape=(len(texts) * dim.value,)).copy().reshape(len(texts), dim.value)
            return out[0] if single else out
        finally:
            if matryoshka_dim is not None:
                self.set_dim(0)

    def encode_tokens(self, text: str, raw: bool = False):
        """Per-token final hidden states [n_tokens, n_embd] (L2-normalised unless raw) and their ids."""
        n = ctypes.c_int(0)
        dim = ctypes.c_int(0)
        fn = self._lib.crispembed_encode_tokens_raw if raw else self._lib.crispembed_encode_tokens
        ptr = fn(self._ctx, text.encode("utf-8"), ctypes.byref(n), ctypes.byref(dim))
        if not ptr:
            raise CrispEmbedError(f"encode_tokens failed: {last_error()}")
        vec = np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)),
                                    shape=(n.value * dim.value,)).copy().reshape(n.value, dim.value)
        ids_ptr = ctypes.cast(self._lib.crispembed_last_token_ids(self._ctx), ctypes.POINTER(ctypes.c_int32))
        ids = np.ctypeslib.as_array(ids_ptr, shape=(n.value,)).copy()
        return vec, ids

    def token_str(self, token_id: int) -> str:
        r = self._lib.crispembed_token_str(self._ctx, int(token_id))
        return r.decode("utf-8", "replace") if r is not None else ""

    @property
    def tokenizer_kind(self) -> int:
        return self._lib.crispembed_tokenizer_kind(self._ctx)

    def attach_ep(self, ep: "ExpertParallel"):
        """Route every MoE block through `ep` (this context keeps only ep's experts)."""
        _check(self._lib.ceb_ep_attach(self._ctx, ep._h), "ceb_ep_attach")
        self._ep = ep  # the exchange must outlive the context's use of it

    def encode_ids(self, ids: np.ndarray, lens: Sequence[int]) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        lens = np.ascontiguousarray(lens, dtype=np.int32)
        dim = ctypes.c_int(0)
        i32p = ctypes.POINTER(ctypes.c_int32)
        ptr = self._lib.crispembed_encode_ids_batch(self._ctx, ids.ctypes.data_as(i32p), lens.ctypes.data_as(i32p),
                                                    len(lens), ctypes.byref(dim))
        if not ptr:
            raise CrispEmbedError(f"encode_ids failed: {last_error()}")
        return np.ctypeslib.as_array(ptr, shape=(len(lens) * dim.value,)).copy().reshape(len(lens), dim.value)

    def encode_ids_routes(self, ids: np.ndarray, lens: Sequence[int]):
        """(embeddings [n_seqs, dim], expert ids [n_moe, M, top_k], router logits
        [n_moe, M, n_experts]) of one synchronous encode (ceb_encode_ids_routes)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        lens = np.ascontiguousarray(lens, dtype=np.int32)
        hp = self.hparams
        M, E, K = int(lens.sum()), int(hp.n_experts), int(hp.n_experts_per_tok)
        n_moe = self.n_moe_blocks
        emb = np.empty((len(lens), self.dim), dtype=np.float32)
        rid = np.empty((n_moe, M, max(K, 1)), dtype=np.int32)
        lg = np.empty((n_moe, M, max(E, 1)), dtype=np.float32)
        i32p = ctypes.POINTER(ctypes.c_int32)
        rc = self._lib.ceb_encode_ids_routes(self._ctx, ids.ctypes.data_as(i32p), lens.ctypes.data_as(i32p), len(lens),
                                             emb.ctypes.data, rid.ctypes.data, lg.ctypes.data)
        _check(rc, "encode_ids_routes")
        return emb, rid, lg

    def encode_ids_device(self, d_ids, lens: np.ndarray, d_out, stream=None) -> int:
        """d_ids: int32 CUDA tensor, d_out: float32 CUDA tensor [n_seqs, dim]."""
        lens = np.ascontiguousarray(lens, dtype=np.int32)
        dim = ctypes.c_int(0)
        rc = self._lib.crispembed_encode_ids_device(self._ctx, d_ids.data_ptr(),
                                                    lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(lens),
                                                    d_out.data_ptr(), ctypes.byref(dim), _stream_ptr(stream))
        _check(rc, "encode_ids_device")
        return dim.value


class MoELayer:
    """One MoE feed-forward block on the device (ceb_moe_layer_create / ceb_moe_ffn)."""

    def __init__(self, d: int, n_experts: int, top_k: int, ffn: int, router_type: int, router_raw: np.ndarray,
                 expert_type: int, fc1_raw: np.ndarray, fc2_raw: np.ndarray, bias: Optional[np.ndarray] = None):
        self._lib = load_library()
        self.d, self.n_experts, self.top_k, self.ffn = d, n_experts, top_k, ffn
        keep = [np.ascontiguousarray(router_raw), np.ascontiguousarray(fc1_raw), np.ascontiguousarray(fc2_raw)]
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self._h = self._lib.ceb_moe_layer_create(d, n_experts, top_k, ffn, router_type, keep[0].ctypes.data,
                                                 expert_type, keep[1].ctypes.data, keep[2].ctypes.data,
                                                 None if b is None else b.ctypes.data)
        if not self._h:
            raise CrispEmbedError(f"ceb_moe_layer_create failed: {last_error()}")

    def close(self):
        if getattr(self, "_h", None):
            self._lib.ceb_moe_layer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward_static(self, x, y, stream=None):
        """ceb_moe_ffn_static: the library's own fixed scratch, no device allocation."""
        import torch
        act = {torch.float32: ACT_F32, torch.bfloat16: ACT_BF16, torch.float16: ACT_F16}[x.dtype]
        _check(self._lib.ceb_moe_ffn_static(self._h, x.data_ptr(), act, x.shape[0], y.data_ptr(), _stream_ptr(stream)),
               "ceb_moe_ffn_static")

    def routing(self, workspace, n_tokens: int):
        """(ids, weights, slot_pos, offsets) of the last call on `workspace` (a uint8
        CUDA tensor), as host numpy arrays (ceb_moe_workspace_routing)."""
        import torch
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        _check(self._lib.ceb_moe_workspace_routing(self._h, n_tokens, workspace.data_ptr(),
                                                   *[ctypes.byref(p) for p in ptrs]), "ceb_moe_workspace_routing")
        K, E = self.top_k, self.n_experts
        out = []
        for p, n, dt in ((ptrs[0], n_tokens * K, torch.int32), (ptrs[1], n_tokens * K, torch.float32),
                         (ptrs[2], n_tokens * K, torch.int32), (ptrs[3], E + 1, torch.int32)):
            off = p.value - workspace.data_ptr()
            out.append(workspace[off:off + 4 * n].view(dt).cpu().numpy())
        ids, w, sp, offsets = out
        return ids.reshape(n_tokens, K), w.reshape(n_tokens, K), sp.reshape(n_tokens, K), offsets

    def workspace_size(self, n_tokens: int) -> int:
        return int(self._lib.ceb_moe_workspace_size(self._h, n_tokens))

    def forward(self, x, y, workspace, ids=None, weights=None, counts=None, logits=None, stream=None):
        import torch
        act = {torch.float32: ACT_F32, torch.bfloat16: ACT_BF16, torch.float16: ACT_F16}[x.dtype]
        rc = self._lib.ceb_moe_ffn(self._h, x.data_ptr(), act, x.shape[0], y.data_ptr(), _ptr(ids), _ptr(weights),
                                   _ptr(counts), _ptr(logits), workspace.data_ptr(), workspace.numel(),
                                   _stream_ptr(stream))
        _check(rc, "ceb_moe_ffn")

    def forward_ep(self, ep: "ExpertParallel", x, y, workspace, stream=None):
        """ceb_moe_ffn_ep: this rank's tokens through the expert-parallel exchange."""
        import torch
        act = {torch.float32: ACT_F32, torch.bfloat16: ACT_BF16, torch.float16: ACT_F16}[x.dtype]
        rc = self._lib.ceb_moe_ffn_ep(self._h, ep._h, x.data_ptr(), act, x.shape[0], y.data_ptr(),
                                      workspace.data_ptr(), workspace.numel(), _stream_ptr(stream))
        _check(rc, "ceb_moe_ffn_ep")

    def route_ln(self, res, y, out, workspace, gamma=None, beta=None, eps=1e-5, out16=None, ids=None, weights=None,
                 logits=None, stream=None):
        """ceb_moe_route_ln: out = LN(res + y), and the router on the normalised rows in the same pass."""
        rc = self._lib.ceb_moe_route_ln(self._h, res.data_ptr(), y.data_ptr(), res.shape[0], _ptr(gamma), _ptr(beta),
                                        float(eps), out.data_ptr(), _ptr(out16), _ptr(ids), _ptr(weights),
                                        _ptr(logits), workspace.data_ptr(), workspace.numel(), _stream_ptr(stream))
        _check(rc, "ceb_moe_route_ln")


EP_HANDLE_BYTES = 64


class ExpertParallel:
    """Expert-parallel exchange of one rank (ceb_ep_create / _ipc_handle / _connect).

    `connect(handles)` takes every rank's handle bytes in rank order; see
    crispembed_b200.dist.connect_expert_parallel for the torch.distributed form."""

    def __init__(self, rank: int, world: int, n_experts: int, top_k: int, d: int, ffn: int, max_local_tokens: int):
        self._lib = load_library()
        self.rank, self.world = rank, world
        self._h = self._lib.ceb_ep_create(rank, world, n_experts, top_k, d, ffn, max_local_tokens)
        if not self._h:
            raise CrispEmbedError(f"ceb_ep_create failed: {last_error()}")

    def handle(self) -> bytes:
        buf = ctypes.create_string_buffer(EP_HANDLE_BYTES)
        _check(self._lib.ceb_ep_ipc_handle(self._h, buf), "ceb_ep_ipc_handle")
        return buf.raw

    def connect(self, handles: Sequence[bytes]):
        if len(handles) != self.world or any(len(h) != EP_HANDLE_BYTES for h in handles):
            raise CrispEmbedError("connect: one handle of EP_HANDLE_BYTES per rank expected")
        blob = ctypes.create_string_buffer(b"".join(handles), EP_HANDLE_BYTES * self.world)
        _check(self._lib.ceb_ep_connect(self._h, blob), "ceb_ep_connect")

    def set_timeout_ms(self, ms: int):
        self._lib.ceb_ep_set_timeout_ms(self._h, int(ms))

    def close(self):
        if getattr(self, "_h", None):
            self._lib.ceb_ep_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Linear:
    """Device-resident linear layer (ceb_linear_create / ceb_linear_forward)."""

    def __init__(self, w_type: int, w_raw: np.ndarray, n_out: int, k: int):
        self._lib = load_library()
        self.n_out, self.k = n_out, k
        w_raw = np.ascontiguousarray(w_raw)
        self._h = self._lib.ceb_linear_create(w_type, w_raw.ctypes.data, n_out, k)
        if not self._h:
            raise CrispEmbedError(f"ceb_linear_create failed: {last_error()}")

    def __call__(self, x, out=None, bias=None, gelu=False, out_f16=False, stream=None):
        import torch
        if out is None:
            out = torch.empty((x.shape[0], self.n_out), dtype=torch.float16 if out_f16 else torch.float32,
                              device=x.device)
        _check(self._lib.ceb_linear_forward(self._h, x.data_ptr(), x.shape[0], _ptr(bias), int(gelu), int(out_f16),
                                            out.data_ptr(), _stream_ptr(stream)), "ceb_linear_forward")
        return out

    def close(self):
        if getattr(self, "_h", None):
            self._lib.ceb_linear_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def matmul(w_type: int, w_raw: np.ndarray, n_out: int, k: int, x, bias=None, gelu=False, out_f16=False, stream=None):
    import torch
    lib = load_library()
    out = torch.empty((x.shape[0], n_out), dtype=torch.float16 if out_f16 else torch.float32, device=x.device)
    w_raw = np.ascontiguousarray(w_raw)
    rc = lib.ceb_matmul(w_type, w_raw.ctypes.data, n_out, k, x.data_ptr(), x.shape[0], _ptr(bias), int(gelu),
                        int(out_f16), out.data_ptr(), _stream_ptr(stream))
    _check(rc, "ceb_matmul")
    return out


def pool_l2(hidden, cu_seqlens, out_dim: Optional[int] = None, stream=None):
    import torch
    lib = load_library()
    n = cu_seqlens.numel() - 1
    d = hidden.shape[1]
    od = out_dim or d
    out = torch.empty((n, od), dtype=torch.float32, device=hidden.device)
    _check(lib.ceb_pool_l2(hidden.data_ptr(), cu_seqlens.data_ptr(), n, d, od, out.data_ptr(), _stream_ptr(stream)),
           "ceb_pool_l2")
    return out


def attention(qkv, cu_seqlens, n_head: int, max_len: Optional[int] = None, stream=None):
    """softmax(Q K^T / sqrt(64)) V per sequence and head; qkv [rows, 3d] fp16 on the device."""
    import torch
    lib = load_library()
    rows, d3 = qkv.shape
    d = d3 // 3
    n = cu_seqlens.numel() - 1
    if max_len is None:
        max_len = int((cu_seqlens[1:] - cu_seqlens[:-1]).max().item()) if n else 0
    out = torch.empty((rows, d), dtype=torch.float16, device=qkv.device)
    _check(lib.ceb_attention_forward(qkv.data_ptr(), rows, cu_seqlens.data_ptr(), n, max_len, d, n_head,
                                     out.data_ptr(), _stream_ptr(stream)), "ceb_attention_forward")
    return out


def gguf_dequantize(ggml_type: int, raw: np.ndarray, n_rows: int, k: int) -> np.ndarray:
    """ceb_gguf_dequantize: host decoding of n_rows GGUF rows of k values to fp32."""
    raw = np.ascontiguousarray(raw)
    out = np.empty((n_rows, k), dtype=np.float32)
    _check(load_library().ceb_gguf_dequantize(int(ggml_type), raw.ctypes.data, int(n_rows), int(k),
                                              out.ctypes.data), "ceb_gguf_dequantize")
    return out


class Tokenizer:
    """The text tokenizer of a GGUF (WordPiece or SentencePiece Unigram), without a device."""

    def __init__(self, gguf_path: str, max_tokens: int = 512):
        self._lib = load_library()
        self._h = self._lib.ceb_tokenizer_load(gguf_path.encode(), int(max_tokens))
        if not self._h:
            raise CrispEmbedError(f"ceb_tokenizer_load failed: {last_error()}")
        self.max_tokens = int(max_tokens)

    @property
    def kind(self) -> int:
        return self._lib.ceb_tokenizer_kind_of(self._h)

    def encode(self, text: str):
        cap = self.max_tokens
        buf = (ctypes.c_int32 * cap)()
        n = self._lib.ceb_tokenizer_encode(self._h, text.encode("utf-8"), buf, cap)
        if n < 0:
            raise CrispEmbedError(f"ceb_tokenizer_encode failed: {last_error()}")
        return [int(buf[i]) for i in range(min(n, cap))]

    def close(self):
        if self._h:
            self._lib.ceb_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sync_check(stream=None):
    _check(load_library().ceb_sync_check(_stream_ptr(stream)), "device check")


PROFILE_CATEGORIES = ("gemm", "attention", "routing", "rowwise", "exchange", "exchange_wait", "moe_gemm")


def launch_count() -> int:
    return int(load_library().ceb_launch_count())


def profile_enable(on: bool = True):
    load_library().ceb_profile_enable(int(on))


def profile_read() -> dict:
    n = len(PROFILE_CATEGORIES)
    L = (ctypes.c_longlong * n)()
    ms, fl, by = (ctypes.c_double * n)(), (ctypes.c_double * n)(), (ctypes.c_double * n)()
    _check(load_library().ceb_profile_read(L, ms, fl, by, n), "ceb_profile_read")
    return {c: dict(launches=int(L[i]), ms=float(ms[i]), flops=float(fl[i]), bytes=float(by[i]))
            for i, c in enumerate(PROFILE_CATEGORIES)}
