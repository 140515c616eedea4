"""GGUF writer/reader: our files parse with gguf-py's reader and vice versa."""
import numpy as np

from crispembed_b200 import gguf_io as G
from crispembed_b200 import quant, synth


def test_roundtrip_with_gguf_py(tmp_path):
    import gguf
    p = str(tmp_path / "t.gguf")
    w = G.GGUFWriter(p)
    w.add_str("general.architecture", "nomic-bert-moe")
    w.add_u32("bert.hidden_size", 64)
    w.add_f32("bert.layer_norm_eps", 1e-5)
    w.add_str_array("tokenizer.ggml.tokens", ["[PAD]", "abcd", "ü"])
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 64)).astype(np.float32)
    w.add_tensor("a.weight", (64, 3), G.GGML_F32, a)
    w.add_tensor("q.weight", (64, 4), G.GGML_Q8_0, quant.quantize_q8_0(np.tile(a[:1], (4, 1))))
    w.write()
    ours = G.read_gguf(p)
    assert ours.kv["bert.hidden_size"] == 64
    assert ours.kv["tokenizer.ggml.tokens"] == ["[PAD]", "abcd", "ü"]
    assert np.array_equal(ours.raw("a.weight").view(np.float32).reshape(3, 64), a)
    r = gguf.GGUFReader(p)
    names = {t.name: t for t in r.tensors}
    assert set(names) == {"a.weight", "q.weight"}
    assert np.array_equal(np.asarray(names["a.weight"].data).reshape(3, 64), a)
    assert int(names["q.weight"].tensor_type) == G.GGML_Q8_0


def test_synthetic_model_layout(tiny_model):
    g = G.read_gguf(tiny_model)
    spec = synth.tiny_spec()
    assert g.kv["general.architecture"] == "nomic-bert-moe"
    assert g.kv["bert.num_experts"] == spec.n_experts
    t = g.tensors["enc.1.ffn.expert_fc1.weight"]
    assert t.ne == (spec.d, spec.expert_ffn, spec.n_experts) and t.ggml_type == G.GGML_Q8_0
    assert g.tensors["enc.0.ffn.fc1.weight"].ne == (spec.d, spec.ffn)
    assert g.kv["general.fixture_order"].split(",")[0] == "token_embd.weight"
    assert synth.vocab_word(5) == "aaaa" and synth.vocab_word(6) == "aaab"


# ---- the library's own GGUF parser on hostile files (no device: ceb_tokenizer_load
# parses the file before anything else).  Every count, length and offset of a model
# file is untrusted; each case must be refused with the parser's own message, never
# crash or allocate what the file claims.
import struct

import pytest

GT_U32, GT_STR, GT_ARR, GT_U64 = 4, 8, 9, 10


def _s(text):
    b = text.encode()
    return struct.pack("<Q", len(b)) + b


def _file(n_tensors=0, n_kv=0, body=b"", version=3, pad=64):
    return b"GGUF" + struct.pack("<IQQ", version, n_tensors, n_kv) + body + b"\0" * pad


def _tensor(name, dims, ggml_type=0, offset=0):
    return _s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", n) for n in dims) + \
        struct.pack("<IQ", ggml_type, offset)


HOSTILE = {
    "too_small": (b"GGUF\3\0\0\0", "not a GGUF file"),
    "no_magic": (b"NOPE" + b"\0" * 60, "no GGUF magic"),
    "version": (_file(version=7), "unsupported GGUF version"),
    "kv_past_end": (b"GGUF" + struct.pack("<IQQ", 3, 0, 5) + _s("a") + struct.pack("<I", GT_U32), "malformed"),
    "string_longer_than_file": (_file(n_kv=1, body=struct.pack("<Q", 1 << 62) + b"k"), "malformed"),
    "u64_array_count_overflows": (_file(n_kv=1, body=_s("a") + struct.pack("<IIQ", GT_ARR, GT_U64, 1 << 61)),
                                  "malformed"),
    "string_array_count_huge": (_file(n_kv=1, body=_s("a") + struct.pack("<IIQ", GT_ARR, GT_STR, 1 << 40)),
                                "malformed"),
    "tensor_dim_huge": (_file(n_tensors=1, body=_tensor("t", [1 << 62])), "malformed"),
    "tensor_dim_zero": (_file(n_tensors=1, body=_tensor("t", [4, 0])), "malformed"),
    "tensor_rows_overflow": (_file(n_tensors=1, body=_tensor("t", [1 << 39, 1 << 39, 1 << 39])), "outside the file"),
    "tensor_offset_past_end": (_file(n_tensors=1, body=_tensor("t", [4], offset=(1 << 63) + 7)), "outside the file"),
    "tensor_offset_wraps": (_file(n_tensors=1, body=_tensor("t", [4], offset=(1 << 64) - 16)), "outside the file"),
    "tensor_bytes_past_end": (_file(n_tensors=1, body=_tensor("t", [1 << 20])), "outside the file"),
}


@pytest.mark.parametrize("case", sorted(HOSTILE))
def test_hostile_gguf_refused_with_message(tmp_path, case):
    from crispembed_b200 import binding
    blob, msg = HOSTILE[case]
    p = tmp_path / f"{case}.gguf"
    p.write_bytes(blob)
    with pytest.raises(binding.CrispEmbedError, match=msg):
        binding.Tokenizer(str(p), 128)


def test_mutated_gguf_files_load_or_are_refused(tmp_path):
    """Seeded byte mutations of a small valid GGUF (tokenizer keys and two tensors):
    the parser either loads the file or refuses it with an error; it never crashes
    the process or follows a count, length or offset past the file."""
    import ctypes

    from crispembed_b200 import binding
    src = tmp_path / "base.gguf"
    w = G.GGUFWriter(str(src))
    w.add_u32("tokenizer.ggml.type", 0)
    w.add_str_array("tokenizer.ggml.tokens", ["[PAD]", "[CLS]", "[SEP]", "[UNK]", "a", "##b"])
    w.add_u32("tokenizer.ggml.cls_token_id", 1)
    w.add_u32("tokenizer.ggml.sep_token_id", 2)
    w.add_u32("tokenizer.ggml.unknown_token_id", 3)
    w.add_f32_array("tokenizer.ggml.scores", np.zeros(6, np.float32))
    w.add_tensor("a.weight", (64, 2), G.GGML_F32, np.zeros((2, 64), np.float32))
    w.add_tensor("b.weight", (32, 4), G.GGML_Q8_0, quant.quantize(np.ones((4, 32), np.float32), G.GGML_Q8_0))
    w.write()
    base = bytearray(src.read_bytes())
    lib = binding.load_library()
    rng = np.random.default_rng(11)
    p = tmp_path / "m.gguf"
    loaded = refused = 0
    for trial in range(500):
        blob = bytearray(base)
        for _ in range(int(rng.integers(1, 6))):
            pos = int(rng.integers(0, min(len(blob), 512)))  # the header, key-value and tensor-info region
            blob[pos] = int(rng.integers(0, 256))
        if trial % 5 == 0:
            blob = blob[:int(rng.integers(0, len(blob)))]  # truncated
        p.write_bytes(bytes(blob))
        h = lib.ceb_tokenizer_load(str(p).encode(), 64)
        if h:
            loaded += 1
            lib.ceb_tokenizer_free(ctypes.c_void_p(h))
        else:
            refused += 1
    assert loaded + refused == 500 and refused > 0
