"""Host tokenizers of the text ABI (crispembed_b200/csrc/tokenizer.cpp), no device.

SentencePiece Unigram is checked against the sentencepiece package on a model
trained here (tests/spm_fixture.py): the segmentation between <s> and </s> must
be identical.  The family decision follows the reference's table
(src/tokenizer.h:37-52); byte fallback and wrapping follow
src/tokenizer_spm.cpp.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(__file__))
import spm_fixture  # noqa: E402

from crispembed_b200 import binding  # noqa: E402
from crispembed_b200 import gguf_io as G  # noqa: E402


def _gguf(path, fill):
    w = G.GGUFWriter(str(path))
    fill(w)
    w.write()
    return str(path)


@pytest.fixture(scope="module")
def spm_model(tmp_path_factory):
    d = tmp_path_factory.mktemp("spm")
    sp = spm_fixture.train(str(d))
    path = _gguf(d / "tok.gguf", lambda w: spm_fixture.write_keys(w, sp))
    return sp, path


def test_sentencepiece_segmentation_matches_sentencepiece(spm_model):
    sp, path = spm_model
    tok = binding.Tokenizer(path, max_tokens=512)
    assert tok.kind == 2
    rng = np.random.default_rng(11)
    texts = spm_fixture.corpus(200, seed=3)
    # unseen combinations, repeated and edge spaces, glued words
    texts += ["a", "the", "  two  spaces", "trailing ", "embeddingmodel", "routergatelayer expert",
              "kernel" * 7, " ".join(spm_fixture.WORDS[:80])]
    for _ in range(50):
        k = int(rng.integers(1, 6))
        texts.append("".join(spm_fixture.WORDS[int(i)] for i in rng.integers(0, len(spm_fixture.WORDS), size=k)))
    for t in texts:
        ids = tok.encode(t)
        assert ids[0] == sp.bos_id() and ids[-1] == sp.eos_id()
        assert ids[1:-1] == sp.encode(t), t


def test_sentencepiece_empty_text_is_the_space_marker(spm_model):
    """The reference prepends a space before replacing spaces by U+2581, so an empty
    text is the single '▁' piece between <s> and </s> (the sentencepiece package
    itself returns no pieces for an empty input)."""
    sp, path = spm_model
    tok = binding.Tokenizer(path)
    assert tok.encode("") == [sp.bos_id(), sp.piece_to_id("▁"), sp.eos_id()]


def test_sentencepiece_truncates_and_keeps_eos(spm_model):
    sp, path = spm_model
    tok = binding.Tokenizer(path, max_tokens=16)
    text = " ".join(spm_fixture.WORDS[:60])
    ids = tok.encode(text)
    assert len(ids) == 16 and ids[0] == sp.bos_id() and ids[-1] == sp.eos_id()
    full = sp.encode(text)
    assert ids[1:-1] == full[:14]


def test_sentencepiece_byte_fallback(tmp_path):
    """Bytes no piece covers: '<0xXX>' pieces when present, else <unk>, one per byte."""
    pieces = ["<unk>", "<s>", "</s>", "▁", "▁a", "b", "<0xC3>", "<0xA9>"]
    scores = [0.0, 0.0, 0.0, -2.0, -1.0, -1.5, 0.0, 0.0]

    def fill(w):
        w.add_str("tokenizer.ggml.model", "llama")
        w.add_str_array("tokenizer.ggml.tokens", pieces)
        w.add_f32_array("tokenizer.ggml.scores", scores)
        w.add_u32("tokenizer.ggml.unknown_token_id", 0)
        w.add_u32("tokenizer.ggml.bos_token_id", 1)
        w.add_u32("tokenizer.ggml.eos_token_id", 2)

    tok = binding.Tokenizer(_gguf(tmp_path / "b.gguf", fill))
    assert tok.kind == 2
    # " abé" -> [▁a][b][<0xC3>][<0xA9>]; "é" is the two bytes C3 A9
    assert tok.encode("abé") == [1, 4, 5, 6, 7, 2]
    # a byte with no <0xXX> piece becomes <unk>
    assert tok.encode("a!") == [1, 4, 0, 2]


def test_sentencepiece_picks_the_max_score_segmentation(tmp_path):
    pieces = ["<unk>", "<s>", "</s>", "▁ab", "▁a", "bc", "c", "▁"]
    # "▁abc": [▁ab][c] = -3 -1.5 = -4.5 vs [▁a][bc] = -1 -1 = -2
    scores = [0.0, 0.0, 0.0, -3.0, -1.0, -1.0, -1.5, -4.0]

    def fill(w):
        w.add_str("tokenizer.ggml.model", "t5")
        w.add_str_array("tokenizer.ggml.tokens", pieces)
        w.add_f32_array("tokenizer.ggml.scores", scores)

    tok = binding.Tokenizer(_gguf(tmp_path / "v.gguf", fill))
    assert tok.encode("abc")[1:-1] == [4, 5]


@pytest.mark.parametrize("keys,n_vocab,kind", [
    ({"type": 0}, 120000, 1),           # an explicit WordPiece type is final, even for a big vocab
    ({"type": 2}, 100, 2),
    ({"model": "t5"}, 100, 2),
    ({"model": "unigram"}, 100, 2),
    ({"model": "bert"}, 120000, 1),     # the model string overrides the size heuristic
    ({"model": "gpt2"}, 100, 3),
    ({}, 120000, 2),                    # neither key: vocabularies above 100k are SentencePiece
    ({}, 1000, 1),
])
def test_tokenizer_family_decision(tmp_path, keys, n_vocab, kind):
    def fill(w):
        if "type" in keys:
            w.add_u32("tokenizer.ggml.type", keys["type"])
        if "model" in keys:
            w.add_str("tokenizer.ggml.model", keys["model"])
        w.add_str_array("tokenizer.ggml.tokens", [f"t{i}" for i in range(n_vocab)])

    tok = binding.Tokenizer(_gguf(tmp_path / "f.gguf", fill))
    assert tok.kind == kind


def test_bpe_family_is_rejected_loudly(tmp_path):
    def fill(w):
        w.add_str("tokenizer.ggml.model", "gpt2")
        w.add_str_array("tokenizer.ggml.tokens", ["a", "b"])

    tok = binding.Tokenizer(_gguf(tmp_path / "g.gguf", fill))
    with pytest.raises(binding.CrispEmbedError, match="BPE"):
        tok.encode("ab")


def test_wordpiece_greedy_longest_match(tmp_path):
    vocab = ["[PAD]", "[CLS]", "[SEP]", "[UNK]", "un", "##aff", "##able", "aff", ",", "hello", "##s"]

    def fill(w):
        w.add_u32("tokenizer.ggml.type", 0)
        w.add_str_array("tokenizer.ggml.tokens", vocab)
        w.add_u32("tokenizer.ggml.cls_token_id", 1)
        w.add_u32("tokenizer.ggml.sep_token_id", 2)
        w.add_u32("tokenizer.ggml.unknown_token_id", 3)

    tok = binding.Tokenizer(_gguf(tmp_path / "w.gguf", fill))
    assert tok.kind == 1
    assert tok.encode("Unaffable, hellos") == [1, 4, 5, 6, 8, 9, 10, 2]
    assert tok.encode("zzz") == [1, 3, 2]


@pytest.fixture(scope="module")
def spm_nfkc_model(tmp_path_factory):
    d = tmp_path_factory.mktemp("spm_nfkc")
    sp = spm_fixture.train(str(d), rule="nmt_nfkc")
    path = _gguf(d / "tok.gguf", lambda w: spm_fixture.write_keys(w, sp))
    return sp, path


NFKC_TEXTS = ["ｍｏｄｅｌ １２",   # fullwidth "model 12"
              "search… end",                              # ellipsis -> "..."
              "model　search",                             # ideographic space -> word boundary
              "ﬁ ﬂ",                                 # ligatures fi fl
              "① Ⅱ ㎏",                          # circled 1, roman II, kg
              "tab\there\nnew line",                           # \t \n -> spaces
              "plain ascii stays the same"]


@pytest.mark.parametrize("text", NFKC_TEXTS)
def test_sentencepiece_nmt_nfkc_normalisation_matches_sentencepiece(spm_nfkc_model, text):
    """The nmt_nfkc charsmap (fullwidth forms, U+2026, U+3000, ligatures, enclosed
    and compatibility characters, control characters) is applied before
    segmentation, as the reference's embedding path does (src/tokenizer_spm.cpp:57-70):
    the ids equal sentencepiece's for a model trained with that rule."""
    sp, path = spm_nfkc_model
    tok = binding.Tokenizer(path, max_tokens=512)
    ids = tok.encode(text)
    assert ids[1:-1] == sp.encode(text), (text, ids, sp.encode(text))


def _vocab_gguf(path, model, tokens, extra=b""):
    import struct

    def s(t):
        b = t.encode()
        return struct.pack("<Q", len(b)) + b
    kvs = [s("tokenizer.ggml.model") + struct.pack("<I", 8) + s(model),
           s("tokenizer.ggml.tokens") + struct.pack("<IIQ", 9, 8, len(tokens)) + b"".join(s(t) for t in tokens)]
    n_kv = len(kvs)
    if extra:
        kvs.append(extra)
        n_kv += 1
    path.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 0, n_kv) + b"".join(kvs) + b"\0" * 64)


def test_special_ids_outside_the_vocabulary_refused(tmp_path):
    """A special id the encoder would emit must name a piece (ids index the token
    table): SentencePiece bos / unknown and WordPiece cls / sep / unknown ids past
    the vocabulary are refused when the tokenizer loads."""
    import struct

    from crispembed_b200 import binding
    p = tmp_path / "spm.gguf"
    key = b"".join([struct.pack("<Q", len(b"tokenizer.ggml.bos_token_id")), b"tokenizer.ggml.bos_token_id"])
    _vocab_gguf(p, "llama", ["<unk>", "<s>", "</s>", "▁h"], extra=key + struct.pack("<II", 4, 77777))
    with pytest.raises(binding.CrispEmbedError, match="bos token id 77777"):
        binding.Tokenizer(str(p), 128)
    p2 = tmp_path / "wpm.gguf"  # WordPiece defaults cls 101 / sep 102 / unk 100 on a 5-piece vocabulary
    _vocab_gguf(p2, "bert", ["[PAD]", "a", "[UNK]", "[CLS]", "[SEP]"])
    with pytest.raises(binding.CrispEmbedError, match="cls token id 101"):
        binding.Tokenizer(str(p2), 128)
    p3 = tmp_path / "spm_ok.gguf"  # defaults bos 0 / eos 2 / unk 3 all name pieces
    _vocab_gguf(p3, "llama", ["<unk>", "<s>", "</s>", "▁h"])
    binding.Tokenizer(str(p3), 128)  # loads


@pytest.mark.parametrize("family", ["sentencepiece", "wordpiece"])
def test_tokenizers_on_arbitrary_bytes(tmp_path, spm_model, family):
    """Seeded random byte strings (broken UTF-8, control bytes, long runs) through the
    C entry point: every call returns, truncates to max_tokens and emits only ids
    of the vocabulary."""
    import ctypes
    if family == "sentencepiece":
        sp, path = spm_model
        n_vocab = sp.get_piece_size()
    else:
        vocab = ["[PAD]", "[CLS]", "[SEP]", "[UNK]", "un", "##aff", "##able", "aff", ",", "hello", "##s"]

        def fill(w):
            w.add_u32("tokenizer.ggml.type", 0)
            w.add_str_array("tokenizer.ggml.tokens", vocab)
            w.add_u32("tokenizer.ggml.cls_token_id", 1)
            w.add_u32("tokenizer.ggml.sep_token_id", 2)
            w.add_u32("tokenizer.ggml.unknown_token_id", 3)
        path = _gguf(tmp_path / "w.gguf", fill)
        n_vocab = len(vocab)
    cap = 64
    tok = binding.Tokenizer(path, max_tokens=cap)
    buf = (ctypes.c_int32 * cap)()
    rng = np.random.default_rng(7)
    for trial in range(400):
        size = int(rng.integers(0, 300))
        raw = bytes(rng.integers(1, 256, size=size, dtype=np.uint8))  # no NUL: a C string
        if trial % 4 == 0:
            raw = (b"\xe2\x96\x81" * size)[:size] + raw  # runs of the space marker's bytes
        n = tok._lib.ceb_tokenizer_encode(tok._h, raw, buf, cap)
        assert 0 < n <= cap, (trial, n)
        assert all(0 <= buf[i] < n_vocab for i in range(n)), trial
