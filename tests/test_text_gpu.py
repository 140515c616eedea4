"""The text ABI end to end with a SentencePiece Unigram model, and the per-token
entry points (src/crispembed.cpp:3272-3393), against the oracle.

The model is the tiny NomicBERT-MoE of the other tests with a SentencePiece
vocabulary trained here (tests/spm_fixture.py) in place of the synthetic
WordPiece one.  Per-token outputs are the oracle's last-layer hidden states,
L2-normalised per token for encode_tokens and as they are for _raw.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(__file__))
import spm_fixture  # noqa: E402

from crispembed_b200 import synth  # noqa: E402

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAXABS = 2e-3
TEXTS = ["embedding model for passage search", "the router gate of a mixture of experts layer",
         "kernel", "throughput latency and memory bandwidth of the encoder"]


@pytest.fixture(scope="module")
def spm_setup(tmp_path_factory):
    d = tmp_path_factory.mktemp("spm_model")
    sp = spm_fixture.train(str(d))
    path = str(d / "tiny_spm.gguf")
    synth.write_model(path, synth.tiny_spec(n_vocab=sp.get_piece_size()),
                      tokenizer=lambda w: spm_fixture.write_keys(w, sp))
    return sp, path


@pytest.fixture(scope="module")
def model(cuda, spm_setup):
    from crispembed_b200 import binding
    m = binding.CrispEmbed(spm_setup[1])
    yield m
    m.close()


def _ids(sp, text):
    return [sp.bos_id()] + sp.encode(text) + [sp.eos_id()]


def test_tokenizer_kind_and_pieces(model, spm_setup):
    sp, _ = spm_setup
    assert model.tokenizer_kind == 2
    for i in (0, 1, 2, 10, sp.get_piece_size() - 1):
        assert model.token_str(i) == sp.id_to_piece(i)
    assert model.token_str(sp.get_piece_size()) == ""


def test_text_equals_ids(model, spm_setup):
    """Text in = the same embeddings as the sentencepiece ids in."""
    sp, _ = spm_setup
    emb = model.encode(TEXTS)
    ids = [_ids(sp, t) for t in TEXTS]
    lens = np.array([len(x) for x in ids], dtype=np.int32)
    ref = model.encode_ids(np.concatenate(ids).astype(np.int32), lens)
    assert np.array_equal(emb, ref)


def test_text_matches_oracle(model, spm_setup, oracle):
    sp, path = spm_setup
    emb = model.encode(TEXTS)
    ids = [_ids(sp, t) for t in TEXTS]
    lens = np.array([len(x) for x in ids], dtype=np.int64)
    ref = oracle.encode(oracle.load_model(path), np.concatenate(ids), lens, oracle.GGML)
    cos = (emb.astype(np.float64) * ref).sum(1) / (np.linalg.norm(emb, axis=1) * np.linalg.norm(ref, axis=1))
    assert cos.min() >= COS_MIN
    assert np.abs(emb - ref).max() <= MAXABS


@pytest.mark.parametrize("raw", [False, True])
def test_encode_tokens_matches_oracle(model, spm_setup, oracle, raw):
    sp, path = spm_setup
    text = TEXTS[1]
    vec, ids = model.encode_tokens(text, raw=raw)
    want = _ids(sp, text)
    assert list(ids) == want
    dump = {}
    om = oracle.load_model(path)
    oracle.encode(om, np.array(want), np.array([len(want)]), oracle.GGML, dump=dump)
    hid = dump[f"layer_{om.hp['n_layer'] - 1}"].astype(np.float64)
    if not raw:
        hid = hid / np.sqrt(np.maximum((hid * hid).sum(1, keepdims=True), 1e-12))
        assert np.allclose(np.linalg.norm(vec, axis=1), 1.0, atol=1e-5)
    assert vec.shape == hid.shape
    cos = (vec * hid).sum(1) / (np.linalg.norm(vec, axis=1) * np.linalg.norm(hid, axis=1))
    assert cos.min() >= COS_MIN
    scale = 1.0 if not raw else max(1.0, float(np.abs(hid).max()))
    assert np.abs(vec - hid).max() <= MAXABS * scale


def test_prefix_is_tokenized_with_the_text(model, spm_setup):
    sp, _ = spm_setup
    model.set_prefix("query ")
    try:
        _, ids = model.encode_tokens("kernel memory")
    finally:
        model.set_prefix("")
    assert list(ids) == _ids(sp, "query kernel memory")
