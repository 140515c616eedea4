"""A small SentencePiece Unigram model trained here (sentencepiece package) and
its GGUF tokenizer keys, shared by the tokenizer tests.

Normalisation is the identity (or nmt_nfkc for the normalisation tests) and
repeated spaces are kept, so the text the model segments is " " + text with
spaces as U+2581 -- the input the reference's SentencePiece tokenizer
(src/tokenizer_spm.cpp) segments.
"""
import os

import numpy as np

WORDS = ("embedding model vector space token query passage search mixture expert router gate layer "
         "attention sequence batch tensor kernel memory bandwidth latency throughput accuracy the a of "
         "to and in is for with on by at from as encoder decoder pooling normalise cosine similarity").split()


def _pseudo_words(n: int = 400, seed: int = 1):
    """Seeded syllable words, so the model has to learn real subword pieces."""
    rng = np.random.default_rng(seed)
    cons, vows = "bdfgklmnprstvz", "aeiou"
    out = []
    for _ in range(n):
        k = int(rng.integers(2, 5))
        out.append("".join(cons[int(rng.integers(len(cons)))] + vows[int(rng.integers(len(vows)))] for _ in range(k)))
    return out


WORDS = WORDS + _pseudo_words()


def corpus(n_lines: int = 4000, seed: int = 0):
    rng = np.random.default_rng(seed)
    lines = []
    for _ in range(n_lines):
        k = int(rng.integers(3, 12))
        lines.append(" ".join(WORDS[int(i)] for i in rng.integers(0, len(WORDS), size=k)))
    return lines


EXTRA_LINES = ["1 2 3 10 12 2026 ... a.b fi fl ( ) kg IV", "model 1... search 2 ... end. kg"]


def train(tmpdir: str, vocab_size: int = 300, rule: str = "identity"):
    """rule "nmt_nfkc": the normaliser XLM-R-family models declare (the corpus gains
    a few lines with digits and dots so its replacements have pieces)."""
    import sentencepiece as spm
    txt = os.path.join(tmpdir, "corpus.txt")
    lines = corpus() + (EXTRA_LINES * 50 if rule != "identity" else [])
    with open(txt, "w") as f:
        f.write("\n".join(lines) + "\n")
    prefix = os.path.join(tmpdir, "spm")
    spm.SentencePieceTrainer.train(
        input=txt, model_prefix=prefix, vocab_size=vocab_size, model_type="unigram",
        normalization_rule_name=rule, add_dummy_prefix=True, remove_extra_whitespaces=False,
        character_coverage=1.0, unk_id=0, bos_id=1, eos_id=2, pad_id=3, num_threads=1, minloglevel=2,
        hard_vocab_limit=False)
    return spm.SentencePieceProcessor(model_file=prefix + ".model")


def write_keys(w, sp, model_str: str = "t5"):
    """GGUF keys of the sentencepiece model, as a llama.cpp-style export writes them."""
    n = sp.get_piece_size()
    w.add_str("tokenizer.ggml.model", model_str)
    w.add_str_array("tokenizer.ggml.tokens", [sp.id_to_piece(i) for i in range(n)])
    w.add_f32_array("tokenizer.ggml.scores", [float(sp.get_score(i)) for i in range(n)])
    w.add_u32("tokenizer.ggml.unknown_token_id", sp.unk_id())
    w.add_u32("tokenizer.ggml.bos_token_id", sp.bos_id())
    w.add_u32("tokenizer.ggml.eos_token_id", sp.eos_id())
    w.add_u32("tokenizer.ggml.padding_token_id", sp.pad_id())
