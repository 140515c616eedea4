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
