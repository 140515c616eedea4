"""End-to-end embeddings through the C ABI against the ggml-faithful oracle.

Bar: cosine >= 0.9999 and max-abs <= 2e-3 per embedding
vector; repeat encodes bit-identical (reference tests/test_moe_parity.py:149-154).
"""
import numpy as np
import pytest

from crispembed_b200 import synth

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAXABS = 2e-3


def _check(emb, ref):
    cos = (emb.astype(np.float64) * ref).sum(1) / (np.linalg.norm(emb, axis=1) * np.linalg.norm(ref, axis=1))
    assert cos.min() >= COS_MIN, cos.min()
    assert np.abs(emb - ref).max() <= MAXABS, np.abs(emb - ref).max()


@pytest.fixture(scope="module")
def model(cuda, tiny_model):
    from crispembed_b200 import binding
    m = binding.CrispEmbed(tiny_model)
    yield m
    m.close()


def test_hparams(model):
    h = model.hparams
    assert (h.n_embd, h.n_layer, h.n_head, h.n_experts, h.n_experts_per_tok) == (256, 4, 4, 4, 2)
    assert model.dim == 256


def test_ids_match_oracle(model, oracle, tiny_model):
    ids, lens = synth.ids_ragged(12, 1, 128, seed=4, hi=1000)
    emb = model.encode_ids(ids, lens)
    ref = oracle.encode(oracle.load_model(tiny_model), ids, lens, oracle.GGML)
    _check(emb, ref)
    assert np.allclose(np.linalg.norm(emb, axis=1), 1.0, atol=1e-5)


def test_repeat_bit_identical(model):
    ids, lens = synth.ids_ragged(5, 10, 90, seed=9, hi=1000)
    a = model.encode_ids(ids, lens)
    b = model.encode_ids(ids, lens)
    assert np.array_equal(a, b)


def test_batch_independent_of_packing(model):
    """A sequence's embedding does not depend on what else is in the batch."""
    ids, lens = synth.ids_ragged(6, 20, 100, seed=12, hi=1000)
    full = model.encode_ids(ids, lens)
    off = int(lens[:3].sum())
    single = model.encode_ids(ids[off:off + lens[3]], lens[3:4])
    cos = float((full[3] * single[0]).sum())
    assert cos >= 0.99999


def test_text_abi_matches_ids(model):
    """Synthetic WordPiece vocab: every word maps to one id, wrapped in [CLS]/[SEP]."""
    words = [synth.vocab_word(i) for i in (5, 6, 77, 500, 999)]
    text = " ".join(words)
    emb_t = model.encode(text)
    ids = np.array([1, 5, 6, 77, 500, 999, 2], dtype=np.int32)
    emb_i = model.encode_ids(ids, [len(ids)])[0]
    assert np.array_equal(emb_t, emb_i)
    batch = model.encode([text, words[0]])
    assert batch.shape == (2, 256)
    assert np.array_equal(batch[0], emb_t)


def test_prefix_and_matryoshka(model, oracle):
    w = synth.vocab_word
    model.set_prefix(w(10) + " ")
    a = model.encode(w(11))
    model.set_prefix("")
    b = model.encode(w(10) + " " + w(11))
    assert np.array_equal(a, b)
    full = model.encode(w(12) + " " + w(13))
    small = model.encode(w(12) + " " + w(13), matryoshka_dim=64)
    assert small.shape == (64,)
    ref = full[:64] / np.linalg.norm(full[:64])
    assert np.abs(small - ref).max() <= 1e-5


def test_device_entry_matches_host_entry(model, cuda):
    import torch
    ids, lens = synth.ids_ragged(7, 3, 64, seed=21, hi=1000)
    host = model.encode_ids(ids, lens)
    d_ids = torch.from_numpy(ids).to(cuda)
    out = torch.empty((len(lens), model.dim), dtype=torch.float32, device=cuda)
    model.encode_ids_device(d_ids, lens, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), host)


def test_rejects_bad_input(model):
    from crispembed_b200 import binding
    with pytest.raises(binding.CrispEmbedError):
        model.encode_ids(np.zeros(600, dtype=np.int32), [600])  # longer than n_max_tokens (128)


@pytest.mark.parametrize("wtype_name", ["Q4_K", "F32"])
def test_other_weight_types(cuda, oracle, tmp_path, wtype_name):
    from crispembed_b200 import binding
    from crispembed_b200.gguf_io import GGML_F32, GGML_Q4_K
    wt = {"Q4_K": GGML_Q4_K, "F32": GGML_F32}[wtype_name]
    spec = synth.tiny_spec(wtype=wt, router_wtype=GGML_F32)
    path = str(tmp_path / f"tiny_{wtype_name}.gguf")
    synth.write_model(path, spec)
    m = binding.CrispEmbed(path)
    ids, lens = synth.ids_ragged(5, 2, 100, seed=31, hi=1000)
    emb = m.encode_ids(ids, lens)
    m.close()
    ref = oracle.encode(oracle.load_model(path), ids, lens, oracle.GGML)
    _check(emb, ref)


# GGUF files as llama.cpp writes them beside the reference converter's: a Q4_K_M-like
# mix (Q4_K, with Q6_K for attn_v, the second FFN matrices and the token table) and
# an IQ4_XS file (IQ4_NL attn_v, Q4_0 token table); routers stay F32 as llama.cpp
# keeps ffn_gate_inp.  Mixed q/k/v formats load through a common form.
MIXES = {
    "q4_k_m": dict(wtype=12, router_wtype=0, type_overrides={
        "attn.v.weight": 14, "ffn.expert_fc2.weight": 14, "ffn.fc2.weight": 14, "token_embd.weight": 14}),
    "iq4_xs": dict(wtype=23, router_wtype=0, type_overrides={"attn.v.weight": 20, "token_embd.weight": 2}),
    "legacy": dict(wtype=6, router_wtype=8, type_overrides={"attn.o.weight": 3, "ffn.expert_fc1.weight": 7}),
}


@pytest.mark.parametrize("mix", list(MIXES))
def test_mixed_format_models_match_oracle(cuda, oracle, tmp_path, mix):
    from crispembed_b200 import binding
    path = str(tmp_path / f"{mix}.gguf")
    synth.write_model(path, synth.tiny_spec(**MIXES[mix]))
    m = binding.CrispEmbed(path)
    ids, lens = synth.ids_ragged(8, 2, 100, seed=12, hi=1000)
    emb = m.encode_ids(ids, lens)
    m.close()
    ref = oracle.encode(oracle.load_model(path), ids, lens, oracle.GGML)
    _check(emb, ref)


@pytest.mark.parametrize("theta", [10000.0, 1000.0])
def test_rope_model_matches_oracle(cuda, oracle, tmp_path, theta):
    """A GGUF without a position table runs RoPE with NEOX pairing on Q and K
    (src/crispembed.cpp:788-795, :1182-1195), base from bert.rope_theta."""
    from crispembed_b200 import binding
    path = str(tmp_path / "rope.gguf")
    synth.write_model(path, synth.tiny_spec(rope_theta=theta, qk_scale=0.12))  # sharp attention: positions matter
    m = binding.CrispEmbed(path)
    ids, lens = synth.ids_ragged(8, 2, 128, seed=14, hi=1000)
    emb = m.encode_ids(ids, lens)
    m.close()
    ref = oracle.encode(oracle.load_model(path), ids, lens, oracle.GGML)
    _check(emb, ref)


@pytest.mark.parametrize("spec_kw", [dict(), dict(wtype=12, router_wtype=0, type_overrides={"ffn.expert_fc2.weight": 14})])
def test_llama_cpp_naming_loads_the_same_model(cuda, tmp_path, spec_kw):
    """llama.cpp's nomic-bert-moe export of the same weights (blk.N.* names, fused
    attn_qkv, ffn_gate_inp / ffn_up_exps / ffn_down_exps, nomic-bert-moe.* keys,
    src/crispembed.cpp:800-845) gives bit-identical embeddings."""
    from crispembed_b200 import binding
    a, b = str(tmp_path / "crisp.gguf"), str(tmp_path / "llama.gguf")
    spec = synth.tiny_spec(**spec_kw)
    synth.write_model(a, spec)
    synth.write_model(b, spec, naming="llama")
    ids, lens = synth.ids_ragged(6, 2, 90, seed=21, hi=1000)
    outs = []
    for p in (a, b):
        m = binding.CrispEmbed(p)
        outs.append(m.encode_ids(ids, lens))
        m.close()
    assert np.array_equal(outs[0], outs[1])


def test_graph_replay_matches_eager(cuda, tiny_model):
    """A batch shape met twice is captured into a CUDA graph and replayed from then
    on: the embeddings stay bit-identical to the first (eager) call, every call
    counts the same kernels, and other shapes in between keep working."""
    from crispembed_b200 import binding
    m = binding.CrispEmbed(tiny_model)
    ids, lens = synth.ids_ragged(5, 2, 70, seed=31, hi=1000)
    ids2, lens2 = synth.ids_ragged(3, 2, 50, seed=32, hi=1000)
    first = m.encode_ids(ids, lens)                 # eager, shape recorded
    counts, outs = [], []
    for i in range(4):                              # capture, then replays
        n0 = binding.launch_count()
        outs.append(m.encode_ids(ids, lens))
        counts.append(binding.launch_count() - n0)
        other = m.encode_ids(ids2, lens2)           # a second shape interleaved
    ref2 = m.encode_ids(ids2, lens2)
    m.close()
    for o in outs:
        assert np.array_equal(o, first)
    assert len(set(counts)) == 1 and counts[0] > 0
    assert np.array_equal(other, ref2)


def test_device_calls_on_default_and_side_streams(cuda, tiny_model):
    """encode_ids_device on torch's default (legacy) stream runs on the context's own
    stream between event fences, so it can be graph-captured; the result is ordered
    before the caller's next work on its stream.  Same embeddings as the host call,
    on the default stream and on a side stream, first (eager) call and replays."""
    import torch
    from crispembed_b200 import binding
    m = binding.CrispEmbed(tiny_model)
    ids, lens = synth.ids_ragged(6, 2, 60, seed=41, hi=1000)
    ref = m.encode_ids(ids, lens)
    d_ids = torch.from_numpy(ids).to(cuda)
    for stream in (None, torch.cuda.Stream()):
        with torch.cuda.stream(stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream()):
            out = torch.empty((len(lens), m.dim), dtype=torch.float32, device=cuda)
            for _ in range(4):
                out.zero_()
                m.encode_ids_device(d_ids, lens, out)
                norms = out.norm(dim=1)                 # queued behind the encode, no host sync
                got = out.cpu().numpy()
                assert np.array_equal(got, ref)
                assert torch.allclose(norms.cpu(), torch.ones(len(lens)), atol=1e-4)
    m.close()


@pytest.mark.parametrize("wtype", [8, 12])  # Q8_0, Q4_K
def test_expanded_and_quantized_planes_give_identical_embeddings(cuda, tmp_path, monkeypatch, wtype):
    """The loader expands Q8_0 / Q4_K planes of pair-GEMM width to fp16 once; with
    CEB_WEIGHT_EXPAND=0 the GEMM dequantizes the blocks per tile instead.  Both feed
    the MMA the same fp16 values in the same order: bit-identical embeddings."""
    from crispembed_b200 import binding
    spec = synth.tiny_spec(wtype=wtype, router_wtype=0 if wtype == 12 else None)  # routers: F32 or Q8_0
    p = str(tmp_path / f"tiny_{wtype}.gguf")
    synth.write_model(p, spec)
    ids, lens = synth.ids_ragged(7, 2, 90, seed=51, hi=1000)
    m = binding.CrispEmbed(p)
    expanded = m.encode_ids(ids, lens)
    m.close()
    monkeypatch.setenv("CEB_WEIGHT_EXPAND", "0")
    m = binding.CrispEmbed(p)
    streamed = m.encode_ids(ids, lens)
    m.close()
    assert np.array_equal(expanded, streamed)


def test_large_host_batches_run_in_sequence_groups(cuda, tiny_model, monkeypatch):
    """A host batch above CEB_MAX_BATCH_TOKENS runs as consecutive groups of whole
    sequences through one workspace; every sequence's embedding is independent of
    its batch, so the grouped result equals the single call bit for bit."""
    from crispembed_b200 import binding
    m = binding.CrispEmbed(tiny_model)
    ids, lens = synth.ids_ragged(40, 2, 100, seed=61, hi=1000)
    whole = m.encode_ids(ids, lens)
    monkeypatch.setenv("CEB_MAX_BATCH_TOKENS", "300")
    grouped = m.encode_ids(ids, lens)
    again = m.encode_ids(ids, lens)
    m.close()
    assert int(lens.sum()) > 3 * 300
    assert np.array_equal(whole, grouped)
    assert np.array_equal(whole, again)


def test_device_calls_queued_back_to_back(cuda, tiny_model):
    """Device-buffer calls with different batches queued without a host synchronisation
    in between (more calls than row-offset staging slots): each output equals the
    host call on the same batch."""
    import torch
    from crispembed_b200 import binding
    m = binding.CrispEmbed(tiny_model)
    batches = [synth.ids_ragged(n, 2, 90, seed=70 + n, hi=1000) for n in (3, 9, 5, 12, 7, 4)]
    refs = [m.encode_ids(i, l) for i, l in batches]
    outs = []
    for i, l in batches:
        d_ids = torch.from_numpy(i).to(cuda)
        out = torch.empty((len(l), m.dim), dtype=torch.float32, device=cuda)
        m.encode_ids_device(d_ids, l, out)
        outs.append((d_ids, out))
    torch.cuda.synchronize()
    for (_, o), r in zip(outs, refs):
        assert np.array_equal(o.cpu().numpy(), r)
    m.close()
