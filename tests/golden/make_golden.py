"""Regenerate the golden fixtures in this directory.

    python tests/golden/make_golden.py

gguf_variants.npz -- blocks of the llama.cpp community / registry formats (Q4_0,
                Q4_1, Q5_0, Q5_1, Q5_K, Q6_K, IQ4_NL, IQ4_XS, BF16) from
                crispembed_b200.quant and gguf-py's decoding of them.
formats.npz  -- pins the GGUF block formats against gguf-py, the library the
                reference's converter calls (models/convert-bert-to-gguf.py:68-77):
                * q8_x / q8_blocks / q8_deq: a seeded float matrix, gguf-py's Q8_0
                  quantization of it and gguf-py's dequantization;
                * q4_blocks / q4_deq: Q4_K blocks from crispembed_b200.quant and
                  gguf-py's dequantization of them.
oracle.npz   -- regression pins of the CPU oracle (not reference outputs): tiny-model
                embeddings in GGML and EXACT modes, and one MoE-operator call.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def make_formats():
    import gguf
    from gguf import quants

    from crispembed_b200 import quant
    rng = np.random.default_rng(1234)
    x = (rng.standard_normal((16, 512), dtype=np.float32) * 0.05).astype(np.float32)
    x[0, :32] = 0.0                       # all-zero block (d = 0)
    x[1, :32] = np.linspace(-1, 1, 32)    # exact ties in x/d
    q8 = quants.quantize(x, gguf.GGMLQuantizationType.Q8_0)
    q8_deq = quants.dequantize(q8, gguf.GGMLQuantizationType.Q8_0)
    q4 = quant.quantize_q4_k(x)
    q4_deq = quants.dequantize(q4, gguf.GGMLQuantizationType.Q4_K).reshape(x.shape)
    np.savez_compressed(os.path.join(HERE, "formats.npz"), q8_x=x, q8_blocks=q8, q8_deq=q8_deq, q4_blocks=q4,
                        q4_deq=q4_deq.astype(np.float32), gguf_version=np.array(getattr(gguf, "__version__", "?")))


def make_variants():
    """gguf_variants.npz -- for each block format of the community / registry GGUFs:
    our encoder's blocks of a seeded matrix and gguf-py's decoding of them."""
    import gguf
    from gguf import quants

    from crispembed_b200 import gguf_io as G
    from crispembed_b200 import quant
    rng = np.random.default_rng(4321)
    x = (rng.standard_normal((8, 512), dtype=np.float32) * 0.05).astype(np.float32)
    x[0, :256] = 0.0                        # all-zero super-block
    x[1, :32] = np.linspace(-1, 1, 32)      # a wide block
    out = {"x": x}
    for name in ("Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q5_K", "Q6_K", "IQ4_NL", "IQ4_XS", "BF16"):
        t = getattr(G, "GGML_" + name)
        blocks = quant.quantize(x, t).view(np.uint8).reshape(x.shape[0], -1)
        out[name + "_blocks"] = blocks
        out[name + "_deq"] = quants.dequantize(blocks, getattr(gguf.GGMLQuantizationType, name)).reshape(
            x.shape).astype(np.float32)
    out["gguf_version"] = np.array(getattr(gguf, "__version__", "?"))
    np.savez_compressed(os.path.join(HERE, "gguf_variants.npz"), **out)


def make_oracle():
    import tempfile

    import oracle as O
    from crispembed_b200 import synth
    from crispembed_b200.gguf_io import GGML_Q8_0
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "tiny.gguf")
        synth.write_model(p, synth.tiny_spec())
        m = O.load_model(p)
        ids, lens = synth.ids_ragged(6, 3, 80, seed=5, hi=1000)
        e_ggml = O.encode(m, ids, lens, O.GGML)
        e_exact = O.encode(m, ids, lens, O.EXACT)
    inp = synth.make_moe_op_inputs(64, d=256, n_experts=4, top_k=2, ffn=512, wtype=GGML_Q8_0, router_wtype=GGML_Q8_0,
                                   zipf_s=None, seed=3, with_bias=True)
    y, rid, rw, lg = O.moe_ffn(inp.x, 4, 2, 512, inp.router_wtype, inp.router_raw, inp.wtype, inp.fc1_raw, inp.fc2_raw,
                               inp.bias, O.GGML)
    np.savez_compressed(os.path.join(HERE, "oracle.npz"), ids=ids, lens=lens, emb_ggml=e_ggml, emb_exact=e_exact,
                        moe_y=y, moe_ids=rid, moe_w=rw, moe_logits=lg)


if __name__ == "__main__":
    make_formats()
    make_variants()
    make_oracle()
    print("wrote", os.listdir(HERE))
