"""Grouped-GEMM kernels (tcgen05) against the oracle.

Weights with an output width that is a multiple of 256 run on the CTA-pair
kernel (cta_group::2), by default from an fp16 plane the loader expanded once on
the device (CEB_WEIGHT_EXPAND=0 keeps Q8_0 / Q4_K blocks and dequantizes them
in the kernel); other widths run on the single-CTA kernel.  The cases below
cover both, including partial token tiles where only the first CTA of a pair
has rows (m mod 256 in 1..128).

The oracle's F16 mode rounds operands exactly as the kernel does (weights to
fp16(dequant), activations fp16) and accumulates in double, so the remaining
difference is fp32 accumulation order: tolerance 2e-4 of the output's max-abs.
Reference product: ggml_mul_mat in build_encoder_graph (src/crispembed.cpp:1160-1416).
"""
import numpy as np
import pytest

from crispembed_b200 import quant
from crispembed_b200 import gguf_io as G
from crispembed_b200.gguf_io import GGML_F16, GGML_F32, GGML_Q4_K, GGML_Q8_0

pytestmark = pytest.mark.gpu

CASES = [
    # (w_type, n_out, k, m)
    (GGML_Q8_0, 128, 64, 1),
    (GGML_Q8_0, 256, 768, 5),
    (GGML_Q8_0, 384, 768, 129),
    (GGML_Q8_0, 768, 3072, 300),
    (GGML_Q8_0, 128, 256, 1000),
    (GGML_Q4_K, 256, 768, 77),
    (GGML_Q4_K, 768, 3072, 256),
    (GGML_F32, 256, 512, 200),
    (GGML_F16, 128, 192, 33),
    (GGML_Q8_0, 768, 768, 1000),
    (GGML_Q8_0, 512, 256, 257),
    (GGML_Q8_0, 256, 128, 128),
    (GGML_Q4_K, 512, 512, 383),
]


def _inputs(w_type, n_out, k, m, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n_out, k), dtype=np.float32) * 0.02).astype(np.float32)
    raw = quant.quantize(w, w_type)
    x = rng.standard_normal((m, k), dtype=np.float32).astype(np.float16)
    bias = (rng.standard_normal(n_out, dtype=np.float32) * 0.02).astype(np.float32)
    return raw, x, bias


@pytest.mark.parametrize("w_type,n_out,k,m", CASES)
def test_matmul_f32_out(cuda, oracle, w_type, n_out, k, m):
    import torch
    from crispembed_b200 import binding
    raw, x, bias = _inputs(w_type, n_out, k, m, seed=n_out + k + m)
    xd = torch.from_numpy(x).to(cuda)
    out = binding.matmul(w_type, raw, n_out, k, xd).cpu().numpy()
    ref = oracle.matmul(w_type, raw, n_out, k, x.astype(np.float32), oracle.F16)
    tol = 2e-4 * max(1.0, float(np.abs(ref).max()))
    assert np.abs(out - ref).max() <= tol, np.abs(out - ref).max()


@pytest.mark.parametrize("w_type,n_out,k,m", [CASES[2], CASES[5], CASES[7], CASES[9], CASES[10], CASES[12]])
def test_matmul_bias_gelu_f16_out(cuda, oracle, w_type, n_out, k, m):
    import torch
    from crispembed_b200 import binding
    raw, x, bias = _inputs(w_type, n_out, k, m, seed=7 * m + 1)
    xd = torch.from_numpy(x).to(cuda)
    bd = torch.from_numpy(bias).to(cuda)
    out = binding.matmul(w_type, raw, n_out, k, xd, bias=bd, gelu=True, out_f16=True).float().cpu().numpy()
    ref = oracle.gelu_erf(oracle.matmul(w_type, raw, n_out, k, x.astype(np.float32), oracle.F16, bias=bias))
    ref16 = ref.astype(np.float16).astype(np.float32)
    tol = 2e-3 * max(1.0, float(np.abs(ref).max()))
    assert np.abs(out - ref16).max() <= tol


def test_matmul_repeatable(cuda):
    import torch
    from crispembed_b200 import binding
    raw, x, _ = _inputs(GGML_Q8_0, 384, 768, 517, seed=3)
    xd = torch.from_numpy(x).to(cuda)
    a = binding.matmul(GGML_Q8_0, raw, 384, 768, xd).cpu().numpy()
    b = binding.matmul(GGML_Q8_0, raw, 384, 768, xd).cpu().numpy()
    assert np.array_equal(a, b)


def test_matmul_zero_rows(cuda):
    import torch
    from crispembed_b200 import binding
    raw, x, _ = _inputs(GGML_Q8_0, 128, 64, 1, seed=1)
    out = binding.matmul(GGML_Q8_0, raw, 128, 64, torch.zeros((0, 64), dtype=torch.float16, device=cuda))
    assert out.shape == (0, 128)


def test_matmul_rejects_bad_shape(cuda):
    import torch
    from crispembed_b200 import binding
    raw, x, _ = _inputs(GGML_Q8_0, 128, 64, 4, seed=1)
    xd = torch.from_numpy(x).to(cuda)
    with pytest.raises(binding.CrispEmbedError):
        binding.matmul(GGML_Q8_0, quant.quantize(np.zeros((96, 64), np.float32), GGML_Q8_0), 96, 64, xd)


def test_pair_and_single_cta_kernels_agree(cuda, tmp_path):
    """The single-CTA kernel (forced by CEB_GEMM_SINGLE_CTA=1 in a child process)
    and the CTA-pair kernel give the same product up to fp32 summation order."""
    import os
    import subprocess
    import sys

    import torch
    from crispembed_b200 import binding
    raw, x, bias = _inputs(GGML_Q8_0, 768, 768, 700, seed=11)
    xd = torch.from_numpy(x).to(cuda)
    bd = torch.from_numpy(bias).to(cuda)
    pair_out = binding.matmul(GGML_Q8_0, raw, 768, 768, xd, bias=bd, gelu=True, out_f16=True).float().cpu().numpy()
    np.save(tmp_path / "raw.npy", raw)
    np.save(tmp_path / "x.npy", x)
    np.save(tmp_path / "bias.npy", bias)
    code = (
        "import numpy as np, torch, sys\n"
        "from crispembed_b200 import binding\n"
        f"d = {str(tmp_path)!r}\n"
        "raw = np.load(d + '/raw.npy'); x = np.load(d + '/x.npy'); b = np.load(d + '/bias.npy')\n"
        "o = binding.matmul(8, raw, 768, 768, torch.from_numpy(x).cuda(), bias=torch.from_numpy(b).cuda(),"
        " gelu=True, out_f16=True).float().cpu().numpy()\n"
        "np.save(d + '/single.npy', o)\n")
    env = dict(os.environ, CEB_GEMM_SINGLE_CTA="1")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    subprocess.run([sys.executable, "-c", code], check=True, env=env, cwd=root, timeout=300)
    single = np.load(tmp_path / "single.npy")
    assert np.abs(single - pair_out).max() <= 2e-3 * max(1.0, float(np.abs(pair_out).max()))


# llama.cpp community / registry formats: IQ4_NL and IQ4_XS run re-encoded as Q8_0
# blocks (pair kernel for widths of 256), the others as fp16 planes (single-CTA
# kernel).  IQ4_XS's sub-block scale d*(ls-32) is rounded to fp16 there, one
# rounding the oracle's fp16(dequant) does not make: wider tolerance for it.
VARIANT_CASES = [(getattr(G, "GGML_" + n), 256, 512, 300) for n in
                 ("Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q5_K", "Q6_K", "IQ4_NL", "IQ4_XS", "BF16")]
VARIANT_CASES += [(G.GGML_Q6_K, 384, 768, 77), (G.GGML_IQ4_XS, 768, 3072, 129), (G.GGML_IQ4_NL, 128, 64, 1)]


@pytest.mark.parametrize("w_type,n_out,k,m", VARIANT_CASES)
def test_matmul_gguf_variants(cuda, oracle, w_type, n_out, k, m):
    import torch
    from crispembed_b200 import binding
    raw, x, bias = _inputs(w_type, n_out, k, m, seed=3 * n_out + k + m + w_type)
    xd = torch.from_numpy(x).to(cuda)
    out = binding.matmul(w_type, raw, n_out, k, xd).cpu().numpy()
    ref = oracle.matmul(w_type, raw, n_out, k, x.astype(np.float32), oracle.F16)
    tol = (2e-3 if w_type == G.GGML_IQ4_XS else 2e-4) * max(1.0, float(np.abs(ref).max()))
    assert np.abs(out - ref).max() <= tol, np.abs(out - ref).max()


@pytest.mark.parametrize("w_type,n_out,k,m", [CASES[1], CASES[3], CASES[6], CASES[10], CASES[12]])
def test_expanded_and_streamed_quant_planes_bit_identical(cuda, monkeypatch, w_type, n_out, k, m):
    """The fp16 plane expanded at load and the quantized plane dequantized inside the
    pair kernel feed the MMA the same fp16 operands in the same order."""
    import torch
    from crispembed_b200 import binding
    raw, x, bias = _inputs(w_type, n_out, k, m, seed=5 * m + n_out)
    xd = torch.from_numpy(x).to(cuda)
    bd = torch.from_numpy(bias).to(cuda)
    expanded = binding.matmul(w_type, raw, n_out, k, xd, bias=bd, gelu=True).cpu().numpy()
    monkeypatch.setenv("CEB_WEIGHT_EXPAND", "0")
    streamed = binding.matmul(w_type, raw, n_out, k, xd, bias=bd, gelu=True).cpu().numpy()
    assert np.array_equal(expanded, streamed)
