"""Varlen multi-head attention against the oracle's restatement of the encoder
graph's attention (src/crispembed.cpp:1278-1297): softmax(Q K^T / 8) V per
sequence and head.  Both kernels are checked: the mma.sync kernel (default) and
the tcgen05 CTA-pair kernel (CEB_ATTN_TC=1; sequences of up to 512 tokens).

Inputs are fp16 (as the QKV projection writes them); the oracle computes in fp32
from the same fp16 values.  P is rounded to fp16 before the P V product on the
GPU, so the tolerance is 3e-3 absolute on outputs of magnitude ~1.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LEN_SETS = [
    [1],
    [17, 31, 32, 33],
    [128, 129, 255, 256, 257],
    [300, 511, 512, 7, 64],
    [600, 40],  # longest > 512: the mma.sync kernel
]


def _qkv(lens, n_head, seed):
    rng = np.random.default_rng(seed)
    d = 64 * n_head
    rows = int(sum(lens))
    qkv = rng.standard_normal((rows, 3 * d), dtype=np.float32).astype(np.float16)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return qkv, cu, d


@pytest.fixture(params=["mma_sync", "tcgen05"])
def attn_impl(request, monkeypatch):
    if request.param == "tcgen05":
        monkeypatch.setenv("CEB_ATTN_TC", "1")
    else:
        monkeypatch.delenv("CEB_ATTN_TC", raising=False)
    return request.param


@pytest.mark.parametrize("n_head", [2, 3])
@pytest.mark.parametrize("lens", LEN_SETS)
def test_attention_matches_oracle(cuda, oracle, attn_impl, lens, n_head):
    import torch
    from crispembed_b200 import binding
    qkv, cu, d = _qkv(lens, n_head, seed=sum(lens))
    out = binding.attention(torch.from_numpy(qkv).to(cuda), torch.from_numpy(cu).to(cuda), n_head)
    binding.sync_check()
    ref = oracle.attention(qkv.astype(np.float32), cu, n_head, d)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= 3e-3, err


def test_attention_twelve_heads_model_shape(cuda, oracle, attn_impl):
    """d = 768, 12 heads, a batch of ragged lengths as in the benchmark workload."""
    import torch
    from crispembed_b200 import binding
    rng = np.random.default_rng(5)
    lens = list(rng.integers(32, 513, size=12))
    qkv, cu, d = _qkv(lens, 12, seed=9)
    out = binding.attention(torch.from_numpy(qkv).to(cuda), torch.from_numpy(cu).to(cuda), 12)
    binding.sync_check()
    ref = oracle.attention(qkv.astype(np.float32), cu, 12, d)
    assert np.abs(out.float().cpu().numpy() - ref).max() <= 3e-3


def test_attention_repeatable(cuda, attn_impl):
    import torch
    from crispembed_b200 import binding
    qkv, cu, _ = _qkv([200, 512, 33], 2, seed=3)
    q = torch.from_numpy(qkv).to(cuda)
    c = torch.from_numpy(cu).to(cuda)
    a = binding.attention(q, c, 2).cpu().numpy()
    b = binding.attention(q, c, 2).cpu().numpy()
    assert np.array_equal(a, b)
