"""Varlen multi-head attention against the oracle's restatement of the encoder
graph's attention (src/crispembed.cpp:1278-1297): softmax(Q K^T / 8) V per
sequence and head.  All three kernels are checked: the single-CTA tcgen05 kernel
(default), the mma.sync kernel (CEB_ATTN_MMA=1) and the tcgen05 CTA-pair kernel
(CEB_ATTN_TC=1; sequences of up to 512 tokens).

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
    [450, 200, 256, 30, 385, 193],
    [600, 40],  # longest > 512: the CTA-pair kernel falls back to mma.sync
    [1500, 130],  # many 128-key chunks per item
    [1] * 150 + [3, 129],  # many one-token sequences: mostly empty query tiles
]


def _qkv(lens, n_head, seed):
    rng = np.random.default_rng(seed)
    d = 64 * n_head
    rows = int(sum(lens))
    qkv = rng.standard_normal((rows, 3 * d), dtype=np.float32).astype(np.float16)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return qkv, cu, d


@pytest.fixture(params=["tcgen05_cta", "mma_sync", "tcgen05_pair"])
def attn_impl(request, monkeypatch):
    """tcgen05_cta: the default single-CTA tcgen05 kernel; mma_sync (CEB_ATTN_MMA=1) and
    tcgen05_pair (CEB_ATTN_TC=1): the other two kernels."""
    monkeypatch.delenv("CEB_ATTN_TC", raising=False)
    monkeypatch.delenv("CEB_ATTN_MMA", raising=False)
    if request.param == "tcgen05_pair":
        monkeypatch.setenv("CEB_ATTN_TC", "1")
    elif request.param == "mma_sync":
        monkeypatch.setenv("CEB_ATTN_MMA", "1")
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


@pytest.mark.parametrize("cu_list,rows,max_len", [
    ([0, 64], 64, 32),      # a sequence longer than max_len
    ([0, 40, 100], 64, 64),  # offsets past the last row
])
def test_inconsistent_row_offsets_reported(cuda, attn_impl, cu_list, rows, max_len):
    """Offsets that disagree with max_len or leave the rows set the device error word
    (status 5 from ceb_sync_check) and write nothing; the context stays usable."""
    import torch
    from crispembed_b200 import binding
    qkv, _, _ = _qkv([rows], 2, seed=4)
    q = torch.from_numpy(qkv).to(cuda)
    cu = torch.tensor(cu_list, dtype=torch.int32, device=cuda)
    out = binding.attention(q, cu, 2, max_len=max_len)
    with pytest.raises(binding.CrispEmbedError, match=r"\(5\).*0x106"):
        binding.sync_check()
    binding.sync_check()  # reported once, then clear
    good = binding.attention(q, torch.tensor([0, rows], dtype=torch.int32, device=cuda), 2)
    binding.sync_check()
    assert torch.isfinite(good.float()).all()
    del out


def test_error_words_are_per_device(attn_impl):
    """A device-side check raised by an operator on GPU 1 is reported by ceb_sync_check
    on GPU 1 only; GPU 0's word stays clear (one error word per device)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from crispembed_b200 import binding
    binding.load_library()
    qkv, _, _ = _qkv([64], 2, seed=4)
    for dev in (0, 1):  # both devices have an error word before the fault is raised
        with torch.cuda.device(dev):
            binding.sync_check()
    with torch.cuda.device(1):
        q = torch.from_numpy(qkv).to("cuda:1")
        binding.attention(q, torch.tensor([0, 64], dtype=torch.int32, device="cuda:1"), 2, max_len=32)
        torch.cuda.synchronize()
    with torch.cuda.device(0):
        binding.sync_check()
    with torch.cuda.device(1):
        with pytest.raises(binding.CrispEmbedError, match=r"\(5\)"):
            binding.sync_check()
        binding.sync_check()


def test_calls_on_two_streams_overlap(cuda):
    """The operator entry keeps one work-item counter per (device, stream): launches on
    two streams that overlap on the GPU give the bits the same calls give one at a time."""
    import torch
    from crispembed_b200 import binding
    binding.load_library()
    cases = []
    for lens, seed in (([300, 511, 64, 200, 17], 11), ([128, 450, 33, 257], 12)):
        qkv, cu, _ = _qkv(lens, 12, seed=seed)
        cases.append((torch.from_numpy(qkv).to(cuda), torch.from_numpy(cu).to(cuda), max(lens)))
    ref = [binding.attention(q, c, 12, max_len=m) for q, c, m in cases]
    torch.cuda.synchronize()
    binding.sync_check()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    got = [[], []]
    for _ in range(4):
        for k, ((q, c, m), s) in enumerate(zip(cases, streams)):
            with torch.cuda.stream(s):
                got[k].append(binding.attention(q, c, 12, max_len=m, stream=s.cuda_stream))
    torch.cuda.synchronize()
    binding.sync_check()
    for k in range(2):
        for o in got[k]:
            assert torch.equal(o, ref[k])
