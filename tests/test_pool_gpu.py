"""Mean-pool + L2 epilogue (ceb_pool_l2) against the oracle.

Reference: encode_tokens' host pooling, src/crispembed.cpp:1822-1846
(sequential float sum over rows, divide by the count, p / sqrtf(max(sum p^2,
1e-12))), and the Matryoshka truncate + renormalise of :2786-2793.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _cu(lens):
    cu = np.zeros(len(lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    return cu


@pytest.mark.parametrize("d", [256, 768, 1024])
def test_pool_matches_oracle(cuda, oracle, d):
    import torch
    from crispembed_b200 import binding
    rng = np.random.default_rng(d)
    lens = np.array([1, 2, 31, 32, 33, 128, 511, 512, 7], dtype=np.int32)
    cu = _cu(lens)
    h = rng.standard_normal((int(cu[-1]), d), dtype=np.float32)
    out = binding.pool_l2(torch.from_numpy(h).to(cuda), torch.from_numpy(cu).to(cuda)).cpu().numpy()
    ref = oracle.pool_l2(h, cu)
    assert np.abs(out - ref).max() <= 2e-6
    assert np.allclose(np.linalg.norm(out, axis=1), 1.0, atol=1e-5)


def test_pool_matryoshka(cuda, oracle):
    import torch
    from crispembed_b200 import binding
    rng = np.random.default_rng(1)
    lens = np.array([5, 77, 300], dtype=np.int32)
    cu = _cu(lens)
    h = rng.standard_normal((int(cu[-1]), 768), dtype=np.float32)
    out = binding.pool_l2(torch.from_numpy(h).to(cuda), torch.from_numpy(cu).to(cuda), out_dim=256).cpu().numpy()
    ref = oracle.truncate_renorm(oracle.pool_l2(h, cu), 256)
    assert out.shape == (3, 256)
    assert np.abs(out - ref).max() <= 2e-6


def test_pool_empty_sequence_and_unaligned_rows(cuda, oracle):
    """A sequence without rows pools to zeros; hidden rows off a 16-byte boundary take
    the scalar path and give the same result."""
    import torch
    from crispembed_b200 import binding
    rng = np.random.default_rng(3)
    lens = np.array([0, 3, 64, 0, 9], dtype=np.int32)
    cu = _cu(lens)
    h = rng.standard_normal((int(cu[-1]), 256), dtype=np.float32)
    out = binding.pool_l2(torch.from_numpy(h).to(cuda), torch.from_numpy(cu).to(cuda)).cpu().numpy()
    ref = oracle.pool_l2(h, cu)
    assert np.all(out[0] == 0.0) and np.all(out[3] == 0.0)
    assert np.abs(out - ref).max() <= 2e-6
    buf = torch.empty(int(cu[-1]) * 256 + 1, dtype=torch.float32, device=cuda)
    shifted = buf[1:].view(int(cu[-1]), 256)  # 4-byte offset
    shifted.copy_(torch.from_numpy(h))
    out2 = binding.pool_l2(shifted, torch.from_numpy(cu).to(cuda)).cpu().numpy()
    assert np.abs(out2 - ref).max() <= 2e-6


def test_pool_zero_vector_epsilon(cuda):
    import torch
    from crispembed_b200 import binding
    h = np.zeros((4, 256), dtype=np.float32)
    cu = _cu(np.array([4], dtype=np.int32))
    out = binding.pool_l2(torch.from_numpy(h).to(cuda), torch.from_numpy(cu).to(cuda)).cpu().numpy()
    assert np.all(out == 0.0)  # sqrt(max(0, 1e-12)) keeps the division finite
