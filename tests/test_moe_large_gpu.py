"""The MoE operator (ceb_moe_ffn) at BASELINE's full operator sizes against the oracle.

Config 3 (T = 65,536, d = 768, E = 8, top-2, F = 3072, Zipf 1.2 loads) and config 5
(T = 131,072, d = 1024, E = 32, top-4, F = 1536, balanced and Zipf 1.5), Q4_K
experts, F32 router, bf16 activations -- the inputs bench.py times.  At full size:

  * expert counts = the histogram of the ids, offsets = their prefix sum, and the
    permutation of every (token, slot) row equal to ggml_mul_mat_id's (expert,
    token, slot) grouping (src/crispembed.cpp:1365,1371), bit for bit;
  * every route is the top-k of the kernel's own logits (where the k-th and
    (k+1)-th differ by more than 1e-6), and every gate weight its softmax
    probability (not renormalised, :1343-1345).

On 2,048 sampled tokens (the oracle's cost grows with the tokens it computes):

  * router logits within 1e-5 of the oracle's, ids bit-exact where the oracle's
    k-th / (k+1)-th logit gap exceeds 1e-4;
  * y within 1e-3 of max-abs of the oracle's expert math at the kernels' operand
    precision (F16 mode) on the kernels' own routing.
"""
import numpy as np
import pytest

from crispembed_b200 import synth
from crispembed_b200.gguf_io import GGML_F32, GGML_Q4_K

pytestmark = pytest.mark.gpu

CASES = {
    "c3_T65536_zipf1.2": dict(T=65536, d=768, n_experts=8, top_k=2, ffn=3072, zipf_s=1.2),
    "c5_T131072_balanced": dict(T=131072, d=1024, n_experts=32, top_k=4, ffn=1536, zipf_s=None),
    "c5_T131072_zipf1.5": dict(T=131072, d=1024, n_experts=32, top_k=4, ffn=1536, zipf_s=1.5),
}
N_SAMPLE = 2048


def _softmax(lg):
    e = np.exp(lg.astype(np.float64) - lg.max(axis=1, keepdims=True))
    return e / e.sum(axis=1, keepdims=True)


@pytest.mark.parametrize("name", list(CASES))
def test_moe_full_size(cuda, oracle, name):
    import torch
    from crispembed_b200 import binding
    cfg = dict(CASES[name])
    T = cfg.pop("T")
    inp = synth.make_moe_op_inputs(T, wtype=GGML_Q4_K, router_wtype=GGML_F32, seed=0, **cfg)
    E, K = inp.n_experts, inp.top_k
    layer = binding.MoELayer(inp.d, E, K, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype, inp.fc1_raw,
                             inp.fc2_raw, inp.bias)
    x = torch.from_numpy(inp.x).to(cuda).to(torch.bfloat16)
    ws = torch.empty(layer.workspace_size(T), dtype=torch.uint8, device=cuda)
    y = torch.empty((T, inp.d), dtype=torch.float32, device=cuda)
    ids = torch.empty((T, K), dtype=torch.int32, device=cuda)
    w = torch.empty((T, K), dtype=torch.float32, device=cuda)
    cnt = torch.empty((E,), dtype=torch.int32, device=cuda)
    lg = torch.empty((T, E), dtype=torch.float32, device=cuda)
    layer.forward(x, y, ws, ids=ids, weights=w, counts=cnt, logits=lg)
    binding.sync_check()
    _, _, slot_pos, offsets = layer.routing(ws, T)
    y, ids, w, cnt, lg = (t.cpu().numpy() for t in (y, ids, w, cnt, lg))
    del x, ws
    layer.close()

    # full size: histogram, offsets, permutation
    flat = ids.reshape(-1)
    assert flat.min() >= 0 and flat.max() < E
    assert np.array_equal(cnt, np.bincount(flat, minlength=E))
    assert np.array_equal(offsets, np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32))
    expect = np.empty(T * K, dtype=np.int32)
    expect[np.argsort(flat, kind="stable")] = np.arange(T * K, dtype=np.int32)
    assert np.array_equal(slot_pos.reshape(-1), expect)
    # full size: routes are the top-k of the kernel's logits (the kernel ranks the rounded
    # probabilities, so only logit gaps above 1e-6 are decisive), weights their probabilities
    order = np.argsort(-lg, axis=1, kind="stable")
    sl = np.take_along_axis(lg, order, axis=1)
    clear = (sl[:, K - 1] - sl[:, K]) > 1e-6
    assert np.array_equal(np.sort(ids[clear], axis=1), np.sort(order[clear, :K], axis=1))
    p = _softmax(lg)
    assert np.allclose(w, np.take_along_axis(p, ids.astype(np.int64), axis=1), rtol=2e-6, atol=1e-7)
    print(f"{name}: expert loads max/mean {cnt.max() / cnt.mean():.2f}, min {cnt.min()}")

    # sampled tokens against the oracle
    sample = np.sort(np.random.default_rng(7).choice(T, N_SAMPLE, replace=False))
    xs = np.ascontiguousarray(inp.x[sample])
    rlg = oracle.matmul(inp.router_wtype, inp.router_raw, E, inp.d, xs, oracle.GGML)
    assert np.allclose(lg[sample], rlg, rtol=1e-5, atol=1e-5), np.abs(lg[sample] - rlg).max()
    rids, rw, _ = oracle.route(rlg, K)
    s = -np.sort(-rlg, axis=1)
    sure = (s[:, K - 1] - s[:, K]) > 1e-4
    assert np.array_equal(ids[sample][sure], rids[sure])
    fy, _, _, _ = oracle.moe_ffn(xs, E, K, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype, inp.fc1_raw,
                                 inp.fc2_raw, inp.bias, oracle.F16, ids_in=ids[sample], wts_in=w[sample])
    scale = max(1e-3, float(np.abs(fy).max()))
    err = float(np.abs(y[sample] - fy).max())
    print(f"{name}: sampled y max-abs error {err:.2e} (scale {scale:.2e}), {int((~sure).sum())} near-ties")
    assert err <= 1e-3 * scale
