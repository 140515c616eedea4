"""MoE feed-forward operator (ceb_moe_ffn) against the CPU oracle.

Reference: the MoE branch of build_encoder_graph, src/crispembed.cpp:1327-1381.
Checks, per BASELINE's bar:
  * router logits bit-identical to the ggml-faithful oracle for Q8_0 routers
    (x re-quantized to Q8_0, integer block dots in ggml's lane order);
  * expert ids bit-exact wherever the k-th/(k+1)-th logit gap exceeds 1e-4;
  * the expert permutation (row of every (token, slot) in the grouped matrices,
    expert row offsets) bit-identical to ggml_mul_mat_id's grouping;
  * expert math within 1e-3 (of max-abs) of the oracle computed with the same
    routing and the kernels' operand precision (F16 mode), and cos >= 0.999 per
    token against the ggml-faithful oracle;
  * repeat calls bit-identical (tests/test_moe_parity.py:149-154 of the reference).
"""
import numpy as np
import pytest

from crispembed_b200 import synth
from crispembed_b200.gguf_io import GGML_F32, GGML_Q4_K, GGML_Q8_0

pytestmark = pytest.mark.gpu

CONFIGS = {
    "q8_small": dict(T=300, d=256, n_experts=4, top_k=2, ffn=512, wtype=GGML_Q8_0, router_wtype=GGML_Q8_0,
                     zipf_s=None, with_bias=True),
    "c3_zipf": dict(T=512, d=768, n_experts=8, top_k=2, ffn=3072, wtype=GGML_Q4_K, router_wtype=GGML_F32,
                    zipf_s=1.2, with_bias=False),
    "c3_q8router": dict(T=257, d=768, n_experts=8, top_k=2, ffn=3072, wtype=GGML_Q8_0, router_wtype=GGML_Q8_0,
                        zipf_s=1.2, with_bias=True),
    "c5_wide": dict(T=200, d=1024, n_experts=32, top_k=4, ffn=1536, wtype=GGML_Q4_K, router_wtype=GGML_F32,
                    zipf_s=None, with_bias=False),
    "c5_zipf": dict(T=129, d=1024, n_experts=32, top_k=4, ffn=1536, wtype=GGML_Q4_K, router_wtype=GGML_F32,
                    zipf_s=1.5, with_bias=False),
    "one_token": dict(T=1, d=256, n_experts=4, top_k=2, ffn=256, wtype=GGML_Q8_0, router_wtype=GGML_Q8_0,
                      zipf_s=None, with_bias=True),
    "skew_empty": dict(T=33, d=256, n_experts=8, top_k=2, ffn=256, wtype=GGML_Q8_0, router_wtype=GGML_Q8_0,
                       zipf_s=3.0, with_bias=False),
}


def _run(cuda, inp, x_dtype="bf16", repeat=1):
    import torch
    from crispembed_b200 import binding
    layer = binding.MoELayer(inp.d, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype,
                             inp.fc1_raw, inp.fc2_raw, inp.bias)
    T = inp.x.shape[0]
    tdt = {"bf16": torch.bfloat16, "f32": torch.float32, "f16": torch.float16}[x_dtype]
    x = torch.from_numpy(inp.x).to(cuda).to(tdt)
    ws = torch.empty(layer.workspace_size(T), dtype=torch.uint8, device=cuda)
    outs = []
    for _ in range(repeat):
        y = torch.empty((T, inp.d), dtype=torch.float32, device=cuda)
        ids = torch.empty((T, inp.top_k), dtype=torch.int32, device=cuda)
        w = torch.empty((T, inp.top_k), dtype=torch.float32, device=cuda)
        cnt = torch.empty((inp.n_experts,), dtype=torch.int32, device=cuda)
        lg = torch.empty((T, inp.n_experts), dtype=torch.float32, device=cuda)
        layer.forward(x, y, ws, ids=ids, weights=w, counts=cnt, logits=lg)
        binding.sync_check()
        _, _, slot_pos, offsets = layer.routing(ws, T)
        outs.append(tuple(t.cpu().numpy() for t in (y, ids, w, cnt, lg)) + (slot_pos, offsets))
    layer.close()
    return outs


def _kth_gap(logits, k):
    s = np.sort(logits, axis=1)[:, ::-1]
    return s[:, k - 1] - s[:, k] if logits.shape[1] > k else np.full(logits.shape[0], np.inf)


@pytest.mark.parametrize("name", list(CONFIGS))
def test_moe_matches_oracle(cuda, oracle, name):
    cfg = dict(CONFIGS[name])
    T = cfg.pop("T")
    inp = synth.make_moe_op_inputs(T, seed=11, **cfg)
    (y, ids, w, cnt, lg, slot_pos, offsets), = _run(cuda, inp)
    x = inp.x
    ry, rids, rw, rlg = oracle.moe_ffn(x, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw,
                                       inp.wtype, inp.fc1_raw, inp.fc2_raw, inp.bias, oracle.GGML)
    # router logits
    if inp.router_wtype == GGML_Q8_0:
        assert np.array_equal(lg, rlg), np.abs(lg - rlg).max()
    else:
        assert np.allclose(lg, rlg, rtol=1e-5, atol=1e-5)
    # routing: bit-exact where the k-th / (k+1)-th logit gap exceeds 1e-4
    gap = _kth_gap(rlg, inp.top_k)
    sure = gap > 1e-4
    assert np.array_equal(ids[sure], rids[sure])
    assert np.allclose(w[sure], rw[sure], rtol=1e-5, atol=1e-7)
    assert np.array_equal(cnt, np.bincount(ids.reshape(-1), minlength=inp.n_experts))
    # permutation: ggml_mul_mat_id's (expert, token, slot) grouping of the same ids, bit for bit
    osp, ooff = oracle.moe_permutation(ids, inp.n_experts)
    assert np.array_equal(offsets, ooff) and np.array_equal(slot_pos, osp)
    if np.array_equal(ids, rids):
        assert np.array_equal(slot_pos, oracle.moe_permutation(rids, inp.n_experts)[0])
    # expert math at kernel precision on the kernel's own routing
    fy, _, _, _ = oracle.moe_ffn(x, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype,
                                 inp.fc1_raw, inp.fc2_raw, inp.bias, oracle.F16, ids_in=ids, wts_in=w)
    scale = max(1e-3, float(np.abs(fy).max()))
    assert np.abs(y - fy).max() <= 1e-3 * scale, np.abs(y - fy).max() / scale
    # against the ggml-faithful oracle (q8 activations) on tokens routed identically
    same = np.all(ids == rids, axis=1)
    a, b = y[same].astype(np.float64), ry[same].astype(np.float64)
    cos = (a * b).sum(1) / np.maximum(np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1), 1e-30)
    assert cos.min() >= 0.999, cos.min()


def test_moe_repeat_bit_identical(cuda):
    inp = synth.make_moe_op_inputs(700, d=768, n_experts=8, top_k=2, ffn=3072, wtype=GGML_Q8_0,
                                   router_wtype=GGML_Q8_0, zipf_s=1.2, seed=5, with_bias=True)
    r = _run(cuda, inp, repeat=2)
    for a, b in zip(r[0], r[1]):
        assert np.array_equal(a, b)


def test_moe_on_two_devices_of_one_process():
    """Launch setup (shared-memory limits, occupancy) is per device: the operator built
    and run on GPU 1 after GPU 0 in the same process gives the same bits on both."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = []
    for T, ffn in ((700, 3072), (40, 384)):  # fc1 of 384 features runs the single-CTA GEMM
        inp = synth.make_moe_op_inputs(T, d=768, n_experts=8, top_k=2, ffn=ffn, wtype=GGML_Q8_0,
                                       router_wtype=GGML_Q8_0, zipf_s=1.2, seed=6, with_bias=True)
        per_dev = []
        for dev in (0, 1):
            with torch.cuda.device(dev):
                per_dev.append(_run(f"cuda:{dev}", inp)[0])
        for a, b in zip(*per_dev):
            assert np.array_equal(a, b)


@pytest.mark.parametrize("E", [16, 32])
def test_f32_router_tile_input_dtypes(cuda, oracle, E):
    """F32 routers with 8 < E <= 32 over activations in memory run the tiled router kernel:
    its logits are the same bits for fp32, fp16 and bf16 inputs holding the same values, and
    match the oracle's F32 router."""
    import dataclasses
    inp = synth.make_moe_op_inputs(300, d=512, n_experts=E, top_k=4, ffn=256, wtype=GGML_Q8_0,
                                   router_wtype=GGML_F32, zipf_s=None, seed=4, with_bias=False)
    # values every input type holds exactly: bf16-representable and zero below fp16's normal range
    x = inp.x.copy()
    x[np.abs(x) < 2.0 ** -14] = 0.0
    inp = dataclasses.replace(inp, x=x)
    res = {dt: _run(cuda, inp, x_dtype=dt)[0] for dt in ("bf16", "f32", "f16")}
    for dt in ("f32", "f16"):
        assert np.array_equal(res[dt][4], res["bf16"][4])  # logits
        assert np.array_equal(res[dt][1], res["bf16"][1])  # ids
    _, rids, _, rlg = oracle.moe_ffn(inp.x, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw,
                                     inp.wtype, inp.fc1_raw, inp.fc2_raw, inp.bias, oracle.GGML)
    lg, ids = res["bf16"][4], res["bf16"][1]
    assert np.allclose(lg, rlg, rtol=1e-5, atol=1e-5), np.abs(lg - rlg).max()
    sure = _kth_gap(rlg, inp.top_k) > 1e-4
    assert np.array_equal(ids[sure], rids[sure])


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_moe_input_dtypes(cuda, oracle, dtype):
    inp = synth.make_moe_op_inputs(96, d=256, n_experts=4, top_k=2, ffn=512, wtype=GGML_Q8_0,
                                   router_wtype=GGML_Q8_0, zipf_s=None, seed=2, with_bias=True)
    (y, ids, w, cnt, lg, _, _), = _run(cuda, inp, x_dtype=dtype)
    (yb, idsb, _, _, _, _, _), = _run(cuda, inp, x_dtype="bf16")
    # x holds bf16-representable values, exactly representable in f32 and (at this range) f16
    assert np.array_equal(ids, idsb)
    assert np.abs(y - yb).max() <= 1e-6 * max(1.0, np.abs(yb).max())


@pytest.mark.parametrize("name", ["q8_small", "c3_q8router", "c3_zipf", "c5_wide", "one_token", "skew_empty"])
def test_route_ln_matches_oracle(cuda, oracle, name):
    """ceb_moe_route_ln: LN(res + y) and the router on the normalised rows, one pass.

    The normalised rows match the oracle's LayerNorm to rounding; the router
    logits are then bit-identical (Q8_0) to the oracle's router applied to the
    kernel's own normalised rows, and the routes follow from them as in
    ceb_moe_ffn.  The fp16 copy is the rounding of the fp32 rows; an aliased
    output (out = res) gives the same results."""
    import torch
    from crispembed_b200 import binding
    cfg = dict(CONFIGS[name])
    T = cfg.pop("T")
    inp = synth.make_moe_op_inputs(T, seed=13, **cfg)
    d, E, K = inp.d, inp.n_experts, inp.top_k
    rng = np.random.default_rng(7)
    res = rng.standard_normal((T, d)).astype(np.float32)
    yv = (rng.standard_normal((T, d)) * 0.5).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    beta = (0.05 * rng.standard_normal(d)).astype(np.float32)
    eps = 1e-12
    layer = binding.MoELayer(d, E, K, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype, inp.fc1_raw, inp.fc2_raw,
                             inp.bias)
    dev = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    ws = torch.empty(layer.workspace_size(T), dtype=torch.uint8, device=cuda)
    out = torch.empty((T, d), dtype=torch.float32, device=cuda)
    out16 = torch.empty((T, d), dtype=torch.float16, device=cuda)
    ids = torch.empty((T, K), dtype=torch.int32, device=cuda)
    w = torch.empty((T, K), dtype=torch.float32, device=cuda)
    lg = torch.empty((T, E), dtype=torch.float32, device=cuda)
    layer.route_ln(dev(res), dev(yv), out, ws, gamma=dev(gamma), beta=dev(beta), eps=eps, out16=out16, ids=ids,
                   weights=w, logits=lg)
    binding.sync_check()
    o, o16, ids_, w_, lg_ = (t.cpu().numpy() for t in (out, out16, ids, w, lg))
    ref_ln = oracle.layernorm(res + yv, gamma, beta, eps)
    assert np.allclose(o, ref_ln, rtol=1e-5, atol=2e-5), np.abs(o - ref_ln).max()
    assert np.array_equal(o16, o.astype(np.float16))
    _, _, _, rlg = oracle.moe_ffn(o, E, K, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype, inp.fc1_raw,
                                  inp.fc2_raw, inp.bias, oracle.GGML)
    if inp.router_wtype == GGML_Q8_0:
        assert np.array_equal(lg_, rlg), np.abs(lg_ - rlg).max()
    else:
        assert np.allclose(lg_, rlg, rtol=1e-5, atol=1e-5)
    rids, rw, _ = oracle.route(rlg, K)
    sure = _kth_gap(rlg, K) > 1e-4
    assert np.array_equal(ids_[sure], rids[sure])
    assert np.allclose(w_[sure], rw[sure], rtol=1e-5, atol=1e-7)
    # in place: out aliases res
    alias = dev(res)
    layer.route_ln(alias, dev(yv), alias, ws, gamma=dev(gamma), beta=dev(beta), eps=eps)
    binding.sync_check()
    assert np.array_equal(alias.cpu().numpy(), o)
    layer.close()


def test_misaligned_activations_rejected_before_any_launch(cuda):
    """Rows are read as 16-byte vectors: an activation pointer off a 16-byte boundary
    is refused on the host with an error, and the next aligned call still works."""
    import torch
    from crispembed_b200 import binding
    inp = synth.make_moe_op_inputs(64, d=256, n_experts=4, top_k=2, ffn=256, wtype=GGML_Q8_0,
                                   router_wtype=GGML_F32, seed=5)
    layer = binding.MoELayer(inp.d, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype,
                             inp.fc1_raw, inp.fc2_raw, inp.bias)
    T = inp.x.shape[0]
    ws = torch.empty(layer.workspace_size(T), dtype=torch.uint8, device=cuda)
    y = torch.empty((T, inp.d), dtype=torch.float32, device=cuda)
    flat = torch.zeros(T * inp.d + 4, dtype=torch.float32, device=cuda)
    x_bad = flat[1:1 + T * inp.d].view(T, inp.d)      # 4 bytes past a 16-byte boundary
    assert x_bad.data_ptr() % 16 != 0
    with pytest.raises(binding.CrispEmbedError):
        layer.forward(x_bad, y, ws)
    x = torch.from_numpy(inp.x).to(cuda)
    layer.forward(x, y, ws)
    binding.sync_check()
    assert torch.isfinite(y).all()
    layer.close()
