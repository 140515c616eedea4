"""The CPU oracle: regression pins (tests/golden/oracle.npz) and internal checks
of the ggml arithmetic it restates."""
import os

import numpy as np
import pytest

from crispembed_b200 import quant, synth

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "oracle.npz"))


def test_encoder_regression(oracle, tiny_model):
    m = oracle.load_model(tiny_model)
    e = oracle.encode(m, GOLD["ids"], GOLD["lens"], oracle.GGML)
    assert np.array_equal(e, GOLD["emb_ggml"])
    e2 = oracle.encode(m, GOLD["ids"], GOLD["lens"], oracle.EXACT)
    assert np.array_equal(e2, GOLD["emb_exact"])


def test_modes_agree_within_bar(oracle):
    a, b = GOLD["emb_ggml"].astype(np.float64), GOLD["emb_exact"].astype(np.float64)
    cos = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    assert cos.min() >= 0.9999
    assert np.allclose(np.linalg.norm(a, axis=1), 1.0, atol=1e-5)


def test_moe_regression(oracle):
    from crispembed_b200.gguf_io import GGML_Q8_0
    inp = synth.make_moe_op_inputs(64, d=256, n_experts=4, top_k=2, ffn=512, wtype=GGML_Q8_0,
                                   router_wtype=GGML_Q8_0, zipf_s=None, seed=3, with_bias=True)
    y, ids, w, lg = oracle.moe_ffn(inp.x, 4, 2, 512, inp.router_wtype, inp.router_raw, inp.wtype, inp.fc1_raw,
                                   inp.fc2_raw, inp.bias, oracle.GGML)
    for got, key in ((y, "moe_y"), (ids, "moe_ids"), (w, "moe_w"), (lg, "moe_logits")):
        assert np.array_equal(got, GOLD[key]), key


def _np_q8_act(x):
    """numpy restatement of ggml's x86 quantize_row_q8_0 (multiplier 127/amax, ties to even)."""
    b = x.reshape(-1, 32).astype(np.float32)
    amax = np.abs(b).max(1)
    d16 = (amax / np.float32(127)).astype(np.float16)
    with np.errstate(divide="ignore"):
        inv = np.where(amax > 0, np.float32(127) / amax, np.float32(0)).astype(np.float32)
    q = np.rint(b * inv[:, None]).astype(np.int8)
    return d16, q


def test_activation_q8_0_matches_numpy(oracle):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(32 * 40).astype(np.float32)
    x[:32] = 0
    x[32:64] = np.arange(32, dtype=np.float32) - 15.5  # many exact .5 products
    blocks = oracle.quant_act_q8_0(x).reshape(-1, 34)
    d16, q = _np_q8_act(x)
    assert np.array_equal(blocks[:, :2].copy().view(np.float16).reshape(-1), d16)
    assert np.array_equal(blocks[:, 2:].view(np.int8), q)


def test_q8_0_dot_lane_order(oracle):
    """ceo_dot_q8_0 == eight FMA lanes (4 products each) summed ((0+4)+(2+6))+((1+5)+(3+7))."""
    rng = np.random.default_rng(4)
    k = 768
    w = quant.quantize_q8_0((rng.standard_normal((1, k)) * 0.02).astype(np.float32)).reshape(-1, 34)
    a = oracle.quant_act_q8_0(rng.standard_normal(k).astype(np.float32)).reshape(-1, 34)
    acc = np.zeros(8, np.float32)
    for b in range(k // 32):
        d = np.float32(w[b, :2].copy().view(np.float16)[0]) * np.float32(a[b, :2].copy().view(np.float16)[0])
        pw = w[b, 2:].view(np.int8).astype(np.int32)
        pa = a[b, 2:].view(np.int8).astype(np.int32)
        s = (pw * pa).reshape(8, 4).sum(1).astype(np.float32)
        acc = (np.float64(d) * s.astype(np.float64) + acc.astype(np.float64)).astype(np.float32)  # exact fma for these sizes
    ref = np.float32(np.float32(np.float32(acc[0] + acc[4]) + np.float32(acc[2] + acc[6])) +
                     np.float32(np.float32(acc[1] + acc[5]) + np.float32(acc[3] + acc[7])))
    L = oracle.lib()
    import ctypes
    wp = np.ascontiguousarray(w.reshape(-1))
    ap = np.ascontiguousarray(a.reshape(-1))
    got = L.ceo_dot_q8_0(k, wp.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), ap.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    assert np.float32(got) == ref


def test_route_semantics(oracle):
    lg = np.array([[0.1, 0.5, 0.5, -1.0], [3.0, 2.0, 1.0, 0.0]], np.float32)
    ids, w, p = oracle.route(lg, 2)
    assert ids.tolist() == [[1, 2], [0, 1]]         # ties -> lower index first
    assert np.allclose(p.sum(1), 1.0, atol=1e-6)
    assert np.array_equal(w, np.take_along_axis(p, ids, 1))  # gate weights not renormalised


def test_pool_l2_epsilon(oracle):
    h = np.zeros((3, 8), np.float32)
    out = oracle.pool_l2(h, np.array([0, 3], np.int32))
    assert np.all(out == 0)


def test_q8_0_dot_avx2_equals_scalar(oracle):
    """The oracle's AVX2 Q8_0 dot (the host fast path) gives the scalar lane form's bits,
    including blocks at the int8 limits, zero blocks and sign mixes."""
    import ctypes
    rng = np.random.default_rng(5)
    L = oracle.lib()
    up = ctypes.POINTER(ctypes.c_uint8)
    for trial in range(200):
        k = 32 * int(rng.integers(1, 97))
        w = np.zeros((k // 32, 34), np.uint8)
        a = np.zeros((k // 32, 34), np.uint8)
        for blk in (w, a):
            blk[:, :2] = (rng.uniform(1e-4, 2.0, k // 32).astype(np.float16)).view(np.uint8).reshape(-1, 2)
            q = rng.integers(-127, 128, (k // 32, 32)).astype(np.int8)
            if trial % 4 == 0:
                q[0] = 127 * np.sign(rng.standard_normal(32)).astype(np.int8)  # the limits
            if trial % 5 == 0:
                q[-1] = 0
            blk[:, 2:] = q.view(np.uint8)
        wp, ap = np.ascontiguousarray(w.reshape(-1)), np.ascontiguousarray(a.reshape(-1))
        fast = L.ceo_dot_q8_0(k, wp.ctypes.data_as(up), ap.ctypes.data_as(up))
        slow = L.ceo_dot_q8_0_scalar(k, wp.ctypes.data_as(up), ap.ctypes.data_as(up))
        assert np.float32(fast).tobytes() == np.float32(slow).tobytes(), trial


@pytest.mark.parametrize("fmt", ["q8_0", "q4_k"])
def test_matmul_blocked_equals_per_dot(oracle, fmt):
    """The ggml-mode matmul forms several dots per pass (Q8_0: two weight x two activation
    rows; Q4_K: one weight row x four activation rows) and gives every output the bits of
    its own ceo_dot_q8_0 / ceo_dot_q4_k (+ bias), for odd row counts and tile edges."""
    import ctypes
    from crispembed_b200.gguf_io import GGML_Q4_K, GGML_Q8_0
    rng = np.random.default_rng(11)
    L = oracle.lib()
    up = ctypes.POINTER(ctypes.c_uint8)
    if fmt == "q8_0":
        t, qz, dot, act = GGML_Q8_0, quant.quantize_q8_0, L.ceo_dot_q8_0, oracle.quant_act_q8_0
        shapes = ((1, 1, 32), (3, 5, 64), (33, 31, 96), (64, 66, 768), (37, 70, 256))
    else:
        def act(v):
            out = np.zeros(v.size // 256 * 292, np.uint8)
            vv = np.ascontiguousarray(v, dtype=np.float32)
            L.ceo_quant_act_q8_k(vv.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), v.size, out.ctypes.data_as(up))
            return out
        t, qz, dot = GGML_Q4_K, quant.quantize_q4_k, L.ceo_dot_q4_k
        shapes = ((1, 1, 256), (3, 5, 512), (34, 31, 256), (67, 40, 768))
    for m_rows, n_out, k in shapes:
        w = qz((rng.standard_normal((n_out, k)) * 0.05).astype(np.float32))
        x = rng.standard_normal((m_rows, k)).astype(np.float32)
        bias = rng.standard_normal(n_out).astype(np.float32)
        got = oracle.matmul(t, w, n_out, k, x, oracle.GGML, bias)
        wrows = np.ascontiguousarray(w).reshape(n_out, -1)
        want = np.empty_like(got)
        for m in range(m_rows):
            a = np.ascontiguousarray(act(x[m]))
            for n in range(n_out):
                wr = np.ascontiguousarray(wrows[n])
                s = np.float32(dot(k, wr.ctypes.data_as(up), a.ctypes.data_as(up)))
                want[m, n] = s + bias[n]
        assert got.tobytes() == want.tobytes(), (fmt, m_rows, n_out, k)


def test_q4_k_dot_avx2_equals_scalar(oracle):
    """The oracle's AVX2 Q4_K x Q8_K dot gives the scalar lane form's bits (random
    super-blocks with every 4-bit value, the 6-bit scale extremes and full-range Q8_K)."""
    import ctypes
    rng = np.random.default_rng(6)
    L = oracle.lib()
    up = ctypes.POINTER(ctypes.c_uint8)
    for trial in range(100):
        k = 256 * int(rng.integers(1, 13))
        w = rng.integers(0, 256, (k // 256, 144)).astype(np.uint8)
        w[:, :4] = rng.uniform(1e-4, 1.0, (k // 256, 2)).astype(np.float16).view(np.uint8).reshape(-1, 4)
        x = rng.standard_normal(k).astype(np.float32) * np.float32(rng.uniform(0.1, 10))
        a = np.zeros(k // 256 * 292, np.uint8)
        L.ceo_quant_act_q8_k(x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), k, a.ctypes.data_as(up))
        wp = np.ascontiguousarray(w.reshape(-1))
        fast = L.ceo_dot_q4_k(k, wp.ctypes.data_as(up), a.ctypes.data_as(up))
        slow = L.ceo_dot_q4_k_scalar(k, wp.ctypes.data_as(up), a.ctypes.data_as(up))
        assert np.float32(fast).tobytes() == np.float32(slow).tobytes(), trial
