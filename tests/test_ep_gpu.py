"""Expert parallelism (ceb_ep_*, ceb_moe_ffn_ep, ceb_ep_attach) against the
single-GPU path.

The exchange keeps every row's arithmetic (same GEMM K-loop order, same combine
slot order), so results must be bit-identical to one GPU.
  * One GPU: a one-rank exchange sends every row through the exchange kernels
    (count publication, dispatch into the receive buffer, return into the ret
    buffer, flag waits) and back.
  * Two GPUs or more (skipped otherwise): ranks run as processes through
    torch.distributed.run (tests/ep_worker.py), each checks its own shard; a rank
    that never joins makes the others' bounded waits expire with status 5 and
    code 0x107 (no GPU fault: the waits give up and return).
"""
import glob
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from crispembed_b200 import synth

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = {
    "q8_e4": dict(T=300, d=256, n_experts=4, top_k=2, ffn=512, wtype=8, router_wtype=8, zipf_s=None, with_bias=True),
    "q4k_e8_zipf": dict(T=700, d=768, n_experts=8, top_k=2, ffn=3072, wtype=12, router_wtype=0, zipf_s=1.2,
                        with_bias=False),
    "q4k_e32_k4": dict(T=200, d=1024, n_experts=32, top_k=4, ffn=1536, wtype=12, router_wtype=0, zipf_s=1.5,
                       with_bias=False),
    "one_token": dict(T=1, d=256, n_experts=4, top_k=2, ffn=256, wtype=8, router_wtype=8, zipf_s=None,
                      with_bias=True),
}


@pytest.mark.parametrize("name", list(CASES))
def test_one_rank_exchange_matches_moe_ffn(cuda, name):
    import torch
    from crispembed_b200 import binding
    cfg = dict(CASES[name])
    T = cfg.pop("T")
    inp = synth.make_moe_op_inputs(T, seed=17, **cfg)
    layer = binding.MoELayer(inp.d, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype,
                             inp.fc1_raw, inp.fc2_raw, inp.bias)
    ep = binding.ExpertParallel(0, 1, inp.n_experts, inp.top_k, inp.d, inp.ffn, T)
    x = torch.from_numpy(inp.x).to(cuda).to(torch.bfloat16)
    ws = torch.empty(layer.workspace_size(T), dtype=torch.uint8, device=cuda)
    y = torch.empty((T, inp.d), dtype=torch.float32, device=cuda)
    layer.forward(x, y, ws)
    binding.sync_check()
    ref = y.cpu().numpy()
    for _ in range(3):  # epochs and count-matrix parity advance
        y_ep = torch.full((T, inp.d), float("nan"), dtype=torch.float32, device=cuda)
        layer.forward_ep(ep, x, y_ep, ws)
        binding.sync_check()
        assert np.array_equal(y_ep.cpu().numpy(), ref)
    ep.close()
    layer.close()


def test_one_rank_exchange_encoder_matches(cuda, tiny_model):
    from crispembed_b200 import binding
    ids, lens = synth.ids_ragged(10, 1, 128, seed=6, hi=1000)
    ref_ctx = binding.CrispEmbed(tiny_model)
    ep_ctx = binding.CrispEmbed(tiny_model)
    h = ep_ctx.hparams
    ep = binding.ExpertParallel(0, 1, h.n_experts, h.n_experts_per_tok, h.n_embd, synth.tiny_spec().expert_ffn,
                                int(lens.sum()))
    ep_ctx.attach_ep(ep)
    ref = ref_ctx.encode_ids(ids, lens)
    for _ in range(2):
        assert np.array_equal(ep_ctx.encode_ids(ids, lens), ref)
    ep_ctx.close()
    ref_ctx.close()
    ep.close()


def test_exchange_rejects_mismatched_block(cuda, tiny_model):
    from crispembed_b200 import binding
    ctx = binding.CrispEmbed(tiny_model)
    h = ctx.hparams
    ep = binding.ExpertParallel(0, 1, h.n_experts * 2, h.n_experts_per_tok, h.n_embd, 512, 256)
    with pytest.raises(binding.CrispEmbedError, match="does not match"):
        ctx.attach_ep(ep)
    ctx.close()
    ep.close()


def test_ep_create_rejects_bad_split(cuda):
    from crispembed_b200 import binding
    with pytest.raises(binding.CrispEmbedError):
        binding.ExpertParallel(0, 3, 8, 2, 256, 512, 64)  # 8 experts do not split over 3 ranks


def _n_gpus():
    import torch
    return torch.cuda.device_count()


def _launch(n, mode, model_path, tmp_path, timeout=300):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.path.dirname(HERE))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}", "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(HERE, "ep_worker.py"), mode, model_path,
           str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout)
    files = sorted(glob.glob(os.path.join(str(tmp_path), "rank*.json")))
    assert r.returncode == 0 and len(files) == n, (r.returncode, r.stdout[-2000:], r.stderr[-4000:])
    return [json.load(open(f)) for f in files]


@pytest.mark.skipif("not __import__('torch').cuda.is_available() or __import__('torch').cuda.device_count() < 2")
def test_two_rank_exchange_op_bit_identical(cuda, tmp_path):
    res = _launch(2, "op", "-", tmp_path)
    for r in res:
        assert "error" not in r, r
        cases = {k: v for k, v in r.items() if isinstance(v, dict)}
        assert len(cases) == 4, r
        for name, v in cases.items():
            assert v["equal"], (r["rank"], name, v)
    assert any(v.get("tokens") == 0 for v in res[-1].values() if isinstance(v, dict))


@pytest.mark.skipif("not __import__('torch').cuda.is_available() or __import__('torch').cuda.device_count() < 2")
def test_two_rank_exchange_encoder_bit_identical(cuda, tiny_model, tmp_path):
    res = _launch(2, "encoder", tiny_model, tmp_path)
    for r in res:
        assert "error" not in r, r
        assert r["encoder"]["equal"], r


@pytest.mark.skipif("not __import__('torch').cuda.is_available() or __import__('torch').cuda.device_count() < 2")
def test_silent_rank_makes_peer_waits_expire(cuda, tmp_path):
    res = _launch(2, "timeout", "-", tmp_path)
    assert "error" not in res[0] and "error" not in res[1], res
    t = res[0]["timeout"]
    assert t["raised"] and "0x" in t["message"] and "107" in t["message"], t


@pytest.mark.skipif("not __import__('torch').cuda.is_available() or __import__('torch').cuda.device_count() < 4")
def test_all_gpu_exchange_op_bit_identical(cuda, tmp_path):
    """Every visible GPU (4 or 8) as one rank: the cases whose expert count splits."""
    import torch
    n = 8 if torch.cuda.device_count() >= 8 else 4
    res = _launch(n, "op", "-", tmp_path)
    for r in res:
        assert "error" not in r, r
        cases = {k: v for k, v in r.items() if isinstance(v, dict)}
        assert cases, r
        for name, v in cases.items():
            assert v["equal"], (r["rank"], name, v)
