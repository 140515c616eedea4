"""Time one kernel of the library in isolation (CUDA events, inputs resident).

    python -m crispembed_b200.kernel_bench gemm --type q8_0 --m 16384 --n 3072 --k 768 [--gelu] [--f16-out]
    python -m crispembed_b200.kernel_bench moe --T 65536 --type q4_k --zipf 1.2
    python -m crispembed_b200.kernel_bench route_ln --T 70825 --router-type q8_0
    python -m crispembed_b200.kernel_bench attn --seqs 256 [--impl mma|tc]
    python -m crispembed_b200.kernel_bench pool --seqs 256
    python -m crispembed_b200.kernel_bench encode --seqs 256
    python -m crispembed_b200.kernel_bench cublas --m 70825 --n 3072 --k 768
    torchrun --nproc-per-node N -m crispembed_b200.kernel_bench a2a --tokens 131072

Used for the roofline numbers of single kernels and as the command that ncu
captures (small cases: a few launches, a few GB at most).  Prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import sys

import numpy as np

TYPES = {"q8_0": 8, "q4_k": 12, "f16": 1, "f32": 0}


def _peaks():
    import os
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return json.load(f), "measured"
    except OSError:
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}, "fallback"


def bench_gemm(a):
    import torch

    from . import binding, quant
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((a.n, a.k), dtype=np.float32) * 0.02).astype(np.float32)
    lin = binding.Linear(TYPES[a.type], quant.quantize(w, TYPES[a.type]), a.n, a.k)
    x = torch.randn((a.m, a.k), device="cuda", dtype=torch.float16)
    bias = torch.randn((a.n,), device="cuda", dtype=torch.float32) * 0.02 if a.bias else None
    out = torch.empty((a.m, a.n), device="cuda", dtype=torch.float16 if a.f16_out else torch.float32)
    for _ in range(a.warmup):
        lin(x, out=out, bias=bias, gelu=a.gelu, out_f16=a.f16_out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        lin(x, out=out, bias=bias, gelu=a.gelu, out_f16=a.f16_out)
    e1.record()
    torch.cuda.synchronize()
    binding.sync_check()
    ms = e0.elapsed_time(e1) / a.iters
    flops = 2.0 * a.m * a.n * a.k
    pk, src = _peaks()
    tf = flops / (ms / 1e3) / 1e12
    lin.close()
    return {"kernel": "gemm", "type": a.type, "m": a.m, "n": a.n, "k": a.k, "gelu": a.gelu, "f16_out": a.f16_out,
            "ms": ms, "tflops": tf, "frac_of_peak": tf / pk["bf16_tflops"], "peak_source": src}


def bench_moe(a):
    import torch

    from . import binding, synth
    inp = synth.make_moe_op_inputs(a.T, d=a.d, n_experts=a.E, top_k=a.topk, ffn=a.F, wtype=TYPES[a.type],
                                   router_wtype=TYPES[a.router_type], zipf_s=a.zipf or None, seed=0)
    layer = binding.MoELayer(inp.d, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype,
                             inp.fc1_raw, inp.fc2_raw, inp.bias)
    x = torch.from_numpy(inp.x).cuda().to(torch.float32 if a.f32_input else torch.bfloat16)
    y = torch.empty((a.T, a.d), dtype=torch.float32, device="cuda")
    ws = torch.empty(layer.workspace_size(a.T), dtype=torch.uint8, device="cuda")
    for _ in range(a.warmup):
        layer.forward(x, y, ws)
    torch.cuda.synchronize()
    binding.profile_enable(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        layer.forward(x, y, ws)
    e1.record()
    torch.cuda.synchronize()
    prof = binding.profile_read()
    binding.profile_enable(False)
    ms = e0.elapsed_time(e1) / a.iters
    layer.close()
    flops = 2.0 * 2 * a.T * a.topk * a.d * a.F
    return {"kernel": "moe_ffn", "T": a.T, "type": a.type, "E": a.E, "k": a.topk, "ms": ms,
            "tokens_per_s": a.T / (ms / 1e3), "tflops": flops / (ms / 1e3) / 1e12,
            "breakdown_ms": {k: v["ms"] / a.iters for k, v in prof.items()}}


def bench_route_ln(a):
    """ceb_moe_route_ln over T rows: residual + LayerNorm + router in one pass.
    Algorithmic bytes: res and y read (fp32), out written in fp32 and fp16."""
    import numpy as np
    import torch

    from . import binding, synth
    inp = synth.make_moe_op_inputs(256, d=a.d, n_experts=a.E, top_k=a.topk, ffn=a.F, wtype=TYPES[a.type],
                                   router_wtype=TYPES[a.router_type], zipf_s=None, seed=0)
    layer = binding.MoELayer(inp.d, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype,
                             inp.fc1_raw, inp.fc2_raw, inp.bias)
    g = torch.Generator(device="cuda").manual_seed(1)
    res = torch.randn((a.T, a.d), device="cuda", generator=g)
    y = torch.randn((a.T, a.d), device="cuda", generator=g)
    gamma = torch.ones(a.d, device="cuda")
    beta = torch.zeros(a.d, device="cuda")
    out = torch.empty_like(res)
    out16 = torch.empty((a.T, a.d), dtype=torch.float16, device="cuda")
    ws = torch.empty(layer.workspace_size(a.T), dtype=torch.uint8, device="cuda")
    run = lambda: layer.route_ln(res, y, out, ws, gamma=gamma, beta=beta, eps=1e-12, out16=out16)  # noqa: E731
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    ms_all = []
    for _ in range(a.iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        ms_all.append(e0.elapsed_time(e1))
    layer.close()
    ms = float(np.median(ms_all))
    nbytes = a.T * a.d * (4 + 4 + 4 + 2)
    peaks, src = _peaks()
    pk = peaks["hbm_gbs"]
    return {"kernel": "moe_route_ln", "T": a.T, "d": a.d, "E": a.E, "router_type": a.router_type, "ms": ms,
            "gbs": nbytes / (ms / 1e3) / 1e9, "frac_of_hbm": nbytes / (ms / 1e3) / 1e9 / pk, "peak_source": src}


def bench_attn(a):
    """Varlen attention (ceb_attention_forward) on config-2 lengths: n_seqs sequences,
    lengths U[lo, hi] seed 2, d = 64 * n_head, fp16 qkv N(0,1).  FLOPs: 4*L^2*d per
    sequence (QK^T and PV)."""
    import os

    import numpy as np
    import torch

    from . import binding
    os.environ.pop("CEB_ATTN_TC", None)
    os.environ.pop("CEB_ATTN_MMA", None)
    if a.impl == "tc":
        os.environ["CEB_ATTN_TC"] = "1"
    elif a.impl == "mma":
        os.environ["CEB_ATTN_MMA"] = "1"
    rng = np.random.default_rng(2)
    lens = rng.integers(a.lo, a.hi + 1, size=a.seqs).astype(np.int32)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).cuda()
    rows, d = int(lens.sum()), 64 * a.heads
    g = torch.Generator(device="cuda").manual_seed(0)
    qkv = torch.randn((rows, 3 * d), device="cuda", generator=g).to(torch.float16)
    for _ in range(a.warmup):
        binding.attention(qkv, cu, a.heads, int(lens.max()))
    torch.cuda.synchronize()
    ms_all = []
    for _ in range(a.iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        binding.attention(qkv, cu, a.heads, int(lens.max()))
        e1.record()
        torch.cuda.synchronize()
        ms_all.append(e0.elapsed_time(e1))
    ms = float(np.median(ms_all))
    flops = 4.0 * float((lens.astype(np.float64) ** 2).sum()) * d
    return {"kernel": "attention", "impl": a.impl, "seqs": a.seqs, "tokens": rows, "heads": a.heads, "ms": ms,
            "tflops": flops / (ms / 1e3) / 1e12}


def _c2_lens(n_seqs):
    from . import synth
    _, lens = synth.config_ids(2)
    return lens[:n_seqs]


def bench_pool(a):
    """Mean pool + L2 (ceb_pool_l2) over config-2 lengths: hidden [M, d] fp32.
    Algorithmic bytes: every hidden value read once (d*4 per token), rows written."""
    import torch

    from . import binding
    lens = _c2_lens(a.seqs)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).cuda()
    M = int(lens.sum())
    g = torch.Generator(device="cuda").manual_seed(0)
    hidden = torch.randn((M, a.d), device="cuda", generator=g)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # larger than L2
    for _ in range(a.warmup):
        binding.pool_l2(hidden, cu)
    torch.cuda.synchronize()
    ms_all = []
    for _ in range(a.iters):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        binding.pool_l2(hidden, cu)
        e1.record()
        torch.cuda.synchronize()
        ms_all.append(e0.elapsed_time(e1))
    binding.sync_check()
    ms = float(np.median(ms_all))
    nbytes = (M + len(lens)) * a.d * 4
    pk, src = _peaks()
    return {"kernel": "pool_l2", "seqs": len(lens), "tokens": M, "ms": ms, "gbs": nbytes / (ms / 1e3) / 1e9,
            "frac_of_hbm": nbytes / (ms / 1e3) / 1e9 / pk["hbm_gbs"], "peak_source": src}


def bench_encode(a):
    """The whole config-2 encoder on the first n_seqs sequences (device ids), the
    command ncu captures the encoder's row-wise kernels from."""
    import os
    import sys as _sys

    import torch

    from . import binding, synth
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    _sys.path.insert(0, root)
    import bench
    ids, lens = synth.config_ids(2)
    lens = lens[:a.seqs]
    ids = np.ascontiguousarray(ids[:int(lens.sum())])
    m = binding.CrispEmbed(bench.model_path(0))
    d_ids = torch.from_numpy(ids).cuda()
    out = torch.empty((len(lens), m.dim), dtype=torch.float32, device="cuda")
    for _ in range(a.warmup):
        m.encode_ids_device(d_ids, lens, out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        m.encode_ids_device(d_ids, lens, out)
    e1.record()
    torch.cuda.synchronize()
    binding.sync_check()
    ms = e0.elapsed_time(e1) / a.iters
    m.close()
    return {"kernel": "encode", "seqs": len(lens), "tokens": int(lens.sum()), "ms": ms,
            "tokens_per_s": int(lens.sum()) / (ms / 1e3)}


def bench_cublas(a):
    """torch.matmul (cuBLAS) on the same shape as a linear layer: fp16 operands, fp32
    accumulation, fp16 output -- the library-GEMM bar for ceb_gemm_pair_kernel."""
    import torch
    x = torch.randn((a.m, a.k), device="cuda", dtype=torch.float16)
    w = torch.randn((a.n, a.k), device="cuda", dtype=torch.float16) * 0.02
    for _ in range(a.warmup):
        y = torch.matmul(x, w.t())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        y = torch.matmul(x, w.t())
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    flops = 2.0 * a.m * a.n * a.k
    pk, src = _peaks()
    tf = flops / (ms / 1e3) / 1e12
    del y
    return {"kernel": "cublas_fp16", "m": a.m, "n": a.n, "k": a.k, "ms": ms, "tflops": tf,
            "frac_of_peak": tf / pk["bf16_tflops"], "peak_source": src}


def bench_a2a(a):
    """NCCL all-to-all of one MoE block's exchange at the config-4 shape: every rank
    holds `tokens` tokens x top_k fp16 rows of d values and sends an equal share to
    every rank (itself included), dispatch then return, with all_to_all_single -- the
    library collective the expert-parallel peer stores replace.  Rank 0 prints the
    time per exchange (max over ranks) and the bytes each rank sends to other ranks
    per second."""
    import datetime
    import os

    import torch
    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
    rows = a.tokens * a.topk // world * world
    x = torch.randn((rows, a.d), device="cuda", dtype=torch.float16)
    y = torch.empty_like(x)
    z = torch.empty_like(x)
    for _ in range(a.warmup):
        dist.all_to_all_single(y, x)
        dist.all_to_all_single(z, y)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        dist.all_to_all_single(y, x)  # dispatch
        dist.all_to_all_single(z, y)  # return
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / a.iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    off_rank = 2 * rows * a.d * 2 * (world - 1) / world  # bytes each rank sends to other ranks per exchange
    r = {"kernel": "nccl_all_to_all", "world": world, "rows_per_rank": rows, "d": a.d,
         "ms_per_exchange": float(ms.item()), "off_rank_bytes": off_rank,
         "off_rank_gbs_per_rank": off_rank / (float(ms.item()) / 1e3) / 1e9}
    dist.barrier()
    dist.destroy_process_group()
    return r if rank == 0 else None


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--type", default="q8_0", choices=list(TYPES))
    g.add_argument("--m", type=int, default=16384)
    g.add_argument("--n", type=int, default=3072)
    g.add_argument("--k", type=int, default=768)
    g.add_argument("--gelu", action="store_true")
    g.add_argument("--bias", action="store_true")
    g.add_argument("--f16-out", action="store_true")
    g.add_argument("--iters", type=int, default=20)
    g.add_argument("--warmup", type=int, default=3)
    m = sub.add_parser("moe")
    m.add_argument("--T", type=int, default=65536)
    m.add_argument("--d", type=int, default=768)
    m.add_argument("--E", type=int, default=8)
    m.add_argument("--topk", type=int, default=2)
    m.add_argument("--F", type=int, default=3072)
    m.add_argument("--type", default="q4_k", choices=list(TYPES))
    m.add_argument("--zipf", type=float, default=1.2)
    m.add_argument("--router-type", default="f32", choices=["f32", "q8_0"])
    m.add_argument("--iters", type=int, default=10)
    m.add_argument("--f32-input", action="store_true")
    m.add_argument("--warmup", type=int, default=3)
    r = sub.add_parser("route_ln")
    r.add_argument("--T", type=int, default=70825)
    r.add_argument("--d", type=int, default=768)
    r.add_argument("--E", type=int, default=8)
    r.add_argument("--topk", type=int, default=2)
    r.add_argument("--F", type=int, default=256)
    r.add_argument("--type", default="q8_0", choices=list(TYPES))
    r.add_argument("--router-type", default="q8_0", choices=["f32", "q8_0"])
    r.add_argument("--iters", type=int, default=20)
    r.add_argument("--warmup", type=int, default=3)
    t = sub.add_parser("attn")
    t.add_argument("--seqs", type=int, default=256)
    t.add_argument("--lo", type=int, default=32)
    t.add_argument("--hi", type=int, default=512)
    t.add_argument("--heads", type=int, default=12)
    t.add_argument("--impl", choices=["fa", "mma", "tc"], default="fa",
                   help="fa: the default single-CTA tcgen05 kernel; mma: mma.sync; tc: the CTA-pair tcgen05 kernel")
    t.add_argument("--iters", type=int, default=20)
    t.add_argument("--warmup", type=int, default=3)
    p = sub.add_parser("pool")
    p.add_argument("--seqs", type=int, default=256)
    p.add_argument("--d", type=int, default=768)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    e = sub.add_parser("encode")
    e.add_argument("--seqs", type=int, default=256)
    e.add_argument("--iters", type=int, default=3)
    e.add_argument("--warmup", type=int, default=1)
    c = sub.add_parser("cublas")
    c.add_argument("--m", type=int, default=70825)
    c.add_argument("--n", type=int, default=3072)
    c.add_argument("--k", type=int, default=768)
    c.add_argument("--iters", type=int, default=20)
    c.add_argument("--warmup", type=int, default=3)
    n = sub.add_parser("a2a")
    n.add_argument("--tokens", type=int, default=131072)
    n.add_argument("--topk", type=int, default=2)
    n.add_argument("--d", type=int, default=768)
    n.add_argument("--iters", type=int, default=20)
    n.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    if a.what == "a2a":
        r = bench_a2a(a)
        if r:
            print(json.dumps(r), flush=True)
        return 0
    r = {"gemm": bench_gemm, "moe": bench_moe, "route_ln": bench_route_ln, "attn": bench_attn, "pool": bench_pool,
         "encode": bench_encode, "cublas": bench_cublas}[a.what](a)
    print(json.dumps(r), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
