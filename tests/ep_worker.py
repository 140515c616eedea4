"""One rank of the multi-GPU expert-parallel tests (tests/test_ep_gpu.py starts
it through torch.distributed.run, one process per GPU).

Modes (argv: mode model_path out_dir):
  op       ceb_moe_ffn_ep on this rank's token slice vs ceb_moe_ffn on the same
           slice on this GPU, bit for bit, for several block shapes (one with no
           tokens on the last rank);
  encoder  an encoder context with the exchange attached vs a plain one on this
           rank's sequences, bit for bit, twice (epochs advance across calls);
  timeout  the last rank never joins the exchange: the other ranks' bounded waits
           expire and ceb_sync_check reports status 5 with code 0x107.
Each rank writes out_dir/rank<r>.json.
"""
import datetime
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

OP_CASES = [
    dict(name="q8_e4", T=600, d=256, n_experts=4, top_k=2, ffn=512, wtype=8, router_wtype=8, zipf_s=None,
         with_bias=True),
    dict(name="q4k_e8_zipf", T=900, d=768, n_experts=8, top_k=2, ffn=3072, wtype=12, router_wtype=0, zipf_s=1.2,
         with_bias=False),
    dict(name="q4k_e32_k4", T=300, d=1024, n_experts=32, top_k=4, ffn=1536, wtype=12, router_wtype=0, zipf_s=1.5,
         with_bias=False),
    dict(name="last_rank_empty", T=200, d=256, n_experts=8, top_k=2, ffn=256, wtype=8, router_wtype=8, zipf_s=None,
         with_bias=True, empty_last=True),
]


def _slice(T, rank, world, empty_last=False):
    n = world - 1 if (empty_last and world > 1) else world
    if empty_last and rank == world - 1 and world > 1:
        return T, T
    base, extra = divmod(T, n)
    t0 = rank * base + min(rank, extra)
    return t0, t0 + base + (1 if rank < extra else 0)


def run_op(rank, world, res):
    import torch

    from crispembed_b200 import binding, synth
    from crispembed_b200.dist import connect_expert_parallel
    for case in OP_CASES:
        cfg = dict(case)
        name, T, empty_last = cfg.pop("name"), cfg.pop("T"), cfg.pop("empty_last", False)
        if cfg["n_experts"] % world:
            continue
        inp = synth.make_moe_op_inputs(T, seed=21, **cfg)
        t0, t1 = _slice(T, rank, world, empty_last)
        layer = binding.MoELayer(inp.d, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw,
                                 inp.wtype, inp.fc1_raw, inp.fc2_raw, inp.bias)
        ep = binding.ExpertParallel(rank, world, inp.n_experts, inp.top_k, inp.d, inp.ffn, T)
        connect_expert_parallel(ep)
        ep.set_timeout_ms(20000)
        n = t1 - t0
        x = torch.from_numpy(np.ascontiguousarray(inp.x[t0:t1])).cuda().to(torch.bfloat16)
        if n == 0:
            x = torch.empty((0, inp.d), dtype=torch.bfloat16, device="cuda")
        ws = torch.empty(layer.workspace_size(max(n, 1)), dtype=torch.uint8, device="cuda")
        y_ep = torch.full((max(n, 1), inp.d), float("nan"), dtype=torch.float32, device="cuda")
        outs = []
        for _ in range(2):  # two exchanges: the epoch and the count-matrix parity advance
            layer.forward_ep(ep, x, y_ep, ws)
            binding.sync_check()
            outs.append(y_ep[:n].cpu().numpy().copy())
        ok = bool(np.array_equal(outs[0], outs[1]))
        if n > 0:
            y = torch.empty((n, inp.d), dtype=torch.float32, device="cuda")
            layer.forward(x, y, ws)
            binding.sync_check()
            ref = y.cpu().numpy()
            ok = ok and bool(np.array_equal(outs[0], ref))
            res[name] = {"tokens": n, "equal": ok, "maxdiff": float(np.abs(outs[0] - ref).max())}
        else:
            res[name] = {"tokens": 0, "equal": ok, "maxdiff": 0.0}
        import torch.distributed as dist
        dist.barrier()
        ep.close()
        layer.close()
        dist.barrier()


def run_encoder(rank, world, model_path, res):
    from crispembed_b200 import binding, synth
    from crispembed_b200.dist import connect_expert_parallel, shard_sequences
    ids, lens = synth.ids_ragged(24, 1, 128, seed=9, hi=1000)
    s0, cnt, tok0, ntok = shard_sequences(lens, rank, world)
    my_ids, my_lens = ids[tok0:tok0 + ntok], lens[s0:s0 + cnt]
    ref_ctx = binding.CrispEmbed(model_path)
    ep_ctx = binding.CrispEmbed(model_path)
    h = ep_ctx.hparams
    ffn = synth.tiny_spec().expert_ffn
    ep = binding.ExpertParallel(rank, world, h.n_experts, h.n_experts_per_tok, h.n_embd, ffn, int(lens.sum()))
    connect_expert_parallel(ep)
    ep.set_timeout_ms(20000)
    ep_ctx.attach_ep(ep)
    ref = ref_ctx.encode_ids(my_ids, my_lens)
    got = [ep_ctx.encode_ids(my_ids, my_lens) for _ in range(2)]
    res["encoder"] = {"seqs": int(cnt), "equal": bool(np.array_equal(got[0], ref) and np.array_equal(got[1], ref)),
                      "maxdiff": float(np.abs(got[0] - ref).max())}
    import torch.distributed as dist
    dist.barrier()
    ep_ctx.close()
    ref_ctx.close()
    ep.close()
    dist.barrier()


def run_timeout(rank, world, res):
    import torch
    import torch.distributed as dist

    from crispembed_b200 import binding, synth
    from crispembed_b200.dist import connect_expert_parallel
    inp = synth.make_moe_op_inputs(64, d=256, n_experts=4, top_k=2, ffn=256, wtype=8, router_wtype=8, zipf_s=None,
                                   seed=3, with_bias=False)
    layer = binding.MoELayer(inp.d, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype,
                             inp.fc1_raw, inp.fc2_raw, inp.bias)
    ep = binding.ExpertParallel(rank, world, inp.n_experts, inp.top_k, inp.d, inp.ffn, 64)
    connect_expert_parallel(ep)
    ep.set_timeout_ms(500)
    if rank != world - 1:  # the last rank never joins: its flags are never released
        x = torch.from_numpy(inp.x).cuda().to(torch.bfloat16)
        y = torch.empty((64, inp.d), dtype=torch.float32, device="cuda")
        ws = torch.empty(layer.workspace_size(64), dtype=torch.uint8, device="cuda")
        layer.forward_ep(ep, x, y, ws)
        try:
            binding.sync_check()
            res["timeout"] = {"raised": False}
        except binding.CrispEmbedError as e:
            res["timeout"] = {"raised": True, "message": str(e)}
        torch.cuda.synchronize()
    else:
        res["timeout"] = {"skipped_exchange": True}
    dist.barrier()  # the silent rank keeps its region mapped until the others are done
    ep.close()
    layer.close()
    dist.barrier()


def main():
    mode, model_path, out_dir = sys.argv[1:4]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    res = {"rank": rank, "world": world}
    try:
        if mode == "op":
            run_op(rank, world, res)
        elif mode == "encoder":
            run_encoder(rank, world, model_path, res)
        elif mode == "timeout":
            run_timeout(rank, world, res)
    except Exception as e:  # reported through the result file
        res["error"] = repr(e)
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
