#!/usr/bin/env python
"""MoE-encoder throughput on B200 -- one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4|c5] [--no-ep] [--no-ops] [--no-cpu-baseline]

Workloads (inputs synthetic and seeded, weights random-init
of the nomic-embed-text-v2-moe architecture, see crispembed_b200/synth.py):
  c2 (default)  NomicBERT-MoE encoder, Q8_0 GGUF, 256 sequences with lengths
                U[32,512] (seed 2, 70825 tokens) per step; one step = embed,
                12 layers (6 MoE), mean-pool + L2 of the whole batch.
  c3            the isolated MoE FFN operator, Q4_K experts, T=65536 bf16 tokens,
                Zipf(1.2) expert loads (seed 0); T=512 and 8192 as other_cases.
  c4            the expert-parallel encoder alone (see below).
  c5            wide routing through the same operator: d=1024, E=32, top-4,
                F=1536, Q4_K, T=131072, balanced; Zipf(1.5) as other_cases.

value  : tokens/s of the whole job with ids already in HBM (device entry point,
         CUDA events on the launching stream, max over ranks).
e2e    : same metric through the host-buffer C-ABI call (crispembed_encode_ids_batch:
         ids copied host->device and embeddings device->host inside the timed call).
Multi-GPU (torchrun): data-parallel replicas, every rank encodes its own copy of
the config-2 batch (weak scaling, no collective on the data path).  The line also
carries "expert_parallel": BASELINE config 4 (512 x 512 tokens per step for the
whole job, sequences sharded over the ranks and the MoE experts split over them,
exchange by the library's own peer-memory kernels), at every N (N=1 runs the
exchange with itself).  --workload c4 prints that measurement as the main line.
At N=1 the line also carries "moe_operator": the c3 and c5 workloads (every case
of each: c3 at T = 65536, 512, 8192; c5 balanced and Zipf 1.5), each with its
own e2e, roofline and CPU baseline; --workload c3|c5 prints one as the main line.
Rooflines: "roofline" covers every launch of the dominant kernel (the tcgen05 GEMM
of all linear layers), "roofline_moe_grouped_gemm" the grouped expert GEMMs alone;
all use the measured sustained bf16 peak, with the burst fraction beside it.
--impl reference: the CPU restatement of the reference's ggml CPU path (oracle/, its
timing build: the C library's expf / erff as ggml calls them,
the reference itself cannot be built here) on all host threads, bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE-encoder tokens/s/GPU (Q8_0, 1/2/4/8 B200); grouped-GEMM TC util %"
CACHE = os.environ.get("CEB_BENCH_CACHE", "/tmp/crispembed_b200_bench")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def model_path(rank_local: int) -> str:
    """config-2 model (Q8_0), written once per box; other local ranks wait for it."""
    from crispembed_b200 import synth
    os.makedirs(CACHE, exist_ok=True)
    path = os.path.join(CACHE, "nomic_moe_q8_0_seed0.gguf")
    if os.path.exists(path):
        return path
    if rank_local == 0:
        tmp = path + f".tmp{os.getpid()}"
        t = time.time()
        synth.write_model(tmp, synth.nomic_moe_spec())
        os.replace(tmp, path)
        log(f"[bench] wrote {path} in {time.time() - t:.1f}s")
    else:
        t0 = time.time()
        while not os.path.exists(path):
            if time.time() - t0 > 600:
                raise RuntimeError("timed out waiting for the model file")
            time.sleep(1.0)
    return path


class ClockSampler:
    """nvidia-smi SM clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout_s: float = 10.0):
        """Block until nvidia-smi has delivered its first sample (it takes ~0.5 s to start)."""
        t0 = time.time()
        while self.proc and not self.lines and time.time() - t0 < timeout_s and self.proc.poll() is None:
            time.sleep(0.02)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(path, ids, lens, budget_s=15.0):
    """Oracle (CPU restatement of ggml's CPU path) on the first sequences of the batch."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.use_timing_build()
    cores = O.set_threads(os.cpu_count() or 1)
    m = O.load_model(path)
    cu = np.concatenate([[0], np.cumsum(lens)])
    done_tok, n, t0 = 0, 0, time.perf_counter()
    while n < len(lens) and (time.perf_counter() - t0) < budget_s:
        O.encode(m, ids[cu[n]:cu[n + 1]], lens[n:n + 1], O.GGML)
        done_tok += int(lens[n])
        n += 1
    dt = time.perf_counter() - t0
    return {"value": done_tok / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"first {n} sequences ({done_tok} tokens) of the config-2 batch, one encode per sequence "
                      f"as the reference's sequential path does, ggml-faithful mode (C library expf/erff), {dt:.1f}s"}


def c2_config(n_seqs, tokens, world):
    return {"workload": f"c2: NomicBERT-MoE Q8_0 encoder, {n_seqs} seqs len U[32,512] seed 2 per rank",
            "tokens_per_step_per_gpu": tokens, "global_batch": n_seqs * world, "seq_len": "U[32,512]",
            "parallelism": f"dp{world} replicas", "l2": "inputs larger than L2 (~3 GB activations/step)"}


def run_reference(args, rank):
    if rank != 0:
        return 0
    from crispembed_b200 import synth
    path = model_path(0)
    ids, lens = synth.config_ids(2)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.use_timing_build()
    cores = O.set_threads(os.cpu_count() or 1)
    m = O.load_model(path)
    cu = np.concatenate([[0], np.cumsum(lens)])
    per_step = 2  # sequences per step: bounded sample of the config-2 batch
    times, toks = [], []
    for s in range(args.warmup + args.steps):
        a = (s * per_step) % len(lens)
        b = min(a + per_step, len(lens))
        t0 = time.perf_counter()
        for q in range(a, b):
            O.encode(m, ids[cu[q]:cu[q + 1]], lens[q:q + 1], O.GGML)
        dt = time.perf_counter() - t0
        if s >= args.warmup:
            times.append(dt)
            toks.append(int(lens[a:b].sum()))
    value = sum(toks) / sum(times)
    sample = (f"{per_step} sequences per step of the config-2 batch (lens U[32,512] seed 2), encoded one by one "
              f"(the reference's sequential encode_tokens path), oracle ggml-faithful CPU restatement with the C "
              f"library's expf/erff")
    out = {"metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint8 blocks / f32",
           "data": "synthetic", "config": c2_config(len(lens), int(lens.sum()), 1),
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "reference ggml cannot be built here (empty submodule); CPU restatement in oracle/ timed instead"}
    print(json.dumps(out), flush=True)
    return 0


def c4_config(world, tokens):
    return {"workload": "c4: NomicBERT-MoE Q8_0 encoder, 512 seqs x 512 tokens seed 3 per step (whole job), "
                        "sequences sharded over the ranks, MoE experts split over the ranks",
            "tokens_per_step": tokens, "global_batch": 512, "seq_len": 512,
            "parallelism": f"ep{world} (experts {8 // world} per GPU) x dp{world} sequence shards",
            "exchange": "per MoE block: counts, dispatch rows (fp16) and expert outputs (fp16) stored into peer "
                        "memory by the permutation / return kernels over NVLink, bounded flag waits",
            "l2": "inputs larger than L2"}


def bench_ep(args, rank, world, local, path, dist):
    """expert-parallel encoder over the ranks of this job (one per GPU)."""
    import torch

    from crispembed_b200 import binding, synth
    from crispembed_b200.dist import connect_expert_parallel, max_over_ranks, shard_sequences
    ids, lens = synth.config_ids(4)
    total = int(lens.sum())
    s0, cnt, tok0, ntok = shard_sequences(lens, rank, world)
    my_ids, my_lens = np.ascontiguousarray(ids[tok0:tok0 + ntok]), np.ascontiguousarray(lens[s0:s0 + cnt])
    m = binding.CrispEmbed(path)
    h = m.hparams
    n_embd = int(h.n_embd)
    ep = binding.ExpertParallel(rank, world, h.n_experts, h.n_experts_per_tok, n_embd,
                                synth.nomic_moe_spec().expert_ffn, ntok)
    connect_expert_parallel(ep)
    ep.set_timeout_ms(30000)
    m.attach_ep(ep)
    d_ids = torch.from_numpy(my_ids).cuda()
    out = torch.empty((cnt, m.dim), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        m.encode_ids_device(d_ids, my_lens, out)
    torch.cuda.synchronize()
    binding.sync_check()
    if dist:
        dist.barrier()
    n0 = binding.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        clk.wait_first()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            m.encode_ids_device(d_ids, my_lens, out)
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = binding.launch_count() - n0
    binding.sync_check()
    binding.profile_enable(True)  # per-launch events in a second pass of the same steps
    for _ in range(args.steps):
        m.encode_ids_device(d_ids, my_lens, out)
    torch.cuda.synchronize()
    prof = binding.profile_read()
    binding.profile_enable(False)
    t = max_over_ranks(ev0.elapsed_time(ev1) / 1000.0, "cuda")
    brk = {k: v["ms"] / args.steps for k, v in prof.items()}
    per_rank = [brk]
    if dist:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, brk)
        dist.barrier()
    for _ in range(2):
        m.encode_ids(my_ids, my_lens)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        emb = m.encode_ids(my_ids, my_lens)
    te = max_over_ranks(time.perf_counter() - t0, "cuda")
    assert np.allclose(np.linalg.norm(emb, axis=1), 1.0, atol=1e-4)
    if dist:
        dist.barrier()
    m.close()
    ep.close()
    if dist:
        dist.barrier()
    return {"value": total * args.steps / t, "unit": "tokens/s", "per_gpu_tokens_per_s": total * args.steps / t / world,
            "ms_per_step": 1000.0 * t / args.steps, "config": c4_config(world, total),
            "e2e": {"value": total * args.steps / te, "unit": "tokens/s", "h2d_bytes_per_step": int(my_ids.nbytes),
                    "d2h_bytes_per_step": int(cnt * n_embd * 4), "note": "rank 0's bytes; every rank copies its shard"},
            "gpu_launches": int(launches), "clocks": clk.summary(),
            "breakdown_ms_per_step_rank0": brk,
            "breakdown_ms_per_step_min_max_over_ranks": {
                k: [min(b[k] for b in per_rank), max(b[k] for b in per_rank)] for k in brk}}


def gemm_roofline(g, pk, pk_src, kernel, traffic, traffic_source):
    """Tensor roofline of a set of GEMM launches: algorithmic FLOPs per launch over the
    mean CUDA-event duration, against the measured sustained bf16 peak (every line of
    this file uses that peak; the fraction of the burst peak is given beside it)."""
    achieved = g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] > 0 else 0.0
    peak = float(pk.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    burst = float(pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    return {"kernel": kernel, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "peak_source": f"{pk_src} bf16_tflops_sustained",
            "frac_of_burst_peak": achieved / burst, "launches": g["launches"],
            "flops_per_launch": g["flops"] / max(1, g["launches"]), "avg_launch_ms": g["ms"] / max(1, g["launches"]),
            "traffic": traffic, "traffic_source": traffic_source,
            "measured": "kernel time from CUDA events around each GEMM launch on its stream, in a pass of the "
                        "same steps right after the timed region"}


def traffic_from_profile(workload):
    p = os.path.join(ROOT, "profiles", f"gemm_traffic_{workload}.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "c5"], default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ep", action="store_true", help="skip the expert-parallel (config 4) block of the c2 line")
    ap.add_argument("--no-ops", action="store_true", help="skip the MoE-operator (configs 3, 5) blocks of the c2 line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return run_reference(args, rank)

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
    from crispembed_b200 import binding, synth
    from crispembed_b200.dist import max_over_ranks

    path = model_path(local) if args.workload in ("c2", "c4") else None
    if world > 1:
        # NCCL's own log lines (its version banner) go to stderr: stdout carries the one JSON line
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    if args.workload in ("c3", "c5"):
        return bench_moe_op(args, rank, world, local) if rank == 0 else 0
    if args.workload == "c4":
        r = bench_ep(args, rank, world, local, path, dist)
        if rank == 0:
            line = {"metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
                    "scaling": "strong", "vs_baseline": None,
                    "dtype": "fp16 (Q8_0 weights dequantized to fp16, fp32 accumulate)",
                    "data": "synthetic (seeded ids; random-init weights of the nomic-embed-text-v2-moe architecture)",
                    "config": r["config"], "per_gpu_tokens_per_s": r["per_gpu_tokens_per_s"], "e2e": r["e2e"],
                    "gpu_launches": r["gpu_launches"], "clocks": r["clocks"]}
            print(json.dumps(line), flush=True)
        if dist:
            dist.destroy_process_group()
        return 0

    ids, lens = synth.config_ids(2)
    n_seqs, tokens = len(lens), int(lens.sum())
    m = binding.CrispEmbed(path)
    dim = m.dim
    d_ids = torch.from_numpy(ids).cuda()
    out = torch.empty((n_seqs, dim), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        m.encode_ids_device(d_ids, lens, out)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    n0 = binding.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        clk.wait_first()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            m.encode_ids_device(d_ids, lens, out)
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = binding.launch_count() - n0
    binding.sync_check()
    # second pass over the same steps with a CUDA event pair around every launch (on the
    # launching stream): per-kernel-category times for the breakdown and the roofline
    binding.profile_enable(True)
    for _ in range(args.steps):
        m.encode_ids_device(d_ids, lens, out)
    torch.cuda.synchronize()
    prof = binding.profile_read()
    binding.profile_enable(False)
    t = ev0.elapsed_time(ev1) / 1000.0
    t = max_over_ranks(t, "cuda")
    if dist:
        dist.barrier()
    value = world * tokens * args.steps / t

    # end to end through the host-buffer C ABI (ids H2D and embeddings D2H inside)
    for _ in range(2):
        m.encode_ids(ids, lens)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        emb = m.encode_ids(ids, lens)
    te = time.perf_counter() - t0
    te = max_over_ranks(te, "cuda")
    e2e = world * tokens * args.steps / te
    assert np.allclose(np.linalg.norm(emb, axis=1), 1.0, atol=1e-4)
    m.close()

    pk, pk_src = peaks()
    g = {k: prof["gemm"][k] + prof["moe_gemm"][k] for k in ("launches", "ms", "flops", "bytes")}
    tr = traffic_from_profile("c2")
    moe_shapes = [sh for sh in (tr or {}).get("shapes", []) if sh["shape"].startswith("MoE")]
    moe_traffic = (sum(sh["dram_read"] + sh["dram_write"] for sh in moe_shapes) / len(moe_shapes)
                   if moe_shapes else None)
    result = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * t / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 (Q8_0 weights dequantized to fp16, fp32 accumulate)",
        "data": "synthetic (seeded ids; random-init weights of the nomic-embed-text-v2-moe architecture)",
        "config": c2_config(n_seqs, tokens, world),
        "per_gpu_tokens_per_s": value / world,
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": int(ids.nbytes),
                "d2h_bytes_per_step": int(n_seqs * dim * 4)},
        "gpu_launches": int(launches),
        "roofline": gemm_roofline(g, pk, pk_src, "ceb_gemm_pair_kernel (tcgen05 CTA-pair GEMM), every launch of "
                                  "the step: dense linear layers and grouped expert GEMMs",
                                  (tr or {}).get("bytes_per_launch"), (tr or {}).get("source")),
        "roofline_moe_grouped_gemm": gemm_roofline(
            prof["moe_gemm"], pk, pk_src, "ceb_gemm_pair_kernel, the grouped expert GEMMs of the MoE blocks only "
            "(fc1 + GELU and fc2, 8 experts per launch)", moe_traffic,
            "mean of the MoE fc1 and fc2 shapes of the same ncu capture (profiles/gemm_traffic_c2.json)"),
        "breakdown_ms_per_step": {k: v["ms"] / args.steps for k, v in prof.items()},
        "clocks": clk.summary(),
    }
    if not args.no_ep:
        if dist:
            dist.barrier()
        result["expert_parallel"] = bench_ep(args, rank, world, local, path, dist)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(path, ids, lens)
    if world == 1 and not args.no_ops:
        result["moe_operator"] = {w: moe_op_block(args, w, local) for w in ("c3", "c5")}
    if rank == 0:
        print(json.dumps(result), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


OP_WORKLOADS = {
    # isolated MoE FFN operator, Q4_K experts, Zipf(1.2) loads; T sweep {512, 8192, 65536}
    "c3": dict(d=768, n_experts=8, top_k=2, ffn=3072, T=65536, zipf=1.2, sweep=[512, 8192], variants=[]),
    # wide routing, E=32 top-4, Q4_K, T=131072, balanced and Zipf(1.5)
    "c5": dict(d=1024, n_experts=32, top_k=4, ffn=1536, T=131072, zipf=None, sweep=[], variants=[1.5]),
}


def _time_moe_op(args, cfg, T, zipf, local, with_clocks=False):
    import torch

    from crispembed_b200 import binding, synth
    from crispembed_b200.gguf_io import GGML_F32, GGML_Q4_K
    inp = synth.make_moe_op_inputs(T, d=cfg["d"], n_experts=cfg["n_experts"], top_k=cfg["top_k"], ffn=cfg["ffn"],
                                   wtype=GGML_Q4_K, router_wtype=GGML_F32, zipf_s=zipf, seed=0)
    layer = binding.MoELayer(inp.d, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype,
                             inp.fc1_raw, inp.fc2_raw, inp.bias)
    x = torch.from_numpy(inp.x).cuda().to(torch.bfloat16)
    y = torch.empty((T, inp.d), dtype=torch.float32, device="cuda")
    ws = torch.empty(layer.workspace_size(T), dtype=torch.uint8, device="cuda")
    cnt = torch.empty((inp.n_experts,), dtype=torch.int32, device="cuda")
    for _ in range(args.warmup):
        layer.forward(x, y, ws, counts=cnt)
    torch.cuda.synchronize()
    binding.sync_check()
    steps = args.steps if T >= 8192 else max(args.steps, 200)
    n0 = binding.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local) if with_clocks else None
    if clk:
        clk.__enter__()
        clk.wait_first()
    ev0.record()
    for _ in range(steps):
        layer.forward(x, y, ws)
    ev1.record()
    torch.cuda.synchronize()
    if clk:
        clk.__exit__(None, None, None)
    launches = (binding.launch_count() - n0) // steps * args.steps
    binding.profile_enable(True)  # per-launch events in a second pass of the same steps
    for _ in range(steps):
        layer.forward(x, y, ws)
    torch.cuda.synchronize()
    prof = binding.profile_read()
    binding.profile_enable(False)
    t = ev0.elapsed_time(ev1) / 1000.0 / steps
    # end to end: every step's x from pinned host memory and its y back to pinned host memory,
    # inside the timed region; the copies run on their own streams into double-buffered device
    # tensors, so step i's download and step i+1's upload overlap the operator's compute
    # (PCIe is full duplex) as a streaming caller would run it
    hx = x.cpu().pin_memory()
    hy = [torch.empty((T, inp.d), dtype=torch.float32).pin_memory() for _ in range(2)]
    xs, ys = [x, torch.empty_like(x)], [y, torch.empty_like(y)]
    comp, s_in, s_out = torch.cuda.current_stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in, ev_done, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(steps):
        b = i & 1
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_done[b])  # step i-2's compute has read xs[b]
            xs[b].copy_(hx, non_blocking=True)
            ev_in[b].record(s_in)
        comp.wait_event(ev_in[b])
        if i >= 2:
            comp.wait_event(ev_out[b])  # step i-2's download has read ys[b]
        layer.forward(xs[b], ys[b], ws)
        ev_done[b].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[b])
            hy[b].copy_(ys[b], non_blocking=True)
            ev_out[b].record(s_out)
    torch.cuda.synchronize()
    te = (time.perf_counter() - t0) / steps
    loads = cnt.cpu().numpy()
    g = prof["moe_gemm"]
    r = {"T": T, "zipf": zipf, "ms": 1000 * t, "tokens_per_s": T / t, "e2e_tokens_per_s": T / te,
         "h2d_bytes": int(hx.numel() * hx.element_size()), "d2h_bytes": int(hy[0].numel() * 4),
         "gemm_tflops": g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] > 0 else 0.0,
         "gemm_ms": g["ms"] / steps, "gemm": g, "launches": int(launches),
         "max_over_mean_expert_load": float(loads.max() / loads.mean()),
         "breakdown_ms": {k: v["ms"] / steps for k, v in prof.items()}, "clocks": clk.summary() if clk else None}
    layer.close()
    return r, inp


OP_E2E_COPIES = ("pinned host x and y; upload and download on their own streams into double-buffered device "
                 "tensors, overlapping the neighbouring steps' compute")


def op_cases(cfg):
    """(T, zipf) of every measured case of an operator workload, the main case first."""
    return [(cfg["T"], cfg["zipf"])] + [(T, cfg["zipf"]) for T in cfg["sweep"]] + [(cfg["T"], z) for z in cfg["variants"]]


def op_metric(cfg):
    skew = f"Zipf {cfg['zipf']}" if cfg["zipf"] else "balanced"
    return (f"MoE FFN operator tokens/s (Q4_K, d={cfg['d']} E={cfg['n_experts']} top-{cfg['top_k']} "
            f"F={cfg['ffn']}, T={cfg['T']}, {skew})"), skew


def moe_op_block(args, workload, local, cpu_budget_s=5.0):
    """One operator workload (BASELINE config 3 or 5) as a block of the default line:
    its main case with e2e, the tensor roofline of its grouped GEMMs, clocks, the
    other cases of the config and the CPU restatement on a bounded sample."""
    cfg = OP_WORKLOADS[workload]
    pk, pk_src = peaks()
    cases = []
    inp = None
    for i, (T, z) in enumerate(op_cases(cfg)):
        r, got = _time_moe_op(args, cfg, T, z, local, with_clocks=(i == 0))
        if i == 0:
            main_r, inp = r, got
        cases.append({k: r[k] for k in ("T", "zipf", "ms", "tokens_per_s", "e2e_tokens_per_s", "gemm_tflops",
                                        "max_over_mean_expert_load")})
    metric, skew = op_metric(cfg)
    tr = traffic_from_profile(workload)
    block = {"metric": metric, "value": main_r["tokens_per_s"], "unit": "tokens/s", "ms_per_step": main_r["ms"],
             "steps": args.steps,
             "config": {"workload": f"{workload}: MoE op, x bf16 N(0,1), router F32, experts Q4_K, {skew}",
                        "tokens": cfg["T"], "l2": "inputs larger than L2"},
             "e2e": {"value": main_r["e2e_tokens_per_s"], "unit": "tokens/s",
                     "h2d_bytes_per_step": main_r["h2d_bytes"], "d2h_bytes_per_step": main_r["d2h_bytes"],
                     "copies": OP_E2E_COPIES},
             "gpu_launches": main_r["launches"],
             "roofline": gemm_roofline(main_r["gemm"], pk, pk_src, "ceb_gemm_pair_kernel, grouped expert GEMMs "
                                       "(fc1 + GELU, fc2) on Q4_K weights expanded to fp16 at load",
                                       (tr or {}).get("bytes_per_launch"), (tr or {}).get("source")),
             "breakdown_ms_per_step": main_r["breakdown_ms"], "clocks": main_r["clocks"], "cases": cases}
    if not args.no_cpu_baseline:
        block["cpu_baseline"] = op_cpu_baseline(inp, budget_s=cpu_budget_s)
    return block


def op_cpu_baseline(inp, budget_s=10.0, n=256):
    """Oracle MoE op (ggml-faithful CPU restatement) on the first n tokens, repeated for ~budget_s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.use_timing_build()
    cores = O.set_threads(os.cpu_count() or 1)
    x = inp.x[:n]
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s or done == 0:
        O.moe_ffn(x, inp.n_experts, inp.top_k, inp.ffn, inp.router_wtype, inp.router_raw, inp.wtype, inp.fc1_raw,
                  inp.fc2_raw, inp.bias, O.GGML)
        done += len(x)
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"the first {n} tokens of the workload, MoE op repeated for {dt:.1f}s, ggml-faithful mode "
                      f"(C library expf/erff)"}


def bench_moe_op(args, rank, world, local):
    """BASELINE configs 3 and 5: the isolated MoE FFN operator (ceb_moe_ffn), Q4_K experts."""
    cfg = OP_WORKLOADS[args.workload]
    main_r, inp = _time_moe_op(args, cfg, cfg["T"], cfg["zipf"], local, with_clocks=True)
    pk, pk_src = peaks()
    flops_tok = 2.0 * 2 * cfg["top_k"] * cfg["d"] * cfg["ffn"]
    metric, skew = op_metric(cfg)
    tr = traffic_from_profile(args.workload)
    rl = gemm_roofline(main_r["gemm"], pk, pk_src, "ceb_gemm_pair_kernel, grouped expert GEMMs (fc1 + GELU, fc2)",
                       (tr or {}).get("bytes_per_launch"), (tr or {}).get("source"))
    rl["op_tflops"] = main_r["tokens_per_s"] * flops_tok / 1e12
    result = {"metric": metric,
              "value": main_r["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
              "warmup": args.warmup, "ms_per_step": main_r["ms"], "higher_is_better": True, "scaling": "weak",
              "vs_baseline": None, "dtype": "fp16 (Q4_K dequant, fp32 accumulate)", "data": "synthetic",
              "config": {"workload": f"{args.workload}: MoE op, x bf16 N(0,1), router F32, experts Q4_K, {skew}",
                         "tokens": cfg["T"], "l2": "inputs larger than L2" if cfg["T"] >= 65536 else "fits L2"},
              "e2e": {"value": main_r["e2e_tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": main_r["h2d_bytes"],
                      "d2h_bytes_per_step": main_r["d2h_bytes"], "copies": OP_E2E_COPIES},
              "gpu_launches": main_r["launches"],
              "roofline": rl,
              "max_over_mean_expert_load": main_r["max_over_mean_expert_load"],
              "breakdown_ms_per_step": main_r["breakdown_ms"], "clocks": main_r["clocks"]}
    others = []
    for T in cfg["sweep"]:
        r, _ = _time_moe_op(args, cfg, T, cfg["zipf"], local)
        others.append({k: r[k] for k in ("T", "zipf", "ms", "tokens_per_s", "e2e_tokens_per_s", "gemm_tflops",
                                         "max_over_mean_expert_load")})
    for z in cfg["variants"]:
        r, _ = _time_moe_op(args, cfg, cfg["T"], z, local)
        others.append({k: r[k] for k in ("T", "zipf", "ms", "tokens_per_s", "e2e_tokens_per_s", "gemm_tflops",
                                         "max_over_mean_expert_load")})
    if others:
        result["other_cases"] = others
    if not args.no_cpu_baseline:
        result["cpu_baseline"] = op_cpu_baseline(inp)
    print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
