"""Build libcrispembed.so (sm_100a) in-tree with nvcc.

    python -m crispembed_b200.build [--force] [--verbose]

Objects go to crispembed_b200/_build/, the shared library to
crispembed_b200/libcrispembed.so.  The CUDA runtime is linked statically, so the
library needs only the NVIDIA driver at run time.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libcrispembed.so")

SOURCES = ["gemm_tc.cu", "attn_tc.cu", "attn_fa.cu", "moe.cu", "moe_static.cu", "ep.cu", "encoder_kernels.cu", "ref_arith.cu", "runtime.cpp", "gguf_quants.cpp", "gguf.cpp", "tokenizer.cpp", "model.cpp", "api.cpp"]
HEADERS = ["common.cuh", "rowwise.cuh", "ceb_internal.h", "ceb_moe_internal.h", "ceb_ep_internal.h", "ceb_encoder_internal.h", "gguf.h", "tokenizer.h", "spm_norm_table.inc",
           "ceb_portable_math.h"]
PUBLIC_HEADERS = [os.path.join(ROOT, "include", h) for h in ("crispembed.h", "ceb_ops.h")]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _flags(src: str):
    common = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", CSRC,
              "-I", os.path.join(ROOT, "include"), "-DCRISPEMBED_BUILD=1"]
    if src.endswith(".cu"):
        # the reference-arithmetic kernels fuse only the multiply-adds written as fmaf
        exact = ["-fmad=false"] if src == "ref_arith.cu" else []
        return ARCH + ["-lineinfo", "-Xptxas", "-warn-spills"] + exact + common
    return ["-x", "cu"] + ARCH + common if src == "api.cpp" else common


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + PUBLIC_HEADERS
    jobs = []
    objs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + hdrs):
            cmd = [cc] + _flags(s) + ["-c", src, "-o", obj]
            jobs.append((s, cmd))

    def run(job):
        name, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return name, r

    failed = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for name, r in ex.map(run, jobs):
                out = (r.stdout + r.stderr).strip()
                if r.returncode != 0:
                    failed.append(name)
                    print(f"[build] {name} FAILED\n{out}", file=sys.stderr)
                elif out and verbose:
                    print(f"[build] {name}\n{out}")
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    if force or jobs or _newer(LIB, objs):
        cmd = [cc] + ARCH + ["-shared", "-o", LIB] + objs + ["-lpthread", "-ldl"]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
