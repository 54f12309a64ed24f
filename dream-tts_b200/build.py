"""Builds the sm_100a kernels and the C ABI into ttsnn/libtts_cuda.so (in-tree).

    python dream-tts_b200/build.py [--force]

nvcc cross-compiles without a GPU. The library links the CUDA runtime statically and reaches
the driver's tensor-map encoder through cudaGetDriverEntryPoint, so it needs no libcuda at
link time.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "ttsnn", "libtts_cuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["runtime.cu", "gemm_decode.cu", "attn_decode.cu", "ops_small.cu",
           "predictor.cu", "attn_short.cu", "topk_sample.cu", "safetensors.cpp",
           "codec_front.cu", "pf_gemm.cu", "pf_attn.cu",
           "conv_nlc.cu", "kv_pool.cu"]
HEADERS = ["tts_common.cuh", "tts_internal.h", "qkrope_row.cuh", "gemm_epilogue.cuh", "pick_rule.cuh",
           "l2_prefetch.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs() -> list[str]:
    return ([os.path.join(CSRC, s) for s in SOURCES + HEADERS]
            + [os.path.join(INCLUDE, "tts_cuda.h")])


# The tracing variant: the same sources with per-CTA timeline records (TTS_TIMELINE; the
# records live in one device buffer, so the objects are relocatable and device-linked).
OUT_TIMELINE = os.path.join(HERE, "ttsnn", "libtts_cuda_tl.so")


def up_to_date_at(out: str) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(p) <= t for p in _inputs())


def up_to_date() -> bool:
    return up_to_date_at(OUT)


def build(force: bool = False, verbose: bool = False, timeline: bool = False) -> str:
    out = OUT_TIMELINE if timeline else OUT
    if not force and up_to_date_at(out):
        return out
    objdir = os.path.join(HERE, "_build_tl" if timeline else "_build")
    os.makedirs(objdir, exist_ok=True)
    extra = ["-rdc=true", "-DTTS_TIMELINE"] if timeline else []
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "tts_cuda.h")]
    newest_header = max(os.path.getmtime(h) for h in headers)
    jobs = []
    objs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(objdir, os.path.splitext(s)[0] + ".o")
        objs.append(obj)
        # an object is reused when it is newer than its source and every header
        if (not force and os.path.exists(obj)
                and os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_header)):
            continue
        cmd = [nvcc(), *NVCC_FLAGS, *extra, "-I", INCLUDE, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        jobs.append(cmd)
    # the sources compile independently: run them side by side
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        for r in list(ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise subprocess.CalledProcessError(r.returncode, r.args)
            elif verbose and (r.stdout or r.stderr):
                sys.stderr.write(r.stdout + r.stderr)
    tmp = out + ".tmp"
    # --no-undefined: a symbol missing from the objects fails the build, not the first load
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *extra[:1],
           "-Xlinker", "--no-undefined", "-o", tmp, *objs]
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--timeline", action="store_true",
                    help="build the tracing variant ttsnn/libtts_cuda_tl.so")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, timeline=args.timeline))
    sys.exit(0)
