"""Builds libcandle_moe_b200.so in this directory from csrc/*.cu with nvcc for sm_100a.

Each translation unit compiles to _build/<name>.o (rebuilt when it or any header is newer), then
nvcc links them into one shared library with the CUDA runtime linked statically.  router.cu is
compiled with --use_fast_math, as the reference builds its router (build.rs:59), so that the
router's arithmetic lowers to the same operations.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libcandle_moe_b200.so")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                 "-I", os.path.join(ROOT, "include"), "-I", CSRC]
EXTRA = {"router.cu": ["--use_fast_math"], "router_proj.cu": ["--use_fast_math"]}
SOURCES = ["router.cu", "router_proj.cu", "route_prep.cu", "moe_simt.cu", "moe_sm100.cu", "moe_sm100_pair.cu",
           "moe_decode.cu", "moe_tf32.cu", "ep_kernels.cu", "peer.cu", "capi.cu"]


def _newest_header() -> float:
    hdrs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hdrs), default=0.0)


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdr_t = _newest_header()
    objs, changed = [], False
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_t):
            cmd = [NVCC] + COMMON + EXTRA.get(src, []) + ["-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
            changed = True
    if changed or not os.path.exists(LIB):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + \
            ["-Xlinker", "--exclude-libs,ALL", "-Xlinker", "-Bsymbolic"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
