"""Build libekv.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python embodied.cpp_b200/build.py [--force] [--verbose]

No fast-math: the Q8_0 append must use IEEE division and rounding to stay bit-exact with the
gguf-py / ggml rule.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libekv.so")
BUILD_DIR = os.path.join(HERE, "_build")
SOURCES = ["ekv_capi.cpp", "ekv_sched.cpp", "ekv_cache_kernels.cu", "ekv_attn_simt.cu", "ekv_attn_tc.cu", "ekv_attn_pair.cu", "ekv_attn_pair128.cu", "ekv_attn_heads.cu", "ekv_noalloc.cu", "ekv_ggml_fa.cu", "ekv_ggml_tc.cu", "ekv_flow.cu", "ekv_project.cu"]
HEADERS = ["ekv_internal.h", "ekv_layout.cuh", "ekv_device.cuh", "ekv_sm100.cuh", "ekv_attn_common.cuh", "ekv_ggml.h"]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I" + os.path.join(ROOT, "include")]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "ekv.h")]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD_DIR, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [NVCC, *ARCH, *COMMON, "-c", s, "-o", o]
            if src.endswith(".cu") and ptxas_info:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError(f"nvcc failed on {src}")
            if ptxas_info or verbose:
                sys.stderr.write(r.stderr)
    if force or _stale(OUT, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", OUT, *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc link failed")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_info))
