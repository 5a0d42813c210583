"""Builds libzerollm_b200.so in-tree: every CUDA source of zerollm_b200/csrc is
compiled for sm_100a (nvcc -gencode arch=compute_100a,code=sm_100a) and
linked with NCCL.  Usage: python -m zerollm_b200.build [-j N]"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libzerollm_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-ccbin", "g++",
         "-I", os.path.join(ROOT, "include"), "-I", CSRC, "--expt-relaxed-constexpr"]
SOURCES = ["kernels.cu", "gemm.cu", "attention.cu", "attention_tc.cu", "model.cu", "dist.cu", "loader.cu"]


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OUT_DIR, os.path.splitext(src)[0] + ".o")
    srcp = os.path.join(CSRC, src)
    deps = [srcp, os.path.join(CSRC, "common.cuh"), os.path.join(ROOT, "include", "zerollm_b200.h")]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", srcp, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    return obj


def build(jobs: int = 4, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lnccl", "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_api_test()
    return LIB


API_TEST_SRC = os.path.join(ROOT, "tests", "cpp", "api_test.cpp")
API_TEST_BIN = os.path.join(OUT_DIR, "api_test")


def build_api_test() -> str:
    """Compiles tests/cpp/api_test.cpp against the C++ drop-in headers and the library."""
    deps = [API_TEST_SRC, LIB] + [os.path.join(CSRC, "api", f) for f in os.listdir(os.path.join(CSRC, "api"))]
    if os.path.exists(API_TEST_BIN) and os.path.getmtime(API_TEST_BIN) >= max(os.path.getmtime(d) for d in deps):
        return API_TEST_BIN
    cmd = [NVCC, "-O2", "-std=c++17", "-ccbin", "g++", "-x", "cu", *ARCH, "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CSRC, "api"), API_TEST_SRC, "-o", API_TEST_BIN, "-L", HERE, "-lzerollm_b200",
           f"-Xlinker=-rpath,{HERE}", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"api_test build failed:\n{r.stdout}\n{r.stderr}")
    return API_TEST_BIN


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=4)
    ap.add_argument("-v", action="store_true", help="print ptxas register/spill info")
    a = ap.parse_args()
    print(build(a.j, a.v))
