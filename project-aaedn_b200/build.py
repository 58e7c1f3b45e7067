#!/usr/bin/env python3
"""Builds libaaedn_b200.so in-tree (project-aaedn_b200/aaedn_b200/).

CUDA sources are compiled for sm_100a only; the host C++ (quant tools,
error state, the reference-API mirror) with g++ without fast-math so the host
quantizer and tables stay bit-exact. Objects go to project-aaedn_b200/build/.

    python project-aaedn_b200/build.py [--force] [--jobs N]
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
HOST = os.path.join(HERE, "host")
BUILD = os.path.join(HERE, "build")
OUT = os.path.join(HERE, "aaedn_b200", "libaaedn_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INCS = ["-I" + os.path.join(ROOT, "include"), "-I" + HOST, "-I" + os.path.join(HOST, "include")]

CU_SRCS = ["api.cu", "model.cu", "ffn.cu", "sample.cu", "gemm_tc.cu"]
CPP_SRCS = ["errors.cpp", "quant_tools.cpp", "abn_file.cpp", "aaedn_api.cpp", "tokenizer.cpp"]


def _deps(src):
    if src.endswith(".cu"):
        return [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(ROOT, "include", "aaedn_b200.h"),
                                                                      os.path.join(HOST, "host_common.hpp")]
    inc = os.path.join(HOST, "include", "aaedn")
    hdrs = [os.path.join(inc, f) for f in os.listdir(inc)] if os.path.isdir(inc) else []
    return [os.path.join(ROOT, "include", "aaedn_b200.h"), os.path.join(HOST, "host_common.hpp")] + hdrs


def _stale(obj, src):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in [src] + _deps(src) if os.path.exists(d))


def _compile(job):
    src, obj, cmd = job
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force=False, jobs=4, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    todo, objs = [], []
    for f in CU_SRCS:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
               "--expt-relaxed-constexpr", *INCS, "-c", src, "-o", obj]
        if force or _stale(obj, src):
            todo.append((src, obj, cmd))
    for f in CPP_SRCS:
        src = os.path.join(HOST, f)
        if not os.path.exists(src):
            continue
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-fno-fast-math", "-ffp-contract=off", *INCS,
               "-I/usr/local/cuda/include", "-c", src, "-o", obj]
        if force or _stale(obj, src):
            todo.append((src, obj, cmd))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for obj, err in ex.map(_compile, todo):
                if verbose and err:
                    print(err, file=sys.stderr)
    if todo or not os.path.exists(OUT):
        cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objs, "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=4)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))
