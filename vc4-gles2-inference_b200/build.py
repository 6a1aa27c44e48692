"""Build the engine's shared library in-tree for sm_100a.

    python vc4-gles2-inference_b200/build.py [--force]

Compiles csrc/*.cu and csrc/*.cpp with nvcc (-gencode arch=compute_100a,
code=sm_100a, --fmad=false so no float expression is contracted) into
vc4b200/_lib/libvc4b200.so.  Objects go to _build/ next to this file.
"""
from __future__ import annotations

import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "vc4b200", "_lib", "libvc4b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "--fmad=false", "-I" + INCLUDE, "-I" + CSRC,
         "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden", "-diag-suppress", "177"]
SOURCES = ["kernels.cu", "ops_q8.cu", "ops_q4.cu", "ops_t3.cu", "engine.cu", "noalloc.cu", "ops.cu", "mmcf.cpp"]
HEADERS = ["vc4b200_internal.h", "kernels.cuh", "batch.cuh", "ops_wt.inc"]


def _newer(target: str, deps: list) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "vc4b200.h")]
    objs, cmds = [], []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        objs.append(obj)
        if force or _newer(obj, [path] + hdrs):
            cmd = [NVCC] + ARCH + FLAGS + ["-c", path, "-o", obj]
            if src.endswith(".cpp"):
                cmd = [NVCC] + ARCH + FLAGS + ["-x", "c++", "-c", path, "-o", obj]
            cmds.append(cmd)
    # the translation units are independent: compile them side by side
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        for cmd in cmds:
            if verbose:
                print(" ".join(cmd), flush=True)
        for f in [ex.submit(subprocess.run, cmd, check=True) for cmd in cmds]:
            f.result()
    if force or _newer(OUT, objs):
        # link next to the target and rename, so a reader never sees a partial file
        tmp = OUT + ".%d.tmp" % os.getpid()
        cmd = [NVCC] + ARCH + ["-shared", "-o", tmp] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
