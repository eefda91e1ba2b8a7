"""Build libactrain.so in-tree for sm_100a (nvcc + g++, no torch extension machinery).

    python audiocraft.cpp_b200/build.py [--jobs N]

Objects go to audiocraft.cpp_b200/_build/, the library to audiocraft.cpp_b200/libactrain.so.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libactrain.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          "-I" + CSRC, "-I" + os.path.join(ROOT, "include")]


def sources():
    out = []
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cpp")):
            out.append(os.path.join(CSRC, f))
    return out


def deps_mtime(src):
    newest = os.path.getmtime(src)
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh")):
                newest = max(newest, os.path.getmtime(os.path.join(d, f)))
    return newest


def compile_one(src, verbose=False):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= deps_mtime(src):
        return obj, None
    cmd = [NVCC] + ARCH + COMMON + ["-c", src, "-o", obj]
    if src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"] if verbose else []
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, r.stderr + r.stdout
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj, None


def build(jobs: int = 8, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(jobs) as ex:
        results = list(ex.map(lambda s: compile_one(s, verbose), srcs))
    errors = [e for _, e in results if e]
    if errors:
        raise RuntimeError("compilation failed:\n" + "\n".join(errors))
    objs = [o for o, _ in results]
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", LIB] + objs + ["-lnccl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr + r.stdout)
    build_trainers()
    return LIB


TRAINER = os.path.join(HERE, "trainer")
BIN = os.path.join(HERE, "bin")
CXX = os.environ.get("CXX", "g++")


def build_trainers() -> list:
    """The mf-train / mg-train front ends: host C++ over libactrain.so (found next to bin/)."""
    os.makedirs(BIN, exist_ok=True)
    common = [os.path.join(TRAINER, f) for f in ("gguf_file.cpp", "train_host.cpp")]
    headers = [os.path.join(TRAINER, f) for f in os.listdir(TRAINER) if f.endswith(".h")]
    headers.append(os.path.join(ROOT, "include", "actrain.h"))
    out = []
    for main, exe in (("mf_train.cpp", "mf-train"), ("mg_train.cpp", "mg-train")):
        src = os.path.join(TRAINER, main)
        if not os.path.exists(src):
            continue
        dst = os.path.join(BIN, exe)
        inputs = [src, LIB] + common + headers
        if not os.path.exists(dst) or os.path.getmtime(dst) < max(os.path.getmtime(f) for f in inputs):
            cmd = [CXX, "-std=c++17", "-O2", "-Wall", "-I" + TRAINER, "-I" + os.path.join(ROOT, "include"), src] + \
                  common + ["-o", dst, "-L" + HERE, "-lactrain", "-Wl,-rpath,$ORIGIN/.."]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(exe + " build failed:\n" + r.stderr + r.stdout)
        out.append(dst)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.jobs, a.verbose))
