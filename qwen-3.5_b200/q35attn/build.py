"""In-tree build of libq35attn.so (sm_100a) with nvcc.

The shared library lands next to this file so that it travels with the
repository snapshot; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)                      # qwen-3.5_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
HOST = os.path.join(ROOT, "host")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(PKG, "libq35attn.so")
BUILD_DIR = os.path.join(ROOT, "_build")

GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def sources():
    cu = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    cpp = sorted(os.path.join(HOST, f) for f in os.listdir(HOST) if f.endswith(".cpp")) if os.path.isdir(HOST) else []
    return cu, cpp


def _deps():
    cu, cpp = sources()
    hdr = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    if os.path.isdir(HOST):
        hdr += [os.path.join(HOST, f) for f in os.listdir(HOST) if f.endswith((".hpp", ".h"))]
    hdr += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return cu + cpp + hdr


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def is_stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(f) > t for f in _deps())


def build(force: bool = False, verbose: bool = False, jobs: int = 8) -> str:
    if not force and not is_stale():
        return LIB
    os.makedirs(BUILD_DIR, exist_ok=True)
    cu, cpp = sources()
    objs, procs = [], []
    env = dict(os.environ)
    env.pop("CC", None)
    env.pop("CXX", None)
    for src in cu + cpp:
        obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
        cmd = [nvcc(), *GENCODE, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-I", HOST, "-ccbin", "g++",
               "-x", "cu" if src.endswith(".cu") else "c++", "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, env=env)))
        objs.append(obj)
        while sum(p.poll() is None for _, p in procs) >= jobs:
            procs[[p.poll() is None for _, p in procs].index(True)][1].wait()
    errs = []
    for src, p in procs:
        out = p.communicate()[0].decode()
        if p.returncode != 0:
            errs.append(f"--- {src}\n{out}")
        elif verbose and out.strip():
            print(out, file=sys.stderr)
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *GENCODE, "-shared", "-ccbin", "g++", "-o", tmp, *objs]
    subprocess.run(cmd, check=True, env=env)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
