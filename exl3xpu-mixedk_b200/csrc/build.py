#!/usr/bin/env python3
"""Build libexl3b200.so for sm_100a (B200) from the .cu sources in this
directory.  nvcc cross-compiles; no GPU is needed.

    python exl3xpu-mixedk_b200/csrc/build.py [--verbose-ptxas] [-j N]

Outputs (in-tree, git-ignored):
  exl3xpu-mixedk_b200/exl3b/libexl3b200.so   the C-ABI library
  exl3xpu-mixedk_b200/exl3b/exl3b_vit        the serve / file-mode worker
                                             (vit_serve.cpp, linked to the library)
Objects are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
OUT = os.path.join(PKG, "exl3b", "libexl3b200.so")
WORKER = os.path.join(PKG, "exl3b", "exl3b_vit")
BUILD = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
         "-I", HERE, "-I", os.path.join(REPO, "include"),
         "--expt-relaxed-constexpr"]


def _deps_mtime() -> float:
    files = glob.glob(os.path.join(HERE, "*.cuh")) + \
        glob.glob(os.path.join(HERE, "*.h")) + \
        glob.glob(os.path.join(REPO, "include", "*.h"))
    return max((os.path.getmtime(f) for f in files), default=0.0)


def _compile(src: str, verbose_ptxas: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(
            os.path.getmtime(src), _deps_mtime()) and not verbose_ptxas:
        return obj, ""
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stdout + r.stderr


def build(verbose_ptxas: bool = False, jobs: int = 8) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        res = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    objs = [o for o, _ in res]
    logs = "".join(l for _, l in res)
    if verbose_ptxas and logs:
        print(logs)
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(OUT) or os.path.getmtime(OUT) < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    src = os.path.join(HERE, "vit_serve.cpp")
    if not os.path.exists(WORKER) or os.path.getmtime(WORKER) < max(
            os.path.getmtime(src), os.path.getmtime(OUT), _deps_mtime()):
        cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-I",
               os.path.join(REPO, "include"), src, "-o", WORKER,
               "-L", os.path.dirname(OUT), "-l:libexl3b200.so", "-Wl,-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"worker build failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    a = ap.parse_args()
    print(build(a.verbose_ptxas, a.j))
    sys.exit(0)
