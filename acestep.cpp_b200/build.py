"""Build libacefa.so (all CUDA sources, sm_100a only) in-tree.

    python acestep.cpp_b200/build.py [--force] [--verbose-ptxas]

The shared library is written next to this file so that it travels with the
source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libacefa.so")
BUILD = os.path.join(HERE, "_build")

SOURCES = ["fa_api.cu", "fa_decode.cu", "fa_dense.cu", "fa_noalloc.cu", "fa_peer.cu", "fa_prologue.cu",
           "cfg_combine.cu"]
HEADERS = ["fa_internal.h", "ptx.cuh", "q8.cuh", "rope_norm.cuh"]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-DNDEBUG"]


def _sources():
    return [s for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]


def _newest_input() -> float:
    paths = [os.path.join(CSRC, s) for s in _sources() + HEADERS if os.path.exists(os.path.join(CSRC, s))]
    paths.append(os.path.join(ROOT, "include", "acefa.h"))
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths)


def build(force: bool = False, ptxas_verbose: bool = False, jobs: int = 4, out: str | None = None,
          defines: list[str] | None = None, build_dir: str | None = None) -> str:
    """Compile and link.  `out`, `defines` (-D macros) and `build_dir` build a
    variant library elsewhere; the defaults build the in-tree libacefa.so."""
    target = out or OUT
    bdir = build_dir or BUILD
    if not force and os.path.exists(target) and os.path.getmtime(target) >= _newest_input():
        return target
    os.makedirs(bdir, exist_ok=True)
    objs, procs = [], []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    extra += [f"-D{d}" for d in (defines or [])]
    for src in _sources():
        obj = os.path.join(bdir, src.replace(".cu", ".o"))
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-I", os.path.join(ROOT, "include"), "-c",
               os.path.join(CSRC, src), "-o", obj]
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = False
    for src, p in procs:
        out, _ = p.communicate()
        if out.strip():
            sys.stderr.write(f"--- {src}\n{out}")
        if p.returncode != 0:
            failed = True
    if failed:
        raise RuntimeError("nvcc failed")
    tmp = target + ".tmp"
    subprocess.check_call([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"])
    os.replace(tmp, target)
    return target


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ptxas_verbose=a.verbose_ptxas))
