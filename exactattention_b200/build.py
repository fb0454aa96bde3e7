"""Builds libexactattn_cuda.so in-tree for sm_100a: python -m exactattention_b200.build

Each source compiles to its own object (in parallel, under _build/), then one link makes the
shared library. Objects are rebuilt when their source or any header changed."""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "libexactattn_cuda.so")
SOURCES = ["ea_simt.cu", "ea_tc.cu", "ea_decode.cu", "ea_api.cu", "ea_synth.cu", "ea_noalloc.cu", "ea_cache.cu",
           "ea_selftest.cu", "ea_nccl.cu"]
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC"]
HEADER = os.path.join(HERE, "..", "include", "exactattn_cuda.h")


def _headers_mtime() -> float:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))] + [HEADER]
    return max(os.path.getmtime(p) for p in hs if os.path.exists(p))


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return _headers_mtime() > t or any(os.path.getmtime(os.path.join(CSRC, f)) > t for f in SOURCES)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        build_synth_host()
        return OUT
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    os.makedirs(OBJ, exist_ok=True)
    hdr = _headers_mtime()

    def compile_one(src: str) -> str:
        obj = os.path.join(OBJ, src.replace(".cu", ".o"))
        s = os.path.join(CSRC, src)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(s), hdr):
            cmd = [nvcc, *FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-c", "-o", obj + ".tmp", src]
            subprocess.run(cmd, cwd=CSRC, check=True)
            os.replace(obj + ".tmp", obj)
        return obj

    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = OUT + ".tmp"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
                    "-o", tmp, *objs], check=True)
    os.replace(tmp, OUT)
    build_synth_host(force)
    return OUT


SYNTH_HOST = os.path.join(HERE, "libea_synth_host.so")


def build_synth_host(force: bool = False) -> str:
    """The host input generator (benchmarks and tests only), gcc with OpenMP."""
    src = os.path.join(CSRC, "ea_synth_host.c")
    if force or not os.path.exists(SYNTH_HOST) or os.path.getmtime(SYNTH_HOST) < os.path.getmtime(src):
        subprocess.run(["gcc", "-O3", "-fopenmp", "-fPIC", "-shared", "-o", SYNTH_HOST + ".tmp", src], check=True)
        os.replace(SYNTH_HOST + ".tmp", SYNTH_HOST)
    return SYNTH_HOST


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
