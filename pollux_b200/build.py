"""Build recipe of libh24.so (the CUDA library behind pollux_b200).

    python -m pollux_b200.build          # compiles into pollux_b200/_lib/

Every CUDA source is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) with line info, and linked with
the static CUDA runtime so that the library does not depend on which
libcudart the host process (e.g. torch) has loaded.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
BUILD_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libh24.so")
SOURCES = ["h24_capi.cu", "h24_pack.cu", "h24_dequant.cu", "h24_lut.cu", "h24_int8.cu", "h24_project.cu", "h24_rowrms.cu", "h24_search.cu", "h24_codebook.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                     "--expt-relaxed-constexpr", "-Werror", "all-warnings"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile (incrementally) and return the path of libh24.so."""
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(BUILD_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(os.path.dirname(HERE), "include", "h24.h"))
    objs, jobs = [], []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD_DIR, src + ".o")
        objs.append(obj)
        if _stale(obj, [path] + headers) or ptxas_info:
            cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + \
                  ["-c", path, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stdout + r.stderr

    with cf.ThreadPoolExecutor(max_workers=len(jobs) or 1) as ex:
        for out in ex.map(run, jobs):
            if verbose and out.strip():
                print(out)
    if jobs or _stale(LIB, objs):
        run([nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs)
    return LIB


if __name__ == "__main__":
    path = build(verbose=True, ptxas_info="-v" in sys.argv)
    print(path)
