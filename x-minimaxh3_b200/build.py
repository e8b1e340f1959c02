"""Build libh3b.so (the sm_100a kernels + C ABI) in place with nvcc.

    python x-minimaxh3_b200/build.py [--verbose-ptxas]

Objects go to x-minimaxh3_b200/_build/, the library to x-minimaxh3_b200/h3b/libh3b.so,
where the Python package loads it from.  Cross-compiles without a GPU.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "h3b", "libh3b.so")
SOURCES = ["h3b_all.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # IEEE single-precision everywhere; fused multiply-adds only where written as fmaf(),
    # so the quantizers and the mask reproduce the CPU oracle bit for bit.
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-I" + os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _stale(obj: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h", ".cu"))]
    headers.append(os.path.join(ROOT, "include", "h3b.h"))
    objs = []
    jobs = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [path] + headers):
            cmd = [nvcc(), *NVCC_FLAGS, "-c", path, "-o", obj]
            if verbose_ptxas:
                cmd += ["-Xptxas", "-v"]
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    failed = False
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for src, r in ex.map(run, jobs):
            if r.returncode != 0 or verbose_ptxas:
                sys.stderr.write(f"--- {src}\n{r.stdout}{r.stderr}")
            if r.returncode != 0:
                failed = True
    if failed:
        raise RuntimeError("nvcc failed")
    if force or jobs or not os.path.exists(OUT) or _stale(OUT, objs):
        cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", OUT, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(args.verbose_ptxas, args.force))
