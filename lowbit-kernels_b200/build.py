"""Build the sm_100a kernel library in-tree: csrc/*.cu -> lowbit/liblowbit_b200.so.

    python lowbit-kernels_b200/build.py [--force] [--verbose]

nvcc cross-compiles without a GPU. Objects go to lowbit-kernels_b200/_build/ (git-ignored); the shared
library lands next to the Python package that loads it, so it travels with the source tree.
"""
import argparse
import concurrent.futures
import os
import pathlib
import shutil
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
BUILD = ROOT / "_build"
OUT = ROOT / "lowbit" / "liblowbit_b200.so"
INCLUDE = ROOT.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", str(INCLUDE)]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build lowbit_b200")
    return exe


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force=False, verbose=False, ptxas_verbose=False):
    BUILD.mkdir(exist_ok=True)
    hdrs = headers()
    jobs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        if force or stale(obj, [src] + hdrs):
            cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append((src, cmd))
    objs = [BUILD / (s.stem + ".o") for s in sources()]

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    if jobs:
        with concurrent.futures.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for src, r in ex.map(run, jobs):
                if r.returncode != 0:
                    sys.stderr.write(r.stdout + r.stderr)
                    raise RuntimeError(f"nvcc failed on {src.name}")
                if verbose or ptxas_verbose:
                    sys.stderr.write(r.stderr)
    if force or jobs or stale(OUT, objs):
        # static cudart: the library shares the process's CUDA context (and torch's streams) through the
        # driver; no particular libcudart.so must be on the loader path
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(OUT), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("linking liblowbit_b200.so failed")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print registers / spills / shared memory per kernel")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas))
