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


FASTCALL_SRC = CSRC / "lb_pyfast.c"
FASTCALL_OUT = ROOT / "lowbit" / "_fastcall.so"


TORCHCALL_SRC = CSRC / "lb_torchcall.cpp"
TORCHCALL_OUT = ROOT / "lowbit" / "_torchcall.so"


def sources():
    return sorted(CSRC.glob("*.cu"))


def build_torchcall(force=False, verbose=False):
    """The CPython extension lowbit/_torchcall.so (ops.gemv's decode path with its tensor checks in C++), compiled
    against torch's headers and linked to torch's libraries and, with an $ORIGIN run path, to liblowbit_b200.so."""
    import sysconfig
    import torch
    from torch.utils import cpp_extension
    deps = [TORCHCALL_SRC, OUT] + sorted(INCLUDE.glob("*.h"))
    if not force and not stale(TORCHCALL_OUT, deps):
        return TORCHCALL_OUT
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("a C++ compiler is needed for lowbit/_torchcall.so")
    torch_lib = pathlib.Path(torch.__file__).resolve().parent / "lib"
    abi = int(torch.compiled_with_cxx11_abi())
    incs = [f"-I{p}" for p in cpp_extension.include_paths(device_type="cuda")]
    cmd = [cxx, "-O2", "-shared", "-fPIC", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", sysconfig.get_paths()["include"], "-I", str(INCLUDE), *incs, str(TORCHCALL_SRC),
           "-L", str(OUT.parent), "-l:" + OUT.name, "-L", str(torch_lib), "-lc10", "-lc10_cuda", "-ltorch",
           "-ltorch_cpu", "-ltorch_python", f"-Wl,-rpath,$ORIGIN:{torch_lib}", "-o", str(TORCHCALL_OUT)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("building lowbit/_torchcall.so failed")
    return TORCHCALL_OUT


def build_fastcall(force=False, verbose=False):
    """The CPython extension lowbit/_fastcall.so (the decode call path without ctypes), linked to the library with
    an $ORIGIN run path so it loads the same liblowbit_b200.so beside it."""
    import sysconfig
    deps = [FASTCALL_SRC, OUT] + sorted(INCLUDE.glob("*.h"))
    if not force and not stale(FASTCALL_OUT, deps):
        return FASTCALL_OUT
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("a C compiler is needed for lowbit/_fastcall.so")
    cmd = [cc, "-O2", "-shared", "-fPIC", "-I", sysconfig.get_paths()["include"], "-I", str(INCLUDE),
           str(FASTCALL_SRC), "-L", str(OUT.parent), "-l:" + OUT.name, "-Wl,-rpath,$ORIGIN", "-o", str(FASTCALL_OUT)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("building lowbit/_fastcall.so failed")
    return FASTCALL_OUT


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
    build_fastcall(force, verbose)
    build_torchcall(force, verbose)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print registers / spills / shared memory per kernel")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas))
