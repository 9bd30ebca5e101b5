"""The reference's own CUDA kernels, built unchanged for sm_100a -- TEST INFRASTRUCTURE ONLY.

The reference's native code is one torch extension, csrc/w4_gemv.cu of YuchenHe985/lowbit-kernels (bindings
w4_gemv, w4_gemm_tc, w4_dequant at csrc/w4_gemv.cu:542-550). ``build()`` compiles that file where it lies in the
reference checkout (read-only; nothing is copied) with torch.utils.cpp_extension, for sm_100a, into oracle/_ref/
(git-ignored, but shipped with the tree so the GPU box can load it without the reference checkout). ``load()``
imports the prebuilt module from oracle/_ref/ by path.

Used by tests/ and bench.py as the bar the north star names: the reference kernel's speed per shape (gemv_v6 at
M = 1, gemm_v5 at M = 2..64) and its error per case ("no worse than the reference kernel's error",
bench/gpu_run.py:231-245). Never imported by the library in lowbit-kernels_b200/.
"""
import importlib.machinery
import importlib.util
import os
import pathlib

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "lowbit_ref_ext"
# where the reference checkout lies in the build container; the GPU box only loads the prebuilt module
REFERENCE_SRC = pathlib.Path(os.environ.get("LOWBIT_REFERENCE", "/root/reference")) / "csrc" / "w4_gemv.cu"

_mod = None


def module_path():
    """The built extension module in oracle/_ref/, or None when it has not been built."""
    hits = sorted(OUT.glob(NAME + "*.so"))
    return hits[0] if hits else None


def build(verbose=False):
    """Compile the reference's csrc/w4_gemv.cu for sm_100a into oracle/_ref/. Returns the module path, or None
    when the reference checkout is absent (a prebuilt module, if any, is kept)."""
    if not REFERENCE_SRC.exists():
        return module_path()
    OUT.mkdir(exist_ok=True)
    have = module_path()
    if have is not None and have.stat().st_mtime >= REFERENCE_SRC.stat().st_mtime:
        return have
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils import cpp_extension
    cpp_extension.load(name=NAME, sources=[str(REFERENCE_SRC)], build_directory=str(OUT),
                       extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo"],
                       extra_cflags=["-O3"], verbose=verbose)
    return module_path()


def load():
    """Import the prebuilt reference extension (torch must be importable). Raises when it was never built."""
    global _mod
    if _mod is None:
        path = module_path()
        if path is None:
            raise RuntimeError("the reference extension is not built: run oracle.ref_kernel.build() where the "
                               "reference checkout is present")
        import torch  # noqa: F401  (the module links against libtorch)
        loader = importlib.machinery.ExtensionFileLoader(NAME, str(path))
        spec = importlib.util.spec_from_file_location(NAME, str(path), loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _mod = mod
    return _mod


def available():
    return module_path() is not None
