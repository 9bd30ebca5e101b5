"""ctypes binding of liblowbit_b200.so (include/lowbit_b200.h) for torch tensors.

``Ext`` offers the reference extension's three bindings (csrc/w4_gemv.cu:542-550) with the same names,
arguments and error behaviour -- ``w4_gemv``, ``w4_gemm_tc``, ``w4_dequant`` -- plus ``w4_quantize`` and
``w4_repack``. Tensor checks raise RuntimeError like the reference's TORCH_CHECK (csrc/w4_gemv.cu:312-325);
the C library validates sizes and alignment and its messages are raised the same way. Every call launches on
the current torch stream of the tensors' device and never synchronizes.

There is no fallback: if the library or a CUDA device is missing, the first call raises.
"""
import ctypes
import pathlib

import torch

LIB_PATH = pathlib.Path(__file__).resolve().parent / "liblowbit_b200.so"
LAYOUT_IDS = {"canonical": 0, "v3": 1, "mma": 2}
OPTIONS = {"pdl": 0, "early_weights": 1, "gemv_ksplit": 2, "gemv_warps": 3, "gemv_depth": 4, "gemv_kernel": 5, "gemv_rowtiles": 6}

_P, _I64, _I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int

# every entry point include/lowbit_b200.h declares, with its ctypes signature
SIGNATURES = {
    "lb_abi_version": ([], _I),
    "lb_status_string": ([_I], ctypes.c_char_p),
    "lb_last_error": ([], ctypes.c_char_p),
    "lb_device_error": ([], _I),
    "lb_clear_device_error": ([], None),
    "lb_set_option": ([_I, _I], _I),
    "lb_get_option": ([_I], _I),
    "lb_w4_gemv": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _P], _I),
    "lb_w4_gemm_tc": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _P], _I),
    "lb_w4_linear": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _P], _I),
    "lb_w4_dequant": ([_P, _P, _P, _I64, _I64, _I64, _I, _P], _I),
    "lb_w4_quantize": ([_P, _I, _P, _P, _I64, _I64, _I64, _P, _I, _P], _I),
    "lb_w4_repack": ([_P, _P, _I64, _I64, _I, _P], _I),
    "lb_decode_embed": ([_P, _P, _P, _I64, _P], _I),
    "lb_decode_rmsnorm": ([_P, _P, _P, _P, _I64, ctypes.c_float, _P], _I),
    "lb_decode_attention_splits": ([_I64], _I),
    "lb_decode_attention": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I64, _P], _I),
    "lb_decode_silu_mul": ([_P, _P, _I64, _P], _I),
    "lb_decode_attention_noalloc": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I64, _P], _I),
    "lb_decode_gemv_fusable": ([_I64, _I64], _I),
    "lb_tp_allreduce": ([_P, _P, _I64, _I64, _P, _P, _I, _I, _P], _I),
    "lb_tp_allreduce_norm": ([_P, _I64, _I64, _P, _P, _I, _I, _P, _P, _P, ctypes.c_float, _P], _I),
    "lb_decode_gemv_swiglu": ([_P, _P, _P, _P, _I64, _I64, _I64, _P], _I),
    "lb_tp_gemv_allreduce_norm": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _I, _I, _P, _P, _P, ctypes.c_float,
                                   _P, _P], _I),
    "lb_decode_gemv_residual_norm": ([_P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, ctypes.c_float, _P, _P], _I),
    "lb_decode_norm_gemv": ([_P, _P, _P, _P, ctypes.c_float, _P, _P, _P, _I64, _I64, _I64, _P], _I),
    "lb_decode_swiglu_gemv": ([_P, _P, _P, _P, _I64, _I64, _I64, _P], _I),
}


def load_library(path=LIB_PATH):
    """dlopen the kernel library and attach the ctypes signatures. Loading needs no GPU."""
    if not pathlib.Path(path).exists():
        raise RuntimeError(f"{path} is missing: build it with `python lowbit-kernels_b200/build.py` "
                           "(this package has no CPU or fallback implementation)")
    lib = ctypes.CDLL(str(path))
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, res
    return lib


def _check(x, w, s, group):
    """csrc/w4_gemv.cu:312-325 (the parts that need tensor metadata)."""
    if not (x.is_cuda and w.is_cuda and s.is_cuda):
        raise RuntimeError("tensors must be on the GPU")
    if w.device != x.device or s.device != x.device:
        raise RuntimeError("x, w and scales must be on the same GPU")
    if group <= 0:
        raise RuntimeError("group size must be positive")
    if x.dtype != torch.float16 or s.dtype != torch.float16 or w.dtype != torch.uint8:
        raise RuntimeError("x and scales must be float16, packed weights uint8")
    if not (x.is_contiguous() and w.is_contiguous() and s.is_contiguous()):
        raise RuntimeError("tensors must be contiguous")
    if x.dim() != 2 or w.dim() != 2 or s.dim() != 2:
        raise RuntimeError("x [M,K], w [N,K/2], scales [N,K/G]")
    k = x.shape[1]
    if group % 32 or k % group:
        raise RuntimeError("K must be a multiple of the group size, itself a multiple of 32")
    if w.shape[1] * 2 != k or s.shape[0] != w.shape[0] or s.shape[1] != k // group:
        raise RuntimeError("shape mismatch")


def _out(out, m, n, device):
    """The output tensor: a new [m, n] fp16 tensor, or `out` after checking that it is one."""
    if out is None:
        return torch.empty((m, n), dtype=torch.float16, device=device)
    if out.shape != (m, n) or out.dtype != torch.float16 or out.device != device or not out.is_contiguous():
        raise RuntimeError(f"out must be a contiguous float16 [{m}, {n}] tensor on {device}")
    return out


class _Device:
    """Make `dev` the current CUDA device for one call (the reference's CUDAGuard), cheaply."""
    __slots__ = ("dev", "prev")

    def __init__(self, dev):
        self.dev, self.prev = dev.index, None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


class Ext:
    """The kernel library with the reference extension's call surface."""

    def __init__(self, lib=None):
        if not torch.cuda.is_available():
            raise RuntimeError("lowbit_b200 needs a CUDA device (sm_100a); none is visible")
        self.lib = lib or load_library()

    def _raise(self, rc):
        msg = self.lib.lb_last_error().decode() or self.lib.lb_status_string(rc).decode()
        raise RuntimeError(msg)

    def set_option(self, name, value):
        """Process-wide launch options (include/lowbit_b200.h, lb_option); returns the previous value."""
        return self.lib.lb_set_option(OPTIONS[name], int(value))

    def get_option(self, name):
        return self.lib.lb_get_option(OPTIONS[name])

    def w4_gemv(self, x, w, s, group, version, rows_per_warp=0, out=None):
        _check(x, w, s, group)
        m, k, n = x.shape[0], x.shape[1], w.shape[0]
        y = _out(out, m, n, x.device)
        with _Device(x.device):
            rc = self.lib.lb_w4_gemv(x.data_ptr(), w.data_ptr(), s.data_ptr(), y.data_ptr(), m, n, k, group,
                                     int(version), int(rows_per_warp), torch.cuda.current_stream().cuda_stream)
        if rc:
            self._raise(rc)
        return y

    def w4_gemm_tc(self, x, w, s, group, row_tiles=0, out=None):
        _check(x, w, s, group)
        m, k, n = x.shape[0], x.shape[1], w.shape[0]
        y = _out(out, m, n, x.device)
        with _Device(x.device):
            rc = self.lib.lb_w4_gemm_tc(x.data_ptr(), w.data_ptr(), s.data_ptr(), y.data_ptr(), m, n, k, group,
                                        int(row_tiles), torch.cuda.current_stream().cuda_stream)
        if rc:
            self._raise(rc)
        return y

    def w4_linear(self, x, w, s, group, version, bias=None, out=None):
        """x [M, K] @ dequant(W)^T + bias with the bias added in the kernel epilogue (lb_w4_linear): version 1-4, 6
        (M <= 8) or 5 (M <= 64). bias: fp16 [N] on the same GPU, or None."""
        _check(x, w, s, group)
        m, k, n = x.shape[0], x.shape[1], w.shape[0]
        if bias is not None and (not bias.is_cuda or bias.device != x.device or bias.dtype != torch.float16
                                 or bias.dim() != 1 or bias.shape[0] != n or not bias.is_contiguous()):
            raise RuntimeError(f"bias must be a contiguous float16 [{n}] tensor on {x.device}")
        y = _out(out, m, n, x.device)
        with _Device(x.device):
            rc = self.lib.lb_w4_linear(x.data_ptr(), w.data_ptr(), s.data_ptr(),
                                       None if bias is None else bias.data_ptr(), y.data_ptr(), m, n, k, group,
                                       int(version), torch.cuda.current_stream().cuda_stream)
        if rc:
            self._raise(rc)
        return y

    def w4_dequant(self, w, s, group, mma_layout=False, layout=None):
        """fp16 [N, K] from packed weights; layout: "canonical", "v3" or "mma" (mma_layout=True = "mma")."""
        if not (w.is_cuda and s.is_cuda and w.device == s.device):
            raise RuntimeError("packed weights and scales must be on the same GPU")
        if w.dtype != torch.uint8 or s.dtype != torch.float16:
            raise RuntimeError("packed weights uint8, scales float16")
        if w.dim() != 2 or s.dim() != 2 or group <= 0:
            raise RuntimeError("w [N,K/2], scales [N,K/G], positive group size")
        if not (w.is_contiguous() and s.is_contiguous()):
            raise RuntimeError("packed weights must be contiguous and 16-byte aligned")
        n, k = w.shape[0], w.shape[1] * 2
        if group % 32 or k % group or s.shape[0] != n or s.shape[1] != k // group:
            raise RuntimeError("shape mismatch")
        lid = LAYOUT_IDS[layout] if layout is not None else (2 if mma_layout else 0)
        out = torch.empty((n, k), dtype=torch.float16, device=w.device)
        with _Device(w.device):
            rc = self.lib.lb_w4_dequant(w.data_ptr(), s.data_ptr(), out.data_ptr(), n, k, group, lid,
                                        torch.cuda.current_stream().cuda_stream)
        if rc:
            self._raise(rc)
        return out

    def w4_quantize(self, w, group=128, clip_grid=None):
        """W fp32/fp16 [N, K] on the GPU -> (canonical packed uint8 [N, K/2], scales fp16 [N, K/G])."""
        if not w.is_cuda:
            raise RuntimeError("tensors must be on the GPU")
        if w.dim() != 2:
            raise RuntimeError("W must be 2-D [N, K]")
        if w.dtype not in (torch.float32, torch.float16):
            w = w.float()
        w = w.contiguous()
        n, k = w.shape
        if group <= 0 or k % group or group % 32:
            raise ValueError(f"K={k} must be a multiple of the group size {group}, itself a multiple of 32")
        packed = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
        scales = torch.empty((n, k // group), dtype=torch.float16, device=w.device)
        grid = None
        n_clip = 0
        if clip_grid:
            vals = [float(a) for a in clip_grid]
            n_clip = len(vals)
            grid = (ctypes.c_float * n_clip)(*vals)
        with _Device(w.device):
            rc = self.lib.lb_w4_quantize(w.data_ptr(), int(w.dtype == torch.float16), packed.data_ptr(),
                                         scales.data_ptr(), n, k, group,
                                         ctypes.cast(grid, ctypes.c_void_p) if grid is not None else None, n_clip,
                                         torch.cuda.current_stream().cuda_stream)
        if rc:
            self._raise(rc)
        return packed, scales

    def w4_repack(self, packed, layout):
        """Canonical packed uint8 [N, K/2] on the GPU -> the "v3" or "mma" layout (a new tensor)."""
        if not packed.is_cuda or packed.dtype != torch.uint8 or packed.dim() != 2:
            raise RuntimeError("packed weights must be a 2-D uint8 GPU tensor")
        packed = packed.contiguous()
        n, k = packed.shape[0], packed.shape[1] * 2
        if layout == "mma" and k % 128:
            raise ValueError(f"K={k} must be a multiple of 128 for the tensor-core layout")
        out = torch.empty_like(packed)
        with _Device(packed.device):
            rc = self.lib.lb_w4_repack(packed.data_ptr(), out.data_ptr(), n, k, LAYOUT_IDS[layout],
                                       torch.cuda.current_stream().cuda_stream)
        if rc:
            self._raise(rc)
        return out
