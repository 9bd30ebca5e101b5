"""Operator API of the B200 W4A16 library: weights on the GPU, decode GEMV / skinny GEMM, prefill dequantize.

Drop-in for lowbit/ops.py of YuchenHe985/lowbit-kernels: the same public names, arguments, defaults and
exceptions. What differs is underneath: the kernels are hand-written for sm_100a and reached through a C ABI
(include/lowbit_b200.h, loaded by ``ext()``), layouts are built on the GPU, and the row-count dispatch
constants come from a B200 sweep (dispatch_b200.json).

Kernel versions (``gemv(x, wq, version)``; the reference's numbering, csrc/w4_gemv.cu:1-22):
  1, 2  canonical layout, M <= 8        -- compatibility kernels (fp32 accumulation)
  3, 4  v3 layout, M <= 8               -- compatibility kernels (fp32 accumulation)
  6     mma layout, M <= 8              -- the decode GEMV (tensor-core fragments fed from registers)
  5     mma layout, M <= 64             -- the skinny tensor-core GEMM
"""
import json
import os
import pathlib

import torch

from . import quant
from ._lib import Ext

_EXT = None


def ext():
    """The kernel library (built ahead of time by build.py; no JIT, no fallback). Raises if it cannot load."""
    global _EXT
    if _EXT is None:
        _EXT = Ext()
    return _EXT


LAYOUTS = ("canonical", "v3", "mma")


def _to_device_u8(a, device):
    t = a if isinstance(a, torch.Tensor) else torch.from_numpy(a)
    return t.to(device=device, dtype=torch.uint8).contiguous()


def _to_device_f16(a, device):
    t = a if isinstance(a, torch.Tensor) else torch.from_numpy(a)
    return t.to(device=device, dtype=torch.float16).contiguous()


class W4Weight:
    """One linear layer's weight in the lowbit/quant.py format, on the GPU. `layouts` picks which copies to keep:
    canonical (versions 1, 2, dequantize), v3 (3, 4), mma (5, 6, dequantize; K and the group size multiples of
    128). None = every layout this shape supports; a model keeps ("mma",). Prefill dequantizes, so one of
    canonical / mma must be kept. `packed` is the canonical layout as a numpy array or a torch tensor (host or
    GPU); the other layouts are built from it on the GPU (lowbit/ops.py:24-54)."""

    def __init__(self, packed, scales, group, layouts=None, device=None):
        self.group = group
        self.n, self.k = int(packed.shape[0]), int(packed.shape[1]) * 2
        mma_ok = self.k % 128 == 0 and group % 128 == 0
        if layouts is None:
            layouts = LAYOUTS if mma_ok else ("canonical", "v3")
        if not set(layouts) <= set(LAYOUTS):
            raise ValueError(f"unknown layout in {layouts}; choose from {LAYOUTS}")
        if "mma" in layouts and not mma_ok:
            raise ValueError(f"the mma layout needs K and the group size to be multiples of 128 (K={self.k}, G={group})")
        if "canonical" not in layouts and "mma" not in layouts:
            raise ValueError("keep the canonical or the mma layout: prefill dequantizes from one of them")
        if device is None:
            device = packed.device if isinstance(packed, torch.Tensor) and packed.is_cuda else torch.device("cuda")
        canonical = _to_device_u8(packed, device)
        self.scales = _to_device_f16(scales, device)
        self.packed_v3 = ext().w4_repack(canonical, "v3") if "v3" in layouts else None
        self.packed_mma = ext().w4_repack(canonical, "mma") if "mma" in layouts else None
        self.packed = canonical if "canonical" in layouts else None

    @classmethod
    def from_float(cls, w, group=128, layouts=None):
        """Quantize a float weight [N, K] (on the GPU, bit-identical to quant.quantize_w4) and keep `layouts`."""
        packed, scales = quantize_w4_gpu(w, group)
        return cls(packed, scales, group, layouts)

    def nbytes(self):
        """Bytes of one copy of the weight (packed values + scales), whatever layouts are kept."""
        return self.n * self.k // 2 + self.scales.numel() * 2

    def launch_args(self, version):
        """(packed pointer, scales pointer, device index) of the layout `version` reads, or None if that layout is
        not kept or not launchable; validated once per tensor object (replacing a layout tensor revalidates)."""
        if version == 5 or version == 6:   # the decode path: one attribute holds the mma copy's arguments
            hit = self.__dict__.get("_mma_launch")
            if hit is not None and hit[0] is self.packed_mma and hit[1] is self.scales:
                return hit[2]
        w, s = getattr(self, NEEDS[version]), self.scales
        cache = self.__dict__.setdefault("_launch", {})
        hit = cache.get(version)
        if hit is not None and hit[0] is w and hit[1] is s:
            return hit[2]
        args = None
        if (w is not None and w.is_cuda and s.is_cuda and w.device == s.device and w.dtype == torch.uint8
                and s.dtype == torch.float16 and w.is_contiguous() and s.is_contiguous() and w.dim() == 2
                and s.dim() == 2 and tuple(w.shape) == (self.n, self.k // 2) and self.group > 0
                and self.group % 32 == 0 and self.k % self.group == 0
                and tuple(s.shape) == (self.n, self.k // self.group)):
            args = (w.data_ptr(), s.data_ptr(), w.get_device())
        cache[version] = (w, s, args)
        if version == 5 or version == 6:
            self.__dict__["_mma_launch"] = (w, s, args)
        return args


def pick_rows(n, m):
    """Rows per warp the compatibility kernels (versions 1-4) use when rows_per_warp = 0 (csrc/w4_gemv.cu:424-427)."""
    return 4 if n >= 512 else 2 if m >= 4 else 1


# the layout each kernel version reads, and the most rows it takes
NEEDS = {1: "packed", 2: "packed", 3: "packed_v3", 4: "packed_v3", 5: "packed_mma", 6: "packed_mma"}
MAX_ROWS = {1: 8, 2: 8, 3: 8, 4: 8, 5: 64, 6: 8}


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_raw_device = getattr(torch._C, "_cuda_getDevice", None)
_F16 = torch.float16
_fast = None   # the _fastcall extension module, or False where it was not built (ctypes carries every call then)
_tc = None     # the _torchcall extension module (tensor checks in C++), or False where it was not built


def _current_stream(dev):
    return _raw_stream(dev) if _raw_stream is not None else torch.cuda.current_stream(dev).cuda_stream


def _fastcall():
    global _fast
    if _fast is None:
        try:
            from . import _fastcall as fc
            ext()   # the library itself, loaded and checked by the ctypes binding (the extension links the same file)
            _fast = fc
        except ImportError:
            _fast = False
    return _fast


def _torchcall():
    global _tc
    if _tc is None:
        try:
            from . import _torchcall as tc
            ext()   # the library itself, loaded and checked by the ctypes binding (the extension links the same file)
            _tc = tc
        except ImportError:
            _tc = False
    return _tc


def _gemv_fast(x, wq, version, out, bias=None):
    """The common decode call with the weight's validated launch arguments cached: cheap checks on x, out and bias,
    one C call -- through the _torchcall extension (the checks in C++) when it was built, else the checks here and
    the _fastcall extension or ctypes. None when anything is unusual: the checked path below then handles it (and
    raises its errors)."""
    args = wq.launch_args(version)
    if args is None:
        return None
    tc = _tc if _tc is not None else _torchcall()
    if tc:
        return tc.gemv(x, args[0], args[1], args[2], wq.n, wq.k, wq.group, version, out, bias)
    if type(x) is not torch.Tensor or x.dtype is not _F16 or x.dim() != 2:
        return None
    w_ptr, s_ptr, dev = args
    m, kx = x.shape
    if (kx != wq.k or m == 0 or x.get_device() != dev or not x.is_contiguous()
            or (_raw_device() if _raw_device is not None else torch.cuda.current_device()) != dev):
        return None
    if bias is not None and (type(bias) is not torch.Tensor or bias.dtype is not _F16 or bias.dim() != 1
                             or bias.shape[0] != wq.n or bias.get_device() != dev or not bias.is_contiguous()):
        return None
    n = wq.n
    if out is None:
        y = torch.empty((m, n), dtype=_F16, device=x.device)
    elif (type(out) is torch.Tensor and out.dtype is _F16 and out.dim() == 2 and out.shape[0] == m
          and out.shape[1] == n and out.get_device() == dev and out.is_contiguous()):
        y = out
    else:
        return None
    fc = _fast if _fast is not None else _fastcall()
    st = _current_stream(dev)
    if fc:
        if bias is None:
            rc = fc.gemv(x.data_ptr(), w_ptr, s_ptr, y.data_ptr(), m, n, kx, wq.group, version, st)
        else:
            rc = fc.linear(x.data_ptr(), w_ptr, s_ptr, bias.data_ptr(), y.data_ptr(), m, n, kx, wq.group, version, st)
    else:
        lib = ext().lib
        if bias is not None:
            rc = lib.lb_w4_linear(x.data_ptr(), w_ptr, s_ptr, bias.data_ptr(), y.data_ptr(), m, n, kx, wq.group,
                                  version, st)
        elif version == 6:
            rc = lib.lb_w4_gemv(x.data_ptr(), w_ptr, s_ptr, y.data_ptr(), m, n, kx, wq.group, 6, 0, st)
        else:
            rc = lib.lb_w4_gemm_tc(x.data_ptr(), w_ptr, s_ptr, y.data_ptr(), m, n, kx, wq.group, 0, st)
    if rc:
        ext()._raise(rc)
    return y


def gemv(x, wq, version=4, rows_per_warp=0, out=None, bias=None):
    """x [M, K] fp16 -> [M, N] fp16. Versions 1-4 and 6: M <= 8; version 5: M <= 64 (tensor cores).
    Versions 5 and 6 read the same layout (packed_mma), so a model needs only that copy. `out`: an optional
    contiguous fp16 [M, N] tensor the result is written into (no allocation). `bias`: an optional fp16 [N] tensor
    added in the kernel's epilogue, with the roundings of adding it to the fp16 output afterwards (both are
    additions to the reference's signature)."""
    if (version == 5 or version == 6) and rows_per_warp == 0 and isinstance(wq, W4Weight):
        y = _gemv_fast(x, wq, version, out, bias)
        if y is not None:
            return y
    if version not in NEEDS:
        raise ValueError(f"version must be one of {sorted(NEEDS)}")
    if getattr(wq, NEEDS[version]) is None:
        raise ValueError(f"v{version} reads {NEEDS[version]}, which this W4Weight does not keep")
    if bias is not None:
        if rows_per_warp != 0:
            raise ValueError("rows_per_warp is chosen by the kernel when a bias is fused")
        return ext().w4_linear(x.contiguous(), getattr(wq, NEEDS[version]), wq.scales, wq.group, version, bias, out)
    if version == 5:
        return ext().w4_gemm_tc(x.contiguous(), wq.packed_mma, wq.scales, wq.group, rows_per_warp, out=out)
    w = wq.packed_mma if version == 6 else wq.packed_v3 if version >= 3 else wq.packed
    return ext().w4_gemv(x.contiguous(), w, wq.scales, wq.group, version, rows_per_warp, out=out)


_GEMV = gemv   # linear()'s shortcut applies only while ops.gemv is this function (tests may replace it)


def quantize_w4_gpu(w, group=128, clip_grid=None, rows_per_pass=2048):
    """Same format and, with clip_grid=None, the same bits as quant.quantize_w4, computed by the quantize kernel.
    clip_grid, e.g. (1.0, 0.95, ..., 0.75): per group, try scale = a * amax / 7 for each a and keep the first one
    with the smallest squared weight error. Returns (packed uint8 [N, K/2], scales fp16 [N, K/G]) on the GPU.
    Rows are converted and quantized `rows_per_pass` at a time, which bounds the fp32 staging copy
    (lowbit/ops.py:81-116)."""
    n, k = w.shape
    if group <= 0 or k % group or group % 32:
        raise ValueError(f"K={k} must be a multiple of the group size {group}, itself a multiple of 32")
    if clip_grid is not None and len(clip_grid) > 32:
        raise ValueError("clip_grid holds at most 32 factors")
    dev = w.device if isinstance(w, torch.Tensor) and w.is_cuda else torch.device("cuda")
    if not isinstance(w, torch.Tensor):
        w = torch.as_tensor(w)
    packed = torch.empty(n, k // 2, dtype=torch.uint8, device=dev)
    scales = torch.empty(n, k // group, dtype=torch.float16, device=dev)
    for r0 in range(0, n, rows_per_pass):
        part = w[r0:r0 + rows_per_pass].detach()
        if part.dtype not in (torch.float32, torch.float16):
            part = part.float()
        p, s = ext().w4_quantize(part.to(dev).contiguous(), group, clip_grid)
        packed[r0:r0 + rows_per_pass] = p
        scales[r0:r0 + rows_per_pass] = s
    return packed, scales


def dequantize_w4_gpu(packed, scales, group=128):
    """fp16 [N, K] from canonical packed weights on the GPU: (u - 8) * scale rounded once to fp16, the bits the
    reference's lowbit/ops.py:119-123 gives. Host arrays belong to quant.dequantize_w4."""
    if not (isinstance(packed, torch.Tensor) and packed.is_cuda):
        raise RuntimeError("dequantize_w4_gpu takes GPU tensors; use lowbit.quant.dequantize_w4 for host arrays")
    return ext().w4_dequant(packed.contiguous(), scales.contiguous(), group, layout="canonical")


def dequant(wq, layout=None):
    """fp16 W [N, K] from the canonical or the mma copy (None: canonical when kept). Both give the same bits."""
    if layout is None:
        layout = "canonical" if wq.packed is not None else "mma"
    if layout == "canonical" and wq.packed is not None:
        return ext().w4_dequant(wq.packed, wq.scales, wq.group)
    if layout == "mma" and wq.packed_mma is not None:
        return ext().w4_dequant(wq.packed_mma, wq.scales, wq.group, True)
    raise ValueError(f"cannot dequantize from the {layout} layout: not kept")


# ------------------------------------------------------------------------------------------ dispatch constants
#
# linear() picks, by row count and layer width: version 6 for up to AUTO_GEMV_ROWS rows, version 5 up to
# AUTO_V5_ROWS rows (AUTO_V5_WIDE_ROWS on layers with N >= AUTO_WIDE_N), dequantize + cuBLAS above. The values
# come from dispatch_b200.json (a B200 sweep). LOWBIT_DISPATCH=reference restores the reference's T4 values
# (lowbit/ops.py:142), under which the reference's own dispatch tests hold verbatim.

_REFERENCE_TABLE = {"AUTO_GEMV_ROWS": 1, "AUTO_V5_ROWS": 32, "AUTO_V5_WIDE_ROWS": 64, "AUTO_WIDE_N": 3072}
DISPATCH_TABLE_PATH = pathlib.Path(__file__).resolve().parent / "dispatch_b200.json"


def _load_dispatch():
    if os.environ.get("LOWBIT_DISPATCH", "") == "reference":
        return dict(_REFERENCE_TABLE, source="reference T4 constants (lowbit/ops.py:142)")
    table = json.loads(DISPATCH_TABLE_PATH.read_text())
    return table


DISPATCH = _load_dispatch()
AUTO_GEMV_ROWS, AUTO_V5_ROWS, AUTO_V5_WIDE_ROWS, AUTO_WIDE_N = (
    int(DISPATCH[k]) for k in ("AUTO_GEMV_ROWS", "AUTO_V5_ROWS", "AUTO_V5_WIDE_ROWS", "AUTO_WIDE_N"))


def gemm_chunked(x, wq, chunk=64):
    """Many rows through version 5 in 64-row slices (no fp16 weight copy is written)."""
    return torch.cat([gemv(x[i:i + chunk], wq, 5) for i in range(0, x.shape[0], chunk)])


def auto_version(m, wq):
    """The kernel linear() uses for m rows, or None for dequantize + cuBLAS. Weights without the mma layout use
    version 4 / 2 up to 8 rows (lowbit/ops.py:151-160)."""
    if wq.packed_mma is not None:
        if m <= AUTO_GEMV_ROWS:
            return 6
        return 5 if m <= (AUTO_V5_WIDE_ROWS if wq.n >= AUTO_WIDE_N else AUTO_V5_ROWS) else None
    if m <= 8:
        return 4 if wq.packed_v3 is not None else 2 if wq.packed is not None else None
    return None


def linear(x, wq, max_gemv_rows=8, version=0, out=None, bias=None):
    """Decode (few rows): an INT4 kernel; prefill (many rows): dequantize, then cuBLAS fp16 GEMM. version 0 =
    auto_version; a fixed version runs up to min(max_gemv_rows, its row limit) rows (version 5: 64), and
    dequantize + cuBLAS above that (lowbit/ops.py:163-178). Additions to the reference's signature: `out`, an
    optional contiguous fp16 [M, N] tensor that receives the result, and `bias`, an optional fp16 [N] tensor added
    to the result (in the INT4 kernels' epilogue; after the cuBLAS product on the prefill path) with the roundings
    of adding it to the fp16 output."""
    m = x.shape[0]
    if version == 0 and m and type(wq) is W4Weight and wq.packed_mma is not None and gemv is _GEMV:
        # the decode call: the rule of auto_version inline, straight to the cached launch (anything unusual falls
        # through to the general path below)
        v = 6 if m <= AUTO_GEMV_ROWS else 5 if m <= (AUTO_V5_WIDE_ROWS if wq.n >= AUTO_WIDE_N else AUTO_V5_ROWS) else 0
        if v:
            y = _gemv_fast(x, wq, v, out, bias)
            if y is not None:
                return y
    if m == 0:
        return x.new_empty(0, wq.n) if out is None else out
    if version == 0:
        v = auto_version(m, wq)
    elif version in MAX_ROWS:
        v = version if m <= (MAX_ROWS[5] if version == 5 else min(max_gemv_rows, MAX_ROWS[version])) else None
    else:
        raise ValueError(f"version must be 0 (auto) or one of {sorted(MAX_ROWS)}")
    if v is not None:
        if bias is not None:
            return gemv(x, wq, v, out=out, bias=bias)
        return gemv(x, wq, v) if out is None else gemv(x, wq, v, out=out)
    y = torch.nn.functional.linear(x, dequant(wq, "mma" if wq.packed_mma is not None else "canonical"))
    if bias is not None:
        y = y + bias
    if out is None:
        return y
    if out.shape != y.shape or out.dtype != y.dtype:
        raise RuntimeError(f"out must be a float16 {tuple(y.shape)} tensor")
    return out.copy_(y)
