"""CPU oracle for the W4A16 path -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU legs as the checker; never by the library in
lowbit-kernels_b200/. Two restatements of the reference's arithmetic live here:

* ``C``: ctypes bindings to lb_oracle.c (built by ``make -C oracle``): bit-level format transforms and the fp64
  GEMV in plain C, used as the independent checker of the CUDA kernels.
* numpy / torch restatements of the reference's CPU path, lowbit/quant.py:23-84 and lowbit/ops.py:119-123
  (dequantize, then a matmul), used as the timed CPU baseline.

Parity of both is pinned against golden vectors that the reference's own Python produced
(tests/golden/make_golden.py -> tests/golden/*.npz) in tests/test_oracle.py.
"""
import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "liblb_oracle.so"
LAYOUT_IDS = {"canonical": 0, "v3": 1, "mma": 2}

_lib = None


def build():
    """Compile lb_oracle.c into liblb_oracle.so with the Makefile beside it."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.lbo_f32_to_f16.argtypes, L.lbo_f32_to_f16.restype = [ctypes.c_float], ctypes.c_uint16
        L.lbo_f16_to_f32.argtypes, L.lbo_f16_to_f32.restype = [ctypes.c_uint16], ctypes.c_float
        L.lbo_quantize.argtypes = [p, i64, i64, i64, p, p]
        L.lbo_dequantize_f32.argtypes = [p, p, i64, i64, i64, p]
        L.lbo_dequantize_f16.argtypes = [p, p, i64, i64, i64, p]
        L.lbo_interleave_gpu.argtypes = [p, i64, i64, p]
        L.lbo_interleave_mma.argtypes = [p, i64, i64, p]
        L.lbo_dequantize_layout_f16.argtypes = [p, i32, p, i64, i64, i64, p]
        L.lbo_gemv_ref.argtypes = [p, i64, p, i32, p, i64, i64, i64, p]
        for f in ("lbo_quantize", "lbo_dequantize_f32", "lbo_dequantize_f16", "lbo_interleave_gpu",
                  "lbo_interleave_mma", "lbo_dequantize_layout_f16", "lbo_gemv_ref"):
            getattr(L, f).restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _ok(rc, what):
    if rc:
        raise ValueError(f"oracle {what} rejected its arguments (code {rc})")


# ---------------------------------------------------------------- C oracle (checker)

def c_quantize(w, group=128):
    """lowbit/quant.py:23-35 in C: W float32 [N, K] -> (packed uint8 [N, K/2], scales float16 [N, K/G])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    packed = np.empty((n, k // 2), np.uint8)
    scales = np.empty((n, max(k // group, 0) if group > 0 else 0), np.float16)
    _ok(lib().lbo_quantize(_ptr(w), n, k, group, _ptr(packed), _ptr(scales)), "quantize")
    return packed, scales


def c_dequantize_f32(packed, scales, group=128):
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = np.ascontiguousarray(scales, np.float16)
    n, k = packed.shape[0], packed.shape[1] * 2
    out = np.empty((n, k), np.float32)
    _ok(lib().lbo_dequantize_f32(_ptr(packed), _ptr(scales), n, k, group, _ptr(out)), "dequantize_f32")
    return out


def c_dequantize_f16(packed, scales, group=128, layout="canonical"):
    """fp16 weights [N, K] = fp16_rn(q * scale) read from the given layout."""
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = np.ascontiguousarray(scales, np.float16)
    n, k = packed.shape[0], packed.shape[1] * 2
    out = np.empty((n, k), np.float16)
    _ok(lib().lbo_dequantize_layout_f16(_ptr(packed), LAYOUT_IDS[layout], _ptr(scales), n, k, group, _ptr(out)),
        "dequantize_f16")
    return out


def c_interleave_gpu(packed):
    packed = np.ascontiguousarray(packed, np.uint8)
    out = np.empty_like(packed)
    _ok(lib().lbo_interleave_gpu(_ptr(packed), packed.shape[0], packed.shape[1] * 2, _ptr(out)), "interleave_gpu")
    return out


def c_interleave_mma(packed):
    packed = np.ascontiguousarray(packed, np.uint8)
    out = np.empty_like(packed)
    _ok(lib().lbo_interleave_mma(_ptr(packed), packed.shape[0], packed.shape[1] * 2, _ptr(out)), "interleave_mma")
    return out


def c_gemv_ref(x16, w, scales, group=128, layout="canonical"):
    """fp64 y [M, N] = x @ dequant(W)^T with x given as float16 [M, K] and W in the given layout."""
    x16 = np.ascontiguousarray(x16, np.float16)
    w = np.ascontiguousarray(w, np.uint8)
    scales = np.ascontiguousarray(scales, np.float16)
    m, k = x16.shape
    n = w.shape[0]
    y = np.empty((m, n), np.float64)
    _ok(lib().lbo_gemv_ref(_ptr(x16), m, _ptr(w), LAYOUT_IDS[layout], _ptr(scales), n, k, group, _ptr(y)), "gemv_ref")
    return y


# ---------------------------------------------------------------- numpy / torch restatement (CPU baseline)

def np_dequantize_w4(packed, scales, group=128):
    """lowbit/quant.py:38-51: unpack nibbles, subtract 8, multiply by the group scale in fp32."""
    packed = np.asarray(packed, np.uint8)
    n, k = packed.shape[0], packed.shape[1] * 2
    q = np.empty((n, k), np.float32)
    q[:, 0::2] = (packed & 0xF).astype(np.float32) - 8
    q[:, 1::2] = (packed >> 4).astype(np.float32) - 8
    s = np.asarray(scales, np.float16).astype(np.float32)
    return (q.reshape(n, k // group, group) * s[:, :, None]).reshape(n, k)


def np_linear(x16, packed, scales, group=128):
    """The reference's numpy CPU path: dequantize_w4 then an fp32 matmul (lowbit/quant.py:47-51)."""
    return np.asarray(x16, np.float32) @ np_dequantize_w4(packed, scales, group).T


def torch_dequantize(packed_t, scales_t, group=128):
    """lowbit/ops.py:119-123 restated on CPU tensors: (u - 8) * scale in fp32, rounded once to fp16."""
    import torch
    u = torch.stack([packed_t & 0xF, packed_t >> 4], -1).reshape(packed_t.shape[0], -1).float() - 8
    n, k = u.shape
    return (u.reshape(n, k // group, group) * scales_t.float()[..., None]).reshape(n, k).half()


def torch_linear(x_t, packed_t, scales_t, group=128):
    """The reference's torch CPU path: dequantize_w4_gpu on CPU tensors, then F.linear in fp32."""
    import torch
    w = torch_dequantize(packed_t, scales_t, group).float()
    return torch.nn.functional.linear(x_t.float(), w)


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
