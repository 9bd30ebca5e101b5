"""The W4A16 weight format: symmetric INT4, one fp16 scale per group of G weights along K.

This module is the host-side definition of the format that every kernel in this package reads. It keeps the
names, argument meanings, bytes and exceptions of lowbit/quant.py in YuchenHe985/lowbit-kernels, so a model
quantized by either library loads in the other.

Format, for an nn.Linear weight W [N, K] (out_features x in_features), group size G (a multiple of 32; K % G == 0):

* ``scale[n, g] = fp16(max|W[n, gG:(g+1)G]| / 7)`` with the division done in fp32; an all-zero group gets 1.0.
* ``q[n, k] = clip(rint(W[n, k] / fp32(scale)), -8, 7)`` (round half to even), stored as the nibble
  ``u = q + 8``.
* canonical bytes: ``byte[n, j] = u[n, 2j] | u[n, 2j + 1] << 4`` (low nibble = even k).

Two reordered copies of the same bytes exist (lowbit/quant.py:55-78):

* the "v3" order: inside every little-endian 32-bit word (8 consecutive k), nibble slot s holds
  ``k0 + SLOT_TO_K[s]``, so ``(word >> 4j) & 0x000F000F`` yields the pair (k0 + 2j, k0 + 2j + 1) in the two
  16-bit halves;
* the "mma" order: inside every 64-byte chunk (128 k) byte ``16t + s`` holds canonical byte ``4s + t``
  (k = 8s + 2t, 8s + 2t + 1), then the v3 slot order is applied to each word. Lane t of a tensor-core quad
  then finds all of its fragment values for one row and one chunk in one 16-byte load.
"""
import numpy as np

QMIN, QMAX, OFFSET = -8, 7, 8

# nibble slot s (bits 4s..4s+3 of a little-endian word) holds the value of k0 + SLOT_TO_K[s]
SLOT_TO_K = np.array([0, 2, 4, 6, 1, 3, 5, 7])

# byte 16t + s of a 64-byte mma chunk is canonical byte 4s + t
MMA_BYTE_ORDER = np.array([4 * s + t for t in range(4) for s in range(16)])


def _check_group(k, group):
    if group <= 0 or k % group or group % 32:
        raise ValueError(f"K={k} must be a multiple of the group size {group}, itself a multiple of 32")


def quantize_w4(w, group=128):
    """W [N, K] float -> (packed uint8 [N, K // 2] canonical, scales float16 [N, K // group]).

    Follows lowbit/quant.py:23-35: amax / 7 in fp32, rounded once to fp16; q = rint(W / scale) in fp32."""
    w = np.asarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError(f"W must be 2-D [N, K], got shape {w.shape}")
    n, k = w.shape
    _check_group(k, group)
    groups = w.reshape(n, k // group, group)
    amax = np.abs(groups).max(axis=2)
    scales = (amax / np.float32(QMAX)).astype(np.float16)
    scales[scales == 0] = np.float16(1.0)
    q = np.rint(groups / scales.astype(np.float32)[:, :, None])
    q = np.clip(q, QMIN, QMAX).astype(np.int16).reshape(n, k)
    u = (q + OFFSET).astype(np.uint8)
    packed = (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)
    return packed, scales


def unpack_w4(packed):
    """packed uint8 [N, K // 2] (canonical order) -> signed int8 [N, K] in -8..7."""
    packed = np.asarray(packed, dtype=np.uint8)
    n, half = packed.shape
    q = np.empty((n, 2 * half), dtype=np.int8)
    q[:, 0::2] = (packed & 0x0F).astype(np.int8) - OFFSET
    q[:, 1::2] = (packed >> 4).astype(np.int8) - OFFSET
    return q


def dequantize_w4(packed, scales, group=128):
    """-> float32 [N, K]: q * scale, exact in fp32 (a 4-bit integer times an fp16 value)."""
    q = unpack_w4(packed).astype(np.float32)
    n, k = q.shape
    s = np.asarray(scales, dtype=np.float16).astype(np.float32)
    return (q.reshape(n, k // group, group) * s[:, :, None]).reshape(n, k)


def _pack_nibbles(u):
    u = u.astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def interleave_for_gpu(packed):
    """Canonical packed [N, K // 2] -> the v3 slot order (same bytes per row, permuted nibbles)."""
    u = unpack_w4(packed).astype(np.int16) + OFFSET
    n, k = u.shape
    if k % 8:
        raise ValueError(f"K={k} must be a multiple of 8")
    words = u.reshape(n, k // 8, 8)[:, :, SLOT_TO_K].reshape(n, k)
    return _pack_nibbles(words)


def interleave_for_mma(packed):
    """Canonical packed [N, K // 2] -> the mma order. K must be a multiple of 128."""
    packed = np.asarray(packed, dtype=np.uint8)
    n, half = packed.shape
    if half % 64:
        raise ValueError(f"K={2 * half} must be a multiple of 128 for the tensor-core layout")
    regrouped = packed.reshape(n, half // 64, 64)[:, :, MMA_BYTE_ORDER].reshape(n, half)
    return interleave_for_gpu(regrouped)


def gemv_reference(x, packed, scales, group=128):
    """y[m, n] = sum_k x[m, k] * dequant(W)[n, k] in float64."""
    w = dequantize_w4(packed, scales, group).astype(np.float64)
    return np.asarray(x, dtype=np.float64) @ w.T
