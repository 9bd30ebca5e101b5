"""Regenerate the golden vectors in this folder from the reference's own Python code.

    python tests/golden/make_golden.py /path/to/lowbit-kernels     # writes tests/golden/format_vectors.npz

Run only where the reference checkout exists; the tests read the committed .npz and never the reference. It
imports the reference's lowbit.quant (numpy golden model, lowbit/quant.py) and lowbit.ops.dequantize_w4_gpu
(lowbit/ops.py:119-123, which runs on CPU tensors), feeds them seeded inputs, and stores inputs and outputs.
"""
import pathlib
import sys

import numpy as np

OUT = pathlib.Path(__file__).resolve().parent / "format_vectors.npz"

# (tag, N, K, G): the group sizes the reference's dispatch matrix covers (bench/gpu_run.py:167-168) and the
# shapes of its unit tests (tests/test_quant.py), all small enough for a CPU oracle
CASES = [("a", 8, 256, 128), ("b", 5, 384, 128), ("c", 4, 96, 32), ("d", 3, 320, 64), ("e", 6, 512, 256),
         ("f", 16, 1024, 128)]


def special_weights(rng):
    """Rows that stress the rounding rules: exact half steps (round half to even), an all-zero group, huge and
    tiny magnitudes (fp16 scale overflow / subnormal scale), mixed signs at the clip boundary."""
    k = 256
    w = rng.standard_normal((8, k)).astype(np.float32)
    w[0, :128] = 0.0
    w[1, :128] = np.linspace(-7.0, 7.0, 128, dtype=np.float32)          # scale 1, many exact integers
    w[1, 128:] = (np.arange(128, dtype=np.float32) - 64) * 0.5           # half steps: ties to even
    w[2] *= 1e-6                                                         # subnormal fp16 scales
    w[3] *= 1e4                                                          # large scales
    w[4, :] = -8.0                                                       # clip at -8 after rint(-8/(8/7))
    w[4, 0] = 8.0
    w[5, ::2] = 3.5
    w[5, 1::2] = -3.5
    w[6] = np.float32(1e-30) * rng.standard_normal(k).astype(np.float32)  # scale rounds to zero -> 1.0
    return w


def main(ref_root):
    sys.path.insert(0, str(ref_root))
    from lowbit import quant  # the reference's golden model
    import torch
    from lowbit import ops

    rng = np.random.default_rng(20261201)
    out = {}
    cases = [(tag, rng.standard_normal((n, k)).astype(np.float32) * 0.02, g) for tag, n, k, g in CASES]
    cases.append(("s", special_weights(rng), 128))
    for tag, w, g in cases:
        packed, scales = quant.quantize_w4(w, g)
        x16 = rng.standard_normal((3, w.shape[1])).astype(np.float16)
        out[f"{tag}_w"] = w
        out[f"{tag}_group"] = np.int64(g)
        out[f"{tag}_packed"] = packed
        out[f"{tag}_scales"] = scales
        out[f"{tag}_v3"] = quant.interleave_for_gpu(packed)
        if w.shape[1] % 128 == 0:
            out[f"{tag}_mma"] = quant.interleave_for_mma(packed)
        out[f"{tag}_deq32"] = quant.dequantize_w4(packed, scales, g)
        out[f"{tag}_deq16"] = ops.dequantize_w4_gpu(torch.from_numpy(packed), torch.from_numpy(scales), g).numpy()
        out[f"{tag}_x16"] = x16
        out[f"{tag}_y64"] = quant.gemv_reference(x16.astype(np.float64), packed, scales, g)
    # bench/gpu_run.py:144-159 known answer: q = 7 (nibble 15), scale 2^-10, one group of 128
    packed = np.full((16, 64), 0xFF, np.uint8)
    scales = np.full((16, 1), 2.0 ** -10, np.float16)
    for xv in (4096.0, -8192.0):
        out[f"overflow_{int(xv)}_y64"] = quant.gemv_reference(np.full((1, 128), xv), packed, scales, 128)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the reference checkout>")
    main(pathlib.Path(sys.argv[1]))
