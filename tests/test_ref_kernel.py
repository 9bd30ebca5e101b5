"""The north star's error bar: on every config-1 and config-2 case, this library's normalized error against the fp64
oracle is no worse than the reference kernel's own -- the reference's csrc/w4_gemv.cu built unchanged for sm_100a
into oracle/_ref/ (oracle/ref_kernel.py), run on the same quantized weights and activations. The reference applies
the same comparison to each of its kernels (bench/gpu_run.py:231-245). Skipped where oracle/_ref was never built.

Up to 16 rows the kernels multiply exact integer fragments and scale each 128-wide chunk in fp32 (the weight is
never rounded), and the bar is strict. From 17 rows the tcgen05 GEMM multiplies the fp16-rounded weights
fp16(q * s) -- exactly the operands of the reference's gemm_v5 and of cuBLAS on dequantize()'s output -- with fp32
accumulation in another order; such results differ from each other only where a value rounds to the other fp16
neighbour, so the bar there is the reference's error plus half an fp16 ulp of the largest output."""
import numpy as np
import pytest
import torch

from lowbit import ops, quant
from oracle import oracle as O
from oracle import ref_kernel

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_kernel.available(), reason="oracle/_ref (the reference kernels) not built")]

# the config-1 projection shapes (K, N) and the reference's tail shapes (bench/gpu_run.py:24-31)
SHAPES = [(896, 896), (896, 128), (896, 4864), (4864, 896), (1536, 1536), (1536, 256), (1536, 8960), (8960, 1536),
          (2048, 2048), (2048, 256), (2048, 11008), (11008, 2048), (128, 1), (256, 1001), (384, 37)]
ROWS = [1, 2, 4, 8, 16, 32, 48, 64]


@pytest.fixture(scope="module")
def ref():
    return ref_kernel.load()


def norm_err(y, y64):
    return float(np.abs(y.double().cpu().numpy() - y64).max() / np.sqrt(np.mean(y64 ** 2)))


@pytest.mark.parametrize("k,n", SHAPES)
def test_no_worse_than_the_reference_kernel(ref, k, n):
    g = torch.Generator().manual_seed(k * 13 + n)
    w = (torch.randn(n, k, generator=g) * 0.02).numpy()
    packed, scales = quant.quantize_w4(w, 128)
    wq = ops.W4Weight(packed, scales, 128, ("mma",))
    w64 = O.c_dequantize_f32(packed, scales, 128).astype(np.float64)
    for m in ROWS:
        x = torch.randn(m, k, generator=g).half()
        y64 = x.double().numpy() @ w64.T
        xc = x.cuda()
        # the reference's decode kernel where it runs (v6: up to 8 rows), its tensor-core kernel (v5) everywhere
        ref_errs = [norm_err(ref.w4_gemm_tc(xc, wq.packed_mma, wq.scales, 128, 0), y64)]
        if m <= 8:
            ref_errs.append(norm_err(ref.w4_gemv(xc, wq.packed_mma, wq.scales, 128, 6, 0), y64))
        bar = min(ref_errs)
        ours = {"linear": norm_err(ops.linear(xc, wq), y64), "v5": norm_err(ops.gemv(xc, wq, 5), y64)}
        if m <= 8:
            ours["v6"] = norm_err(ops.gemv(xc, wq, 6), y64)
        rms = float(np.sqrt(np.mean(y64 ** 2)))
        flip = 0.5 * float(np.spacing(np.float16(np.abs(y64).max()))) / rms   # one output rounding the other way
        for path, e in ours.items():
            assert e <= 3e-3, (k, n, m, path, e)
            allowed = bar if m <= 16 else bar + flip
            assert e <= allowed, f"K={k} N={n} M={m} {path}: {e:.3e} > reference {bar:.3e} ({ref_errs}) + {allowed - bar:.1e}"
