"""GPU parity of every kernel against the CPU oracle on the same seeded inputs (B200 only: -m gpu).

Bars (from the reference's gates, bench/gpu_run.py:201-247, and the build's own contract):
  * dequantize, quantize and repack: bit-exact against the oracle / the golden model;
  * mma.sync GEMV / GEMM (up to 16 rows): normalized error max|y - y64| / RMS(y64) <= 3e-3 against the fp64
    oracle, and every output within 1 fp16 ulp of the correctly rounded fp64 result (the kernels accumulate
    exact products in fp32 per 128-wide chunk, so only the final rounding to fp16 remains), which is tighter
    than the reference kernels' own error (fp16 partial sums);
  * tcgen05 GEMM (17-64 rows): the same 3e-3 gate, and no worse than cuBLAS on the same fp16-dequantized
    weights (check_gemm_output);
  * the overflow known answer exactly (bench/gpu_run.py:144-159).
"""
import numpy as np
import pytest
import torch

from lowbit import model, ops, quant
from oracle import oracle as O

pytestmark = pytest.mark.gpu

# (name, K, N): the Qwen2.5 projection shapes of the benchmark configs, plus tails (bench/gpu_run.py:24-31)
SHAPES = [("0.5b.q", 896, 896), ("0.5b.kv", 896, 128), ("0.5b.up", 896, 4864), ("0.5b.down", 4864, 896),
          ("1.5b.q", 1536, 1536), ("1.5b.kv", 1536, 256), ("1.5b.up", 1536, 8960), ("1.5b.down", 8960, 1536),
          ("3b.q", 2048, 2048), ("3b.kv", 2048, 256), ("3b.up", 2048, 11008), ("3b.down", 11008, 2048)]
EDGE = [("tiny", 128, 1), ("odd_n", 256, 1001), ("odd_n2", 384, 37), ("k128", 128, 37)]
NORM_BOUND = 3e-3


def seeded(n, k, seed, scale=0.02):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * scale).numpy()


def x_for(m, k, seed):
    g = torch.Generator().manual_seed(seed + 17)
    return torch.randn(m, k, generator=g).half()


def ref_y(x16_cpu, packed, scales, group):
    """fp64 reference: x @ (q * scale)^T (lowbit/quant.py:81-84), dequantized by the C oracle."""
    w = O.c_dequantize_f32(packed, scales, group).astype(np.float64)
    return x16_cpu.double().numpy() @ w.T


def check_output(y_gpu, y64, what):
    y = y_gpu.double().cpu().numpy()
    rms = np.sqrt(np.mean(y64 ** 2))
    err = np.abs(y - y64).max() / rms
    assert np.isfinite(y).all(), what
    assert err <= NORM_BOUND, f"{what}: normalized error {err:.3e}"
    # within one fp16 ulp of the correctly rounded result, plus an fp32-accumulation allowance of 2e-5 RMS
    # (50x finer than fp16's own resolution at RMS magnitude) for outputs that sit close to zero
    want = torch.from_numpy(y64).half().double().numpy()
    ulp = np.spacing(np.abs(want).astype(np.float16)).astype(np.float64)
    tol = ulp * 1.0001 + 2e-5 * rms
    assert np.all(np.abs(y - want) <= tol), f"{what}: worst {np.max(np.abs(y - want) / ulp):.2f} ulp"
    return err


@pytest.fixture(scope="module")
def layers():
    out = {}
    for name, k, n in SHAPES + EDGE:
        w = seeded(n, k, k * 7 + n)
        packed, scales = quant.quantize_w4(w, 128)
        out[name] = (k, n, w, packed, scales, ops.W4Weight(packed, scales, 128))
    return out


def test_library_loads_and_reports_b200():
    e = ops.ext()
    assert torch.cuda.get_device_capability() == (10, 0)
    assert e.lib.lb_abi_version() >= 1


# ---------------------------------------------------------------- format kernels: bit-exact

@pytest.mark.parametrize("name", [s[0] for s in SHAPES + EDGE])
def test_repack_matches_golden_model(layers, name):
    k, n, w, packed, scales, wq = layers[name]
    assert np.array_equal(wq.packed.cpu().numpy(), packed)
    assert np.array_equal(wq.packed_v3.cpu().numpy(), quant.interleave_for_gpu(packed))
    assert np.array_equal(wq.packed_mma.cpu().numpy(), quant.interleave_for_mma(packed))


@pytest.mark.parametrize("name", [s[0] for s in SHAPES + EDGE])
def test_dequant_bit_exact_every_layout(layers, name):
    k, n, w, packed, scales, wq = layers[name]
    want = O.c_dequantize_f16(packed, scales, 128).view(np.uint16)
    for layout in ("canonical", "v3", "mma"):
        got = ops.ext().w4_dequant(getattr(wq, {"canonical": "packed", "v3": "packed_v3", "mma": "packed_mma"}[layout]),
                                   wq.scales, 128, layout=layout)
        assert np.array_equal(got.cpu().numpy().view(np.uint16), want), layout
    assert torch.equal(ops.dequant(wq, "mma"), ops.dequant(wq, "canonical"))


@pytest.mark.parametrize("group", [32, 64, 128, 256])
def test_dequant_other_group_sizes(group):
    k, n = 512, 200
    w = seeded(n, k, group)
    packed, scales = quant.quantize_w4(w, group)
    got = ops.dequantize_w4_gpu(torch.from_numpy(packed).cuda(), torch.from_numpy(scales).cuda(), group)
    assert np.array_equal(got.cpu().numpy().view(np.uint16), O.c_dequantize_f16(packed, scales, group).view(np.uint16))


@pytest.mark.parametrize("name", ["0.5b.q", "1.5b.up", "3b.down", "odd_n", "tiny"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_gpu_quantizer_bit_exact(layers, name, dtype):
    k, n, w, packed, scales, wq = layers[name]
    wt = torch.from_numpy(w).to(dtype)
    p, s = ops.quantize_w4_gpu(wt.cuda(), 128)
    want_p, want_s = quant.quantize_w4(wt.float().numpy(), 128)
    assert np.array_equal(p.cpu().numpy(), want_p)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), want_s.view(np.uint16))


def test_gpu_quantizer_golden_special_rows(golden):
    for t in ("s", "c", "d", "e"):
        w, g = golden[f"{t}_w"], int(golden[f"{t}_group"])
        p, s = ops.quantize_w4_gpu(torch.from_numpy(w).cuda(), g)
        assert np.array_equal(p.cpu().numpy(), golden[f"{t}_packed"]), t
        assert np.array_equal(s.cpu().numpy().view(np.uint16), golden[f"{t}_scales"].view(np.uint16)), t


def test_gpu_quantizer_clip_grid_picks_a_best_candidate():
    """With a clip grid the chosen scale of every group must be a candidate whose squared error is the smallest
    (up to fp32 summation order), and the bits must be that candidate's quantization."""
    grid = tuple(round(1.0 - 0.025 * i, 3) for i in range(11))
    w = seeded(64, 512, 5, scale=1.0)
    w[3, :128] *= 50   # an outlier group, where clipping pays
    p, s = ops.quantize_w4_gpu(torch.from_numpy(w).cuda(), 128, grid)
    p, s = p.cpu().numpy(), s.cpu().numpy()
    g = w.reshape(64, 4, 128)
    amax = np.abs(g).max(-1)
    errs, cands = [], []
    for a in grid:
        sc = ((amax * np.float32(a) if a != 1.0 else amax) / np.float32(7)).astype(np.float16)
        sc[sc == 0] = 1
        q = np.clip(np.rint(g / sc.astype(np.float32)[..., None]), -8, 7)
        errs.append(((q * sc.astype(np.float32)[..., None] - g) ** 2).sum(-1))
        cands.append(sc)
    errs, cands = np.stack(errs), np.stack(cands)
    chosen = np.argmax(cands.view(np.uint16) == s.view(np.uint16)[None], axis=0)
    assert np.all((cands.view(np.uint16) == s.view(np.uint16)[None]).any(0))
    assert np.all(errs[chosen, np.arange(64)[:, None], np.arange(4)[None]] <= errs.min(0) * (1 + 1e-5) + 1e-12)
    # the packed bits are the chosen scale's quantization
    q = np.clip(np.rint(g / s.astype(np.float32)[..., None]), -8, 7).astype(np.int16).reshape(64, 512) + 8
    assert np.array_equal(p, (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8))


# ---------------------------------------------------------------- GEMV / GEMM numerics

@pytest.mark.parametrize("name", [s[0] for s in SHAPES + EDGE])
@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
def test_v6_gemv_parity(layers, name, m):
    k, n, w, packed, scales, wq = layers[name]
    x = x_for(m, k, k + n + m)
    y = ops.gemv(x.cuda(), wq, 6)
    check_output(y, ref_y(x, packed, scales, 128), f"v6 {name} M={m}")


@pytest.mark.parametrize("kernel", [0, 2, 3, 4, 5])
@pytest.mark.parametrize("name", ["0.5b.kv", "1.5b.up", "3b.down", "odd_n", "tiny", "k128"])
@pytest.mark.parametrize("m", [1, 3, 7, 8, 16, 24])
def test_every_gemv_kernel(layers, kernel, name, m):
    """Each kernel forced through the option against the oracle, whatever the dispatch would pick: automatic (0),
    the tcgen05 GEMM (2), the one-shot GEMV with CTA-wide staging (3), the bulk-copy GEMV (4; 3 and 4 up to 8 rows,
    the automatic choice beyond) and the skinny mma.sync GEMM (5; exact per-group products up to 16 rows)."""
    k, n, w, packed, scales, wq = layers[name]
    x = x_for(m, k, k + n + 5 * m)
    e = ops.ext()
    prev = e.set_option("gemv_kernel", kernel)
    try:
        y = ops.gemv(x.cuda(), wq, 6 if m <= 8 else 5)
    finally:
        e.set_option("gemv_kernel", prev)
    y64 = ref_y(x, packed, scales, 128)
    if kernel == 2 or m > 16:   # above 16 rows every path multiplies fp16-rounded weights
        check_gemm_output(y, y64, x, packed, scales, 128, f"kernel {kernel} {name} M={m}")
    else:
        check_output(y, y64, f"kernel {kernel} {name} M={m}")


def check_gemm_output(y_gpu, y64, x16, packed, scales, group, what):
    """The tcgen05 GEMM multiplies by fp16_rn(q * scale) -- the dequantized weights -- and accumulates a whole
    row of K in the tensor core's fp32 accumulator, exactly the arithmetic of cuBLAS on dequantize()'s output
    (the path it replaces). Bars: normalized error <= 3e-3 against fp64, and against the fp64 product with the
    same fp16 weights, a max error at most 2x and a mean error at most 1.5x those of cuBLAS on the same inputs."""
    y = y_gpu.double().cpu().numpy()
    rms = np.sqrt(np.mean(y64 ** 2))
    assert np.isfinite(y).all(), what
    err = np.abs(y - y64).max() / rms
    assert err <= NORM_BOUND, f"{what}: normalized error {err:.3e}"
    w16 = O.c_dequantize_f16(packed, scales, group)
    y16w = x16.double().numpy() @ w16.astype(np.float64).T
    yc = torch.nn.functional.linear(x16.cuda(), torch.from_numpy(w16).cuda()).double().cpu().numpy()
    e_ours, e_cublas = np.abs(y - y16w), np.abs(yc - y16w)
    assert e_ours.max() <= 2 * e_cublas.max(), f"{what}: max error {e_ours.max():.3e} vs cuBLAS {e_cublas.max():.3e}"
    assert e_ours.mean() <= 1.5 * e_cublas.mean(), \
        f"{what}: mean error {e_ours.mean():.3e} vs cuBLAS {e_cublas.mean():.3e}"


@pytest.mark.parametrize("name", [s[0] for s in SHAPES + EDGE])
@pytest.mark.parametrize("m", [1, 17, 24, 32, 33, 48, 64])
def test_tcgen05_gemm_parity(layers, name, m):
    """The tcgen05 kernel at every NB (32 / 48 / 64), forced for M < 17 too."""
    k, n, w, packed, scales, wq = layers[name]
    x = x_for(m, k, k + n + 3 * m)
    e = ops.ext()
    prev = e.set_option("gemv_kernel", 2)
    try:
        y = ops.gemv(x.cuda(), wq, 5)
    finally:
        e.set_option("gemv_kernel", prev)
    check_gemm_output(y, ref_y(x, packed, scales, 128), x, packed, scales, 128, f"tcgen05 {name} M={m}")


@pytest.mark.parametrize("name", [s[0] for s in SHAPES + EDGE])
@pytest.mark.parametrize("m", [1, 9, 16, 17, 24, 32, 33, 40, 48, 49, 64])
def test_mma_gemm_parity(layers, name, m):
    """The skinny mma.sync GEMM at every activation-tile width (16 / 32 / 48 / 64 rows), forced at every M: exact
    per-group products up to 16 rows (the GEMV's bar), fp16-rounded weights above (the cuBLAS bar)."""
    k, n, w, packed, scales, wq = layers[name]
    x = x_for(m, k, k + n + 11 * m)
    e = ops.ext()
    prev = e.set_option("gemv_kernel", 5)
    try:
        y = ops.gemv(x.cuda(), wq, 5)
    finally:
        e.set_option("gemv_kernel", prev)
    y64 = ref_y(x, packed, scales, 128)
    if m > 16:
        check_gemm_output(y, y64, x, packed, scales, 128, f"mma gemm {name} M={m}")
    else:
        check_output(y, y64, f"mma gemm {name} M={m}")


@pytest.mark.parametrize("ksplit", [1, 2, 3, 7, 8])
@pytest.mark.parametrize("rt", [1, 2])
@pytest.mark.parametrize("m", [12, 40])
def test_mma_gemm_forced_splits_and_row_tiles(ksplit, rt, m):
    """Every cluster size and row-tile count of the skinny GEMM gives the same result within its bar (the split
    only changes the fp32 summation order)."""
    e = ops.ext()
    k, n = 4864, 1000
    packed, scales = quant.quantize_w4(seeded(n, k, 5), 128)
    wq = ops.W4Weight(packed, scales, 128, ("mma",))
    x = x_for(m, k, 5)
    prev = {o: e.set_option(o, v) for o, v in (("gemv_kernel", 5), ("gemv_ksplit", ksplit), ("gemv_rowtiles", rt))}
    try:
        y = ops.gemv(x.cuda(), wq, 5)
    finally:
        for o, v in prev.items():
            e.set_option(o, v)
    y64 = ref_y(x, packed, scales, 128)
    if m > 16:
        check_gemm_output(y, y64, x, packed, scales, 128, f"ksplit={ksplit} rt={rt} M={m}")
    else:
        check_output(y, y64, f"ksplit={ksplit} rt={rt} M={m}")


@pytest.mark.parametrize("m", [1, 8, 12, 16, 40])
def test_long_k_every_row_count(m):
    """K = 24576 (192 chunks): the decode GEMV's staged activations stop fitting shared memory as M grows, and the
    dispatch falls through to the skinny GEMM, whose shared memory does not grow with K."""
    k, n = 24576, 320
    packed, scales = quant.quantize_w4(seeded(n, k, 13), 128)
    wq = ops.W4Weight(packed, scales, 128, ("mma",))
    x = x_for(m, k, 13 + m)
    y = ops.gemv(x.cuda(), wq, 6 if m <= 8 else 5)
    y64 = ref_y(x, packed, scales, 128)
    if m > 16:
        check_gemm_output(y, y64, x, packed, scales, 128, f"long K M={m}")
    else:
        check_output(y, y64, f"long K M={m}")


def test_mma_gemm_group_256_and_bias(layers):
    """Two chunks per scale group, and the bias epilogue, through the skinny GEMM."""
    k, n = 2048, 768
    w = seeded(n, k, 9)
    packed, scales = quant.quantize_w4(w, 256)
    wq = ops.W4Weight(packed, scales, 256, ("mma",))
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(4)) * 0.1).half()
    for m in (12, 37, 64):
        x = x_for(m, k, 21 + m)
        y64 = ref_y(x, packed, scales, 256)
        e = ops.ext()
        prev = e.set_option("gemv_kernel", 5)
        try:
            y = ops.gemv(x.cuda(), wq, 5)
            yb = ops.gemv(x.cuda(), wq, 5, bias=bias.cuda())
        finally:
            e.set_option("gemv_kernel", prev)
        if m > 16:
            check_gemm_output(y, y64, x, packed, scales, 256, f"G=256 M={m}")
        else:
            check_output(y, y64, f"G=256 M={m}")
        want = (y.float() + bias.cuda().float()).half()
        assert torch.equal(yb, want), f"bias M={m}"


@pytest.mark.parametrize("name", [s[0] for s in SHAPES + EDGE])
@pytest.mark.parametrize("m", [1, 4, 12, 16, 33, 48, 64])
def test_v5_gemm_parity(layers, name, m):
    k, n, w, packed, scales, wq = layers[name]
    x = x_for(m, k, k + n + m + 1)
    y = ops.gemv(x.cuda(), wq, 5)
    if m > 16:
        check_gemm_output(y, ref_y(x, packed, scales, 128), x, packed, scales, 128, f"v5 {name} M={m}")
    else:
        check_output(y, ref_y(x, packed, scales, 128), f"v5 {name} M={m}")


@pytest.mark.parametrize("version", [1, 2, 3, 4])
@pytest.mark.parametrize("group", [32, 64, 128, 256])
@pytest.mark.parametrize("m", [1, 3, 8])
def test_compat_versions(version, group, m):
    k, n = 512, 300
    w = seeded(n, k, version * 100 + group)
    packed, scales = quant.quantize_w4(w, group)
    wq = ops.W4Weight(packed, scales, group, ("canonical", "v3"))
    x = x_for(m, k, group + m)
    for rpw in (0, 1, 2, 4):
        y = ops.gemv(x.cuda(), wq, version, rpw)
        check_output(y, ref_y(x, packed, scales, group), f"v{version} G={group} M={m} R={rpw}")


def test_overflow_known_answer():
    k = 128
    wq = ops.W4Weight(np.full((16, k // 2), 0xFF, np.uint8), np.full((16, 1), 2.0 ** -10, np.float16), k)
    for xv, want in ((4096.0, 3584.0), (-8192.0, -7168.0)):
        x = torch.full((1, k), xv, dtype=torch.half, device="cuda")
        for v in (1, 2, 3, 4, 5, 6):
            y = ops.gemv(x, wq, v).float()
            assert torch.all(y == want), (v, xv, y[0, :4])


def test_large_activations_stay_finite():
    """|x| near the fp16 limit with real weights: products and sums live in fp32, so nothing overflows until the
    fp16 output itself would."""
    k, n = 1024, 256
    packed, scales = quant.quantize_w4(seeded(n, k, 9), 128)
    wq = ops.W4Weight(packed, scales, 128)
    x = (x_for(4, k, 9).float() * 3000).clamp(-60000, 60000).half()
    y64 = ref_y(x, packed, scales, 128)
    assert np.abs(y64).max() < 60000
    for v in (5, 6):
        check_output(ops.gemv(x.cuda(), wq, v), y64, f"v{v} large x")


# ---------------------------------------------------------------- API behaviour (reference gates)

def test_dispatch_matrix():
    """linear() across the dispatch boundaries on the copies a model keeps, G = 32/64/256 (bench/gpu_run.py:162-198)."""
    cases = [("mma_only_g128", 1024, 3072, 128, ("mma",)), ("mma_only_narrow", 1536, 1000, 128, ("mma",)),
             ("canonical_g32", 96, 200, 32, None), ("canonical_g64", 320, 130, 64, None),
             ("mma_g256", 512, 4096, 256, ("mma",))]
    for name, k, n, g, layouts in cases:
        w = seeded(n, k, k + n + g, scale=1.0)
        packed, scales = quant.quantize_w4(w, g)
        wq = ops.W4Weight(packed, scales, g, layouts)
        for m in (1, 2, 8, 9, 17, 31, 32, 33, 63, 64, 65, 130):
            x = x_for(m, k, m + g)
            y = ops.linear(x.cuda(), wq)
            y64 = ref_y(x, packed, scales, g)
            err = np.abs(y.double().cpu().numpy() - y64).max() / np.sqrt(np.mean(y64 ** 2))
            assert err <= NORM_BOUND, (name, m, err)


def test_linear_out_writes_in_place_with_the_same_bits():
    """out= (used by the end-to-end benchmark): the result lands in the given slice of a larger buffer, bit-equal to
    the allocating call, for the INT4 kernels and the dequantize + cuBLAS path; a wrong buffer is refused."""
    wq = ops.W4Weight.from_float(torch.randn(1000, 1536))
    buf = torch.full((3000,), float("nan"), device="cuda").half()
    for m in (1, 3, 20, 70):
        x = torch.randn(m, 1536).half().cuda()
        out = torch.empty(m, 1000, device="cuda").half() if m > 1 else buf[1000:2000].view(1, 1000)
        assert ops.linear(x, wq, out=out) is out
        assert torch.equal(out, ops.linear(x, wq))
    assert torch.isnan(buf[:1000].float()).all() and torch.isnan(buf[2000:].float()).all()
    with pytest.raises(RuntimeError):
        ops.linear(torch.randn(1, 1536).half().cuda(), wq, out=torch.empty(1, 999, device="cuda").half())


def test_cached_launch_path_matches_the_checked_path():
    """ops.gemv's cached-argument path (versions 5 and 6) gives the bits of the fully checked call; unusual inputs
    (a strided x) take the checked path; replacing a layout tensor revalidates the cache."""
    e = ops.ext()
    wq = ops.W4Weight.from_float(torch.randn(2048, 1536))
    for m, v in ((1, 6), (4, 6), (24, 5)):
        x = torch.randn(m, 1536).half().cuda()
        if v == 6:
            want = e.w4_gemv(x, wq.packed_mma, wq.scales, wq.group, 6)
        else:
            want = e.w4_gemm_tc(x, wq.packed_mma, wq.scales, wq.group)
        assert torch.equal(ops.gemv(x, wq, v), want)
        assert wq.launch_args(v) is not None
        out = torch.empty(m, 2048, device="cuda").half()
        assert ops.gemv(x, wq, v, out=out) is out and torch.equal(out, want)
    xs = torch.randn(1536, 2).half().cuda().t()[:1]            # not contiguous
    assert torch.equal(ops.gemv(xs, wq, 6), e.w4_gemv(xs.contiguous(), wq.packed_mma, wq.scales, wq.group, 6))
    x = torch.randn(1, 1536).half().cuda()
    before = ops.gemv(x, wq, 6)
    wq.packed_mma = wq.packed_mma.clone()
    assert torch.equal(ops.gemv(x, wq, 6), before)
    assert wq.launch_args(6)[0] == wq.packed_mma.data_ptr()


def test_fixed_version_past_its_limit_falls_back():
    wq = ops.W4Weight.from_float(torch.randn(256, 512))
    x = torch.randn(9, 512).half().cuda()
    assert torch.isfinite(ops.linear(x, wq, max_gemv_rows=16, version=6)).all()


def test_side_stream_gives_the_same_bits():
    wq = ops.W4Weight.from_float(torch.randn(1000, 1536))
    x = torch.randn(3, 1536).half().cuda()
    want = [ops.linear(x[:m], wq) for m in (1, 3)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        got = [ops.linear(x[:m], wq) for m in (1, 3)]
    s.synchronize()
    for a, b in zip(want, got):
        assert torch.equal(a, b)


def test_refusals():
    wq = ops.W4Weight.from_float(torch.randn(256, 512), layouts=None)
    x = torch.randn(9, 512).half().cuda()
    with pytest.raises(RuntimeError):
        ops.ext().w4_dequant(wq.packed, wq.scales.cpu(), 128)            # CPU scales
    with pytest.raises(RuntimeError):
        ops.ext().w4_gemv(x[:1], wq.packed, wq.scales, 0, 1, 0)          # group 0
    with pytest.raises(RuntimeError):
        ops.ext().w4_gemv(x, wq.packed, wq.scales, 128, 1, 0)            # 9 rows into a GEMV
    with pytest.raises(RuntimeError):
        ops.ext().w4_gemv(x[:1].float(), wq.packed, wq.scales, 128, 6, 0)
    with pytest.raises(RuntimeError):
        ops.ext().w4_gemm_tc(torch.randn(65, 512).half().cuda(), wq.packed_mma, wq.scales, 128)
    with pytest.raises(RuntimeError):
        ops.dequantize_w4_gpu(wq.packed.cpu(), wq.scales.cpu())


def test_cuda_graph_capture_and_pdl_options_give_identical_bits():
    e = ops.ext()
    wqs = [ops.W4Weight.from_float(torch.randn(n, k), layouts=("mma",)) for k, n in ((2048, 11008), (11008, 2048),
                                                                                       (896, 128))]
    rows = (1, 16, 40)   # one-shot GEMV, one-shot GEMM, tcgen05 GEMM
    xs = [torch.randn(m, wq.k).half().cuda() for wq in wqs for m in rows]
    pairs = [(x, wq) for x, wq in zip(xs, [w for w in wqs for _ in rows])]
    eager = [ops.linear(x, wq) for x, wq in pairs]
    prev = {k: e.get_option(k) for k in ("pdl", "early_weights")}
    try:
        for pdl, early in ((0, 0), (1, 0), (1, 1)):
            e.set_option("pdl", pdl)
            e.set_option("early_weights", early)
            assert all(torch.equal(ops.linear(x, wq), y) for (x, wq), y in zip(pairs, eager))
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                [ops.linear(x, wq) for x, wq in pairs]
            torch.cuda.current_stream().wait_stream(s)
            with torch.cuda.graph(g):
                outs = [ops.linear(x, wq) for x, wq in pairs]
            g.replay()
            torch.cuda.synchronize()
            assert all(torch.equal(a, b) for a, b in zip(outs, eager)), (pdl, early)
    finally:
        for k, v in prev.items():
            e.set_option(k, v)


@pytest.mark.parametrize("ksplit", [1, 2, 3, 5, 8])
def test_forced_k_splits_agree(ksplit):
    e = ops.ext()
    packed, scales = quant.quantize_w4(seeded(512, 4864, 3), 128)
    wq = ops.W4Weight(packed, scales, 128, ("mma",))
    x = x_for(4, 4864, 3)
    prev = e.set_option("gemv_ksplit", ksplit)
    try:
        y = ops.gemv(x.cuda(), wq, 6)
    finally:
        e.set_option("gemv_ksplit", prev)
    check_output(y, ref_y(x, packed, scales, 128), f"ksplit={ksplit}")


# ---------------------------------------------------------------- model integration

def test_w4linear_matches_fake_quant_linear():
    torch.manual_seed(0)
    lin = torch.nn.Linear(1536, 1000, bias=True).half().cuda()
    seq = torch.nn.Sequential()
    seq.add_module("up_proj", lin)
    layers = model.quantize_layers(seq)
    assert len(layers) == 1
    _, _, _, packed, scales = layers[0]
    fake = torch.nn.Linear(1536, 1000, bias=True).half().cuda()
    fake.load_state_dict(lin.state_dict())
    model.apply_fake_quant([(None, None, fake, packed, scales)])
    count, nbytes = model.apply_int4(layers)
    assert count == 1 and nbytes == 1000 * 768 + 1000 * 12 * 2
    w4 = seq.up_proj
    for shape in ((1, 1536), (2, 3, 1536), (40, 1536), (200, 1536)):
        x = torch.randn(*shape).half().cuda()
        y, yf = w4(x), fake(x)
        assert y.shape == (*shape[:-1], 1000)
        rel = ((y.float() - yf.float()).abs().max() / yf.float().pow(2).mean().sqrt()).item()
        assert rel < 5e-3, (shape, rel)


def test_no_kernel_wait_gave_up():
    """Every bounded wait in the kernels completed (the device error word is still zero)."""
    torch.cuda.synchronize()
    assert ops.ext().lib.lb_device_error() == 0



# ---------------------------------------------------------------- bias in the epilogue (lb_w4_linear)

@pytest.mark.parametrize("name", ["1.5b.q", "3b.down", "odd_n", "tiny"])
@pytest.mark.parametrize("m", [1, 3, 8, 16, 24, 64])
def test_bias_epilogue_matches_separate_add_and_fp64(layers, name, m):
    """ops.gemv / ops.linear with bias=: bit-identical to the kernel's fp16 output plus the fp16 bias (the
    reference's W4Linear.forward, lowbit/model.py:22-27), and within the GEMV bar of the fp64 product plus bias."""
    k, n, w, packed, scales, wq = layers[name]
    g = torch.Generator().manual_seed(n + m)
    bias = (torch.randn(n, generator=g) * 0.5).half()
    x = x_for(m, k, k + 7 * m)
    xc, bc = x.cuda(), bias.cuda()
    y64 = ref_y(x, packed, scales, 128) + bias.double().numpy()[None]
    versions = [5] + ([1, 2, 3, 4, 6] if m <= 8 else [])
    for v in versions:
        got = ops.gemv(xc, wq, v, bias=bc)
        assert torch.equal(got, ops.gemv(xc, wq, v) + bc), (name, m, v)
        rms = np.sqrt(np.mean(y64 ** 2))
        err = np.abs(got.double().cpu().numpy() - y64).max() / rms
        # the bias add rounds to fp16 once more: half an ulp at the largest output on top of the GEMV bar
        extra = 0.5 * float(np.spacing(np.float16(np.abs(y64).max()))) / rms
        assert err <= NORM_BOUND + extra, (name, m, v, err, extra)
    lin = ops.linear(xc, wq, bias=bc)
    assert torch.equal(lin, ops.linear(xc, wq) + bc)


def test_bias_on_the_prefill_path_and_refusals():
    wq = ops.W4Weight.from_float(torch.randn(300, 512))
    bias = torch.randn(300).half().cuda()
    x = torch.randn(130, 512).half().cuda()
    assert torch.equal(ops.linear(x, wq, bias=bias), ops.linear(x, wq) + bias)
    with pytest.raises(RuntimeError):
        ops.ext().w4_linear(x[:2], wq.packed_mma, wq.scales, 128, 6, bias=bias[:299].contiguous())
    with pytest.raises(RuntimeError):
        ops.ext().w4_linear(x[:2], wq.packed_mma, wq.scales, 128, 6, bias=bias.float())
