"""The decode harness (random-init Qwen2 decoder, INT4 projections, one CUDA graph per step) on a small config.

The INT4 model is compared with the fake-quant model -- the same quantized values as fp16 nn.Linear weights run
through cuBLAS (the split the reference's bench/e2e.py uses to isolate kernel error from quantization error).
"""
import pytest
import torch

from lowbit import decode, ops

pytestmark = pytest.mark.gpu

TINY = dict(hidden_size=256, intermediate_size=640, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, vocab_size=1024, tie_word_embeddings=True)


@torch.no_grad()
@pytest.mark.parametrize("fuse", [(), ("epilogue",)])
def test_int4_decoder_matches_fake_quant_and_replays_bit_exactly(fuse):
    decode.enable_decode_options()
    gen = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, TINY["vocab_size"], (24,), generator=gen)
    seq = torch.randint(0, TINY["vocab_size"], (12,), generator=gen).tolist()

    dec = decode.Int4Decoder(decode.build(TINY, seed=3), max_len=64, fuse=fuse)
    assert dec.int4_bytes > 0
    first = dec.prefill(prompt).float()
    got = dec.forced(seq)

    f = decode.to_fake_quant(decode.build(TINY, seed=3))
    full = torch.cat([prompt, torch.tensor(seq)]).view(1, -1).cuda()
    want = f(input_ids=full).logits[0].float()
    p = prompt.numel()
    want_first, want_rows = want[p - 1], want[p:]
    rms = want_rows.pow(2).mean().sqrt()
    err = (got - want_rows).abs().max() / rms
    assert err < 2e-2, f"normalized logit error {err:.3e}"
    assert ((first - want_first).abs().max() / rms) < 2e-2
    agree = (got.argmax(-1) == want_rows.argmax(-1)).float().mean().item()
    assert agree >= 0.9, agree

    # a graph replay is the eager step, bit for bit
    for run in ("graph", "eager"):
        dec.pos.fill_(p)
        dec.tok.fill_(seq[0])
        if run == "graph":
            dec.graph.replay()
            replay = dec.logits[0].clone()
        else:
            dec._step()
    assert torch.equal(dec.logits[0], replay)
    assert ops.ext().lib.lb_device_error() == 0


@torch.no_grad()
@pytest.mark.parametrize("fuse", [(), ("epilogue",)])
def test_greedy_continuation_is_the_argmax(fuse):
    """Free-running decode: each step's token is the argmax of that step's logits."""
    decode.enable_decode_options()
    dec = decode.Int4Decoder(decode.build(TINY, seed=5), max_len=48, fuse=fuse)
    dec.prefill(torch.arange(16) * 37 % TINY["vocab_size"])
    for _ in range(8):
        dec.step()
        assert dec.tok.item() == dec.logits[0].argmax().item()
    assert dec.pos.item() == 24


def _lib():
    return ops.ext().lib


@torch.no_grad()
def test_epilogue_decoder_matches_separate_kernels():
    """The epilogue-fused step computes the separate kernels' values; only the RMSNorms' sums of squares run in
    another order (an fp16 ulp of the normalized row), so logits agree closely and the launch count drops by 3 per
    layer."""
    decode.enable_decode_options()
    prompt = torch.arange(12) * 53 % TINY["vocab_size"]
    seq = (torch.arange(8) * 97 % TINY["vocab_size"]).tolist()
    plain = decode.Int4Decoder(decode.build(TINY, seed=7), max_len=32)
    fused = decode.Int4Decoder(decode.build(TINY, seed=7), max_len=32, fuse=("epilogue",))
    assert plain.launches_per_step() - fused.launches_per_step() == 3 * TINY["num_hidden_layers"]
    plain.prefill(prompt)
    fused.prefill(prompt)
    a, b = plain.forced(seq), fused.forced(seq)
    assert (a - b).abs().max() / a.pow(2).mean().sqrt() < 5e-3
    assert torch.equal(a.argmax(-1), b.argmax(-1))
    assert _lib().lb_device_error() == 0


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("H", [2048, 3584])
def test_rmsnorm_kernel(H):
    g = torch.Generator(device="cuda").manual_seed(H)
    x = torch.randn(H, device="cuda", generator=g).half()
    r = torch.randn(H, device="cuda", generator=g).half()
    w = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).half()
    want_x = x + r
    n = (want_x.float() * torch.rsqrt(want_x.float().pow(2).mean() + 1e-6)).half()
    want_h = w * n
    h = torch.empty_like(x)
    assert _lib().lb_decode_rmsnorm(x.data_ptr(), r.data_ptr(), w.data_ptr(), h.data_ptr(), H, 1e-6, _stream()) == 0
    assert torch.equal(x, want_x)      # the residual add is one fp16 rounding, as in torch
    # the fp32 sum of squares is summed in another order: allow one fp16 ulp
    ulp = torch.finfo(torch.half).eps * want_h.float().abs().clamp_min(2 ** -14)
    assert torch.all((h.float() - want_h.float()).abs() <= 2 * ulp)


def _rope(t, pos, inv_freq):
    """rotate-half RoPE (transformers apply_rotary_pos_emb), fp32."""
    ang = pos * inv_freq
    c, s = torch.cos(ang), torch.sin(ang)
    half = t.shape[-1] // 2
    a, b = t[..., :half], t[..., half:]
    return torch.cat([a * c - b * s, b * c + a * s], -1)


@pytest.mark.parametrize("pos", [0, 63, 64, 257, 3000])
# (16, 2, 128), (28, 4, 128), (4, 2, 64): tensor-core scores and P V; (32, 2, 128): 16 heads per kv head, the
# scalar loops at a compile-time head dim; (8, 2, 96): the generic path
@pytest.mark.parametrize("heads", [(16, 2, 128), (28, 4, 128), (4, 2, 64), (32, 2, 128), (8, 2, 96)])
def test_fused_attention_kernel(pos, heads):
    nh, nkv, hd = heads
    max_len = 320 if pos < 320 else 4096     # 3000: 47 splits hold cached rows, 17 are empty
    g = torch.Generator(device="cuda").manual_seed(pos + nh)
    qkv = torch.randn((nh + 2 * nkv) * hd, device="cuda", generator=g).half()
    bias = (0.1 * torch.randn((nh + 2 * nkv) * hd, device="cuda", generator=g)).half()
    kc = torch.randn(nkv, max_len, hd, device="cuda", generator=g).half()
    vc = torch.randn(nkv, max_len, hd, device="cuda", generator=g).half()
    kc0, vc0 = kc.clone(), vc.clone()
    inv_freq = (1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))).cuda()
    splits = _lib().lb_decode_attention_splits(max_len)
    part_o = torch.empty(nh * splits * hd, device="cuda")
    part_ml = torch.empty(nh * splits * 2, device="cuda")
    out = torch.empty(nh * hd, device="cuda").half()
    p = torch.tensor([pos], device="cuda")
    assert _lib().lb_decode_attention(qkv.data_ptr(), bias.data_ptr(), inv_freq.data_ptr(), p.data_ptr(),
                                      kc.data_ptr(), vc.data_ptr(), part_o.data_ptr(), part_ml.data_ptr(),
                                      out.data_ptr(), nh, nkv, hd, max_len, _stream()) == 0
    torch.cuda.synchronize()
    b = (qkv + bias).float().view(nh + 2 * nkv, hd)
    q = _rope(b[:nh], pos, inv_freq).half().float()
    k_new = _rope(b[nh:nh + nkv], pos, inv_freq).half()
    v_new = b[nh + nkv:].half()
    # the new row is appended, every other row untouched
    assert torch.allclose(kc[:, pos].float(), k_new.float(), atol=2e-3, rtol=2e-3)
    assert torch.equal(vc[:, pos], v_new)
    keep = torch.ones(max_len, dtype=torch.bool)
    keep[pos] = False
    assert torch.equal(kc[:, keep], kc0[:, keep]) and torch.equal(vc[:, keep], vc0[:, keep])
    K, V = kc[:, :pos + 1].float(), vc[:, :pos + 1].float()
    grp = nh // nkv
    Kx, Vx = K.repeat_interleave(grp, 0), V.repeat_interleave(grp, 0)
    att = torch.softmax((q[:, None, :] @ Kx.transpose(1, 2))[:, 0] / hd ** 0.5, -1)
    want = (att[:, None, :] @ Vx)[:, 0]
    assert torch.allclose(out.float().view(nh, hd), want, atol=3e-3, rtol=3e-3)


def test_attention_position_outside_the_cache_writes_nothing():
    """pos lives in device memory, so the host cannot check it: a pos >= max_len makes every CTA return before any
    read or write, and the status word reads 3."""
    lib, nh, nkv, hd, max_len = _lib(), 16, 2, 128, 128
    qkv = torch.randn((nh + 2 * nkv) * hd, device="cuda").half()
    kc, vc = torch.randn(nkv, max_len, hd, device="cuda").half(), torch.randn(nkv, max_len, hd, device="cuda").half()
    kc0, vc0 = kc.clone(), vc.clone()
    inv_freq = torch.ones(hd // 2, device="cuda")
    splits = lib.lb_decode_attention_splits(max_len)
    part_o, part_ml = torch.empty(nh * splits * hd, device="cuda"), torch.empty(nh * splits * 2, device="cuda")
    out = torch.zeros(nh * hd, device="cuda").half()
    lib.lb_clear_device_error()
    p = torch.tensor([max_len], device="cuda")
    assert lib.lb_decode_attention(qkv.data_ptr(), None, inv_freq.data_ptr(), p.data_ptr(), kc.data_ptr(),
                                   vc.data_ptr(), part_o.data_ptr(), part_ml.data_ptr(), out.data_ptr(), nh, nkv, hd,
                                   max_len, _stream()) == 0
    torch.cuda.synchronize()
    assert lib.lb_device_error() == 3
    assert torch.equal(kc, kc0) and torch.equal(vc, vc0)
    lib.lb_clear_device_error()
    assert lib.lb_device_error() == 0


def test_silu_mul_kernel():
    I = 11008
    g = torch.Generator(device="cuda").manual_seed(0)
    gu = (3 * torch.randn(2 * I, device="cuda", generator=g)).half()
    a = torch.empty(I, device="cuda").half()
    assert _lib().lb_decode_silu_mul(gu.data_ptr(), a.data_ptr(), I, _stream()) == 0
    want = torch.nn.functional.silu(gu[:I]) * gu[I:]
    assert torch.allclose(a.float(), want.float(), atol=1e-3, rtol=2e-3)


def _w4(n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return ops.W4Weight.from_float(torch.randn(n, k, device="cuda", generator=g) * 0.02, 128, ("mma",))


@pytest.mark.parametrize("nk", [(2560, 2048), (22016, 2048), (896, 896)])
@pytest.mark.parametrize("with_residual", [True, False])
def test_norm_gemv_matches_rmsnorm_then_gemv(nk, with_residual):
    n, k = nk
    wq = _w4(n, k, n + k)
    g = torch.Generator(device="cuda").manual_seed(k)
    x = torch.randn(k, device="cuda", generator=g).half()
    r = torch.randn(k, device="cuda", generator=g).half() if with_residual else None
    ln = (1 + 0.1 * torch.randn(k, device="cuda", generator=g)).half()
    x_out = torch.zeros_like(x)
    y = torch.empty(1, n, device="cuda").half()
    rc = _lib().lb_decode_norm_gemv(x.data_ptr(), None if r is None else r.data_ptr(), ln.data_ptr(),
                                    x_out.data_ptr() if with_residual else None, 1e-6, wq.packed_mma.data_ptr(),
                                    wq.scales.data_ptr(), y.data_ptr(), n, k, 128, _stream())
    assert rc == 0, _lib().lb_last_error()
    # the separate path: RMSNorm kernel (updates its own copy of x in place), then the GEMV
    xs, h = x.clone(), torch.empty_like(x)
    assert _lib().lb_decode_rmsnorm(xs.data_ptr(), None if r is None else r.data_ptr(), ln.data_ptr(), h.data_ptr(),
                                    k, 1e-6, _stream()) == 0
    want = ops.gemv(h.view(1, k), wq, 6)
    torch.cuda.synchronize()
    if with_residual:
        assert torch.equal(x_out, xs)          # x + r, one fp16 rounding
    # the sums of squares run in another order: normalized values may move by an fp16 ulp
    rms = want.float().pow(2).mean().sqrt()
    assert (y.float() - want.float()).abs().max() / rms < 2e-3


@pytest.mark.parametrize("nk", [(2048, 11008), (896, 4864)])
def test_swiglu_gemv_is_silu_mul_then_gemv(nk):
    n, k = nk
    wq = _w4(n, k, 7 * n + k)
    g = torch.Generator(device="cuda").manual_seed(n)
    gu = (2 * torch.randn(1, 2 * k, device="cuda", generator=g)).half()
    y = torch.empty(1, n, device="cuda").half()
    assert _lib().lb_decode_swiglu_gemv(gu.data_ptr(), wq.packed_mma.data_ptr(), wq.scales.data_ptr(), y.data_ptr(),
                                        n, k, 128, _stream()) == 0
    a = torch.empty(1, k, device="cuda").half()
    assert _lib().lb_decode_silu_mul(gu.data_ptr(), a.data_ptr(), k, _stream()) == 0
    want = ops.gemv(a, wq, 6)
    torch.cuda.synchronize()
    assert torch.equal(y, want)


def _ulp_close(a, b, ulps=1):
    """fp16 tensors equal up to `ulps` units in the last place of the larger magnitude (normalizations whose sums of
    squares run in another order)."""
    a, b = a.float(), b.float()
    ulp = torch.maximum(a.abs(), b.abs()).clamp_min(2.0 ** -14)
    ulp = torch.exp2(torch.floor(torch.log2(ulp)) - 10)
    return bool(((a - b).abs() <= ulps * ulp).all())


# (N, K, forced row tiles): 3B gate|up, a 0.5B-like gate|up, a K long enough for the cluster split-K path, two
# 16-row tiles per CTA
@pytest.mark.parametrize("nkr", [(22016, 2048, 0), (9728, 896, 0), (1024, 18944, 0), (4096, 2048, 2)])
def test_gemv_swiglu_epilogue_is_gemv_then_silu_mul(nkr):
    """lb_decode_gemv_swiglu on rows interleaving gate and up: bit-identical to the plain GEMV (lb_w4_gemv version
    6) followed by lb_decode_silu_mul on the de-interleaved [gate | up] row."""
    n, k, rt = nkr
    wq = _w4(n, k, 3 * n + k)
    g = torch.Generator(device="cuda").manual_seed(k)
    x = torch.randn(1, k, device="cuda", generator=g).half()
    e = ops.ext()
    prev = e.set_option("gemv_rowtiles", rt)
    try:
        y = ops.gemv(x, wq, 6)
        a = torch.full((n // 2,), float("nan"), device="cuda").half()
        rc = _lib().lb_decode_gemv_swiglu(x.data_ptr(), wq.packed_mma.data_ptr(), wq.scales.data_ptr(), a.data_ptr(),
                                          n, k, 128, _stream())
        assert rc == 0, _lib().lb_last_error()
    finally:
        e.set_option("gemv_rowtiles", prev)
    gu = torch.cat([y[0, 0::2], y[0, 1::2]]).contiguous()
    want = torch.empty(n // 2, device="cuda").half()
    assert _lib().lb_decode_silu_mul(gu.data_ptr(), want.data_ptr(), n // 2, _stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(a, want)


# (N, K): 3B o and down, 7B down on one GPU (K split over a cluster), 0.5B o
@pytest.mark.parametrize("nk", [(2048, 2048), (2048, 11008), (3584, 18944), (896, 896)])
def test_gemv_residual_norm_epilogue(nk):
    """lb_decode_gemv_residual_norm: y has the plain GEMV's bits, the residual stream gets x + y (one fp16
    rounding), h matches lb_decode_rmsnorm to an fp16 ulp, and the counter is left zero, so a second call in a row
    (another residual row) is right too."""
    n, k = nk
    wq = _w4(n, k, n + 5 * k)
    g = torch.Generator(device="cuda").manual_seed(n)
    ln = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).half()
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call in range(2):
        x = torch.randn(1, k, device="cuda", generator=g).half()
        res = (4 * torch.randn(n, device="cuda", generator=g)).half()
        res0 = res.clone()
        y = torch.empty(1, n, device="cuda").half()
        h = torch.full((n,), float("nan"), device="cuda").half()
        rc = _lib().lb_decode_gemv_residual_norm(x.data_ptr(), wq.packed_mma.data_ptr(), wq.scales.data_ptr(),
                                                 y.data_ptr(), n, k, 128, res.data_ptr(), ln.data_ptr(), h.data_ptr(),
                                                 1e-6, counter.data_ptr(), _stream())
        assert rc == 0, _lib().lb_last_error()
        want_y = ops.gemv(x, wq, 6)
        xs, want_h = res0.clone(), torch.empty(n, device="cuda").half()
        assert _lib().lb_decode_rmsnorm(xs.data_ptr(), want_y.data_ptr(), ln.data_ptr(), want_h.data_ptr(), n, 1e-6,
                                        _stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(y, want_y), call
        assert torch.equal(res, xs), call
        assert _ulp_close(h, want_h), call
        assert counter.item() == 0


def test_tp_allreduce_norm_simulated_peer():
    """lb_tp_allreduce_norm at world 2 with the peer simulated on this GPU: the residual stream gets x + the
    rank-ordered sum, h matches lb_decode_rmsnorm on it to an fp16 ulp, and the input is left as it was."""
    lib, cap, n = _lib(), 4096, 3584
    mine = torch.zeros(128 + 2 * cap, device="cuda").half()
    peer = torch.zeros(128 + 2 * cap, device="cuda").half()
    epoch = torch.ones(1, device="cuda", dtype=torch.int32)     # epoch 1 -> 2: slot 0
    g = torch.Generator(device="cuda").manual_seed(3)
    t = torch.randn(n, device="cuda", generator=g).half()
    other = torch.randn(n, device="cuda", generator=g).half()
    peer[128:128 + n] = other
    mine.view(torch.int32)[1] = 2
    res = (4 * torch.randn(n, device="cuda", generator=g)).half()
    res0, t0 = res.clone(), t.clone()
    ln = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).half()
    h = torch.full((n,), float("nan"), device="cuda").half()
    bufs = torch.tensor([mine.data_ptr(), peer.data_ptr()], dtype=torch.int64, device="cuda")
    assert lib.lb_tp_allreduce_norm(t.data_ptr(), n, cap, bufs.data_ptr(), epoch.data_ptr(), 0, 2, res.data_ptr(),
                                    ln.data_ptr(), h.data_ptr(), 1e-6, _stream()) == 0
    total = (t0.float() + other.float()).half()
    xs, want_h = res0.clone(), torch.empty(n, device="cuda").half()
    assert lib.lb_decode_rmsnorm(xs.data_ptr(), total.data_ptr(), ln.data_ptr(), want_h.data_ptr(), n, 1e-6,
                                 _stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(t, t0) and epoch.item() == 2
    assert torch.equal(res, xs)
    assert _ulp_close(h, want_h)
    assert lib.lb_device_error() == 0


def _fused_ar_call(lib, x, wq, y, cap, bufs, epoch, rank, world, res, ln, h, counter):
    return lib.lb_tp_gemv_allreduce_norm(x.data_ptr(), wq.packed_mma.data_ptr(), wq.scales.data_ptr(),
                                         None if y is None else y.data_ptr(), wq.n, wq.k, 128, cap, bufs.data_ptr(),
                                         epoch.data_ptr(), rank, world, res.data_ptr(), ln.data_ptr(), h.data_ptr(),
                                         1e-6, counter.data_ptr(), _stream())


def _ll_words(half_vec, epoch):
    """fp16 [n] -> the fused allreduce's n / 2 words: epoch << 32 | two fp16 outputs (little-endian pair)."""
    bits = half_vec.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return bits | (epoch << 32)


# (N, K): 7B o and down at tensor-parallel degree 2 (down splits K over a cluster at degree 1: 18944), 3B down at 2
@pytest.mark.parametrize("nk", [(3584, 1792), (3584, 9472), (2048, 5504), (3584, 18944)])
def test_tp_gemv_allreduce_norm_simulated_peer(nk):
    """lb_tp_gemv_allreduce_norm at world 2 with the peer simulated on this GPU (its partial written beforehand as
    epoch-tagged words): this rank's tiles land in region (0, rank 0) of both buffers tagged with epoch 2, the sum
    is rank 0's GEMV bits plus the peer's partial (fp32, one rounding), the residual and h match lb_decode_rmsnorm,
    the epoch advances."""
    n, k = nk
    lib, cap = _lib(), n
    wq = _w4(n, k, 11 * n + k)
    g = torch.Generator(device="cuda").manual_seed(k)
    x = torch.randn(1, k, device="cuda", generator=g).half()
    other = torch.randn(n, device="cuda", generator=g).half()
    res = (4 * torch.randn(n, device="cuda", generator=g)).half()
    ln = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).half()
    res0 = res.clone()
    words = 32 + 4 * cap // 2       # int64 words: 256 bytes of header, then 2 parities x 2 ranks x cap / 2
    mine = torch.zeros(words, device="cuda", dtype=torch.int64)
    peer = torch.zeros(words, device="cuda", dtype=torch.int64)
    region = lambda buf, par, src: buf[32 + (2 * par + src) * (cap // 2):32 + (2 * par + src) * (cap // 2) + n // 2]
    epoch = torch.ones(1, device="cuda", dtype=torch.int32)      # epoch 1 -> 2: parity 0
    region(mine, 0, 1).copy_(_ll_words(other, 2))
    bufs = torch.tensor([mine.data_ptr(), peer.data_ptr()], dtype=torch.int64, device="cuda")
    counter = torch.zeros(1, device="cuda", dtype=torch.int32)
    y = torch.full((n,), float("nan"), device="cuda").half()
    h = torch.full((n,), float("nan"), device="cuda").half()
    assert _fused_ar_call(lib, x, wq, y, cap, bufs, epoch, 0, 2, res, ln, h, counter) == 0, lib.lb_last_error()
    part = ops.gemv(x, wq, 6)[0]
    total = (part.float() + other.float()).half()
    xs, want_h = res0.clone(), torch.empty(n, device="cuda").half()
    assert lib.lb_decode_rmsnorm(xs.data_ptr(), total.data_ptr(), ln.data_ptr(), want_h.data_ptr(), n, 1e-6,
                                 _stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(region(mine, 0, 0), _ll_words(part, 2)) and torch.equal(region(peer, 0, 0), _ll_words(part, 2))
    assert torch.equal(y, total)
    assert torch.equal(res, xs)
    assert _ulp_close(h, want_h)
    assert epoch.item() == 2 and counter.item() == 0
    assert lib.lb_device_error() == 0


def test_tp_gemv_allreduce_norm_world_one_is_the_residual_norm_gemv():
    """At world 1 the fused kernel's residual and h have the bits of lb_decode_gemv_residual_norm."""
    n, k = 2048, 2048
    lib = _lib()
    wq = _w4(n, k, 5)
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(1, k, device="cuda", generator=g).half()
    res = (4 * torch.randn(n, device="cuda", generator=g)).half()
    ln = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).half()
    res2 = res.clone()
    buf = torch.zeros(32 + n, device="cuda", dtype=torch.int64)     # header + 2 parities x 1 rank x n / 2 words
    bufs = torch.tensor([buf.data_ptr()], dtype=torch.int64, device="cuda")
    epoch = torch.zeros(1, device="cuda", dtype=torch.int32)
    c1, c2 = torch.zeros(1, device="cuda", dtype=torch.int32), torch.zeros(1, device="cuda", dtype=torch.int32)
    h1, h2 = torch.empty(n, device="cuda").half(), torch.empty(n, device="cuda").half()
    assert _fused_ar_call(lib, x, wq, None, n, bufs, epoch, 0, 1, res, ln, h1, c1) == 0, lib.lb_last_error()
    y = torch.empty(1, n, device="cuda").half()
    assert lib.lb_decode_gemv_residual_norm(x.data_ptr(), wq.packed_mma.data_ptr(), wq.scales.data_ptr(),
                                            y.data_ptr(), n, k, 128, res2.data_ptr(), ln.data_ptr(), h2.data_ptr(),
                                            1e-6, c2.data_ptr(), _stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(res, res2) and torch.equal(h1, h2)
    assert epoch.item() == 1 and lib.lb_device_error() == 0


def test_tp_gemv_allreduce_norm_wait_runs_out_and_reports():
    """A peer that never publishes: the last CTA gives up after about a second, the status word reads 2, the epoch
    does not advance, the counter is left zero and the context stays usable."""
    n, k, lib = 896, 896, _lib()
    wq = _w4(n, k, 1)
    x = torch.ones(1, k, device="cuda").half()
    res, ln, h = (torch.zeros(n, device="cuda").half(), torch.ones(n, device="cuda").half(),
                  torch.empty(n, device="cuda").half())
    mine = torch.zeros(32 + 2 * n, device="cuda", dtype=torch.int64)
    peer = torch.zeros(32 + 2 * n, device="cuda", dtype=torch.int64)
    bufs = torch.tensor([mine.data_ptr(), peer.data_ptr()], dtype=torch.int64, device="cuda")
    epoch = torch.zeros(1, device="cuda", dtype=torch.int32)
    counter = torch.zeros(1, device="cuda", dtype=torch.int32)
    lib.lb_clear_device_error()
    assert _fused_ar_call(lib, x, wq, None, n, bufs, epoch, 0, 2, res, ln, h, counter) == 0
    torch.cuda.synchronize()
    assert lib.lb_device_error() == 2
    assert epoch.item() == 0 and counter.item() == 0
    lib.lb_clear_device_error()
    assert lib.lb_device_error() == 0
    assert torch.isfinite((x + 1).float()).all()


def test_decode_gemv_fusable_rule():
    assert _lib().lb_decode_gemv_fusable(2048, 11008) == 1      # 3B down: 86 chunks over 16 warps
    assert _lib().lb_decode_gemv_fusable(3584, 18944) == 0      # 7B down on one GPU: longer than one CTA holds
    assert _lib().lb_decode_gemv_fusable(3584, 9472) == 1       # the same at tensor-parallel degree 2


def _ar_call(lib, t, cap, bufs, epoch, rank, world):
    return lib.lb_tp_allreduce(t.data_ptr(), t.data_ptr(), t.numel(), cap, bufs.data_ptr(), epoch.data_ptr(), rank,
                               world, _stream())


def test_tp_allreduce_single_rank_and_simulated_peer():
    """world 1: the sum is the input; world 2 with the peer simulated on this GPU (its flag and slot written
    beforehand): the kernel passes its wait and adds the two slots in rank order."""
    lib, cap, n = _lib(), 4096, 3584
    mine = torch.zeros(128 + 2 * cap, device="cuda").half()
    peer = torch.zeros(128 + 2 * cap, device="cuda").half()
    epoch = torch.zeros(1, device="cuda", dtype=torch.int32)
    t = torch.randn(n, device="cuda").half()
    t0 = t.clone()
    bufs = torch.tensor([mine.data_ptr()], dtype=torch.int64, device="cuda")
    assert _ar_call(lib, t, cap, bufs, epoch, 0, 1) == 0
    torch.cuda.synchronize()
    assert torch.equal(t, t0) and epoch.item() == 1
    # world 2, epoch 1 -> 2: slot 0; the "peer" has published epoch 2 into this rank's flags[1]
    epoch.zero_()
    epoch += 1
    other = torch.randn(n, device="cuda").half()
    peer[128:128 + n] = other
    mine.view(torch.int32)[1] = 2
    bufs = torch.tensor([mine.data_ptr(), peer.data_ptr()], dtype=torch.int64, device="cuda")
    assert _ar_call(lib, t, cap, bufs, epoch, 0, 2) == 0
    torch.cuda.synchronize()
    assert torch.equal(t, (t0.float() + other.float()).half()) and epoch.item() == 2
    assert lib.lb_device_error() == 0


def test_tp_allreduce_wait_runs_out_and_reports():
    """A peer that never publishes its epoch: the wait gives up after about a second, the status word reads 2 and
    the epoch does not advance; the context stays usable."""
    lib, cap, n = _lib(), 1024, 1000   # n, cap multiples of 8
    mine = torch.zeros(128 + 2 * cap, device="cuda").half()
    peer = torch.zeros(128 + 2 * cap, device="cuda").half()
    epoch = torch.zeros(1, device="cuda", dtype=torch.int32)
    bufs = torch.tensor([mine.data_ptr(), peer.data_ptr()], dtype=torch.int64, device="cuda")
    t = torch.ones(n, device="cuda").half()
    lib.lb_clear_device_error()
    assert _ar_call(lib, t, cap, bufs, epoch, 0, 2) == 0
    torch.cuda.synchronize()
    assert lib.lb_device_error() == 2
    assert epoch.item() == 0
    lib.lb_clear_device_error()
    assert lib.lb_device_error() == 0
    assert torch.isfinite((t + 1).float()).all()     # the context still runs kernels
