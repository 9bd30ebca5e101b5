"""lb_decode_attention_noalloc (scratch held by the library) against lb_decode_attention (caller-owned scratch).

Self-contained and collected last: it passes alone and after every other test file.
"""
import pytest
import torch

from lowbit import _lib

LB_ERR_ARGUMENT = 1


def test_noalloc_refuses_calls_larger_than_its_scratch():
    """64 heads over a 65536-token cache need 64 * 1024 * 130 floats, far above the 262144 the library holds: the
    call fails with LB_ERR_ARGUMENT before touching the device (fake, aligned pointers; no GPU needed)."""
    lib = _lib.load_library()
    p = 0x10000
    rc = lib.lb_decode_attention_noalloc(p, None, p, p, p, p, p, 64, 8, 128, 65536, None)
    assert rc == LB_ERR_ARGUMENT
    msg = lib.lb_last_error().decode()
    assert "scratch" in msg and "262144" in msg and "lb_decode_attention" in msg


def test_attention_refuses_shapes_its_kernels_do_not_take():
    """head dims that are not a multiple of 8, caches longer than 65536 rows and head groups whose tiles exceed a
    CTA's shared memory fail with a message before touching the device (fake, aligned pointers; no GPU needed)."""
    lib = _lib.load_library()
    p = 0x10000
    call = lambda nh, nkv, hd, max_len: lib.lb_decode_attention(p, None, p, p, p, p, p, p, p, nh, nkv, hd, max_len,
                                                                None)
    assert call(16, 2, 12, 1024) == LB_ERR_ARGUMENT and "multiple of 8" in lib.lb_last_error().decode()
    assert call(16, 2, 128, 65537) == LB_ERR_ARGUMENT and "65536" in lib.lb_last_error().decode()
    assert call(128, 1, 1024, 1024) == 3 and "shared memory" in lib.lb_last_error().decode()   # LB_ERR_UNSUPPORTED


@pytest.mark.gpu
@pytest.mark.parametrize("heads", [(16, 2, 128), (28, 4, 128)])
def test_noalloc_matches_caller_scratch_on_two_calls_in_a_row(heads):
    from lowbit import ops
    lib = ops.ext().lib
    nh, nkv, hd = heads
    max_len = 1024
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(nh)
    rows = (nh + 2 * nkv) * hd
    bias = (0.1 * torch.randn(rows, device="cuda", generator=g)).half()
    inv_freq = (1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))).cuda()
    k0 = torch.randn(nkv, max_len, hd, device="cuda", generator=g).half()
    v0 = torch.randn(nkv, max_len, hd, device="cuda", generator=g).half()
    caches = {"own": (k0.clone(), v0.clone()), "noalloc": (k0.clone(), v0.clone())}
    splits = lib.lb_decode_attention_splits(max_len)
    part_o = torch.empty(nh * splits * hd, device="cuda")
    part_ml = torch.empty(nh * splits * 2, device="cuda")
    for pos in (700, 701):   # the second call reads the cache row the first one appended
        qkv = torch.randn(rows, device="cuda", generator=g).half()
        p = torch.tensor([pos], device="cuda")
        out = {}
        for path, (kc, vc) in caches.items():
            o = torch.full((nh * hd,), float("nan"), device="cuda").half()
            if path == "own":
                rc = lib.lb_decode_attention(qkv.data_ptr(), bias.data_ptr(), inv_freq.data_ptr(), p.data_ptr(),
                                             kc.data_ptr(), vc.data_ptr(), part_o.data_ptr(), part_ml.data_ptr(),
                                             o.data_ptr(), nh, nkv, hd, max_len, st)
            else:
                rc = lib.lb_decode_attention_noalloc(qkv.data_ptr(), bias.data_ptr(), inv_freq.data_ptr(),
                                                     p.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), nh,
                                                     nkv, hd, max_len, st)
            assert rc == 0, lib.lb_last_error()
            out[path] = o
        torch.cuda.synchronize()
        assert torch.isfinite(out["own"].float()).all()
        assert torch.equal(out["own"], out["noalloc"]), pos
        assert torch.equal(caches["own"][0], caches["noalloc"][0])
        assert torch.equal(caches["own"][1], caches["noalloc"][1])
