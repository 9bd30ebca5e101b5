"""The C-ABI library: it loads without a GPU, exports every entry point include/*.h declares, and rejects bad
arguments with the documented status codes before any CUDA call (so these run on a CPU-only machine)."""
import ctypes
import pathlib
import re

import pytest

from lowbit import _lib

ROOT = pathlib.Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"LB_API\s+[\w\s\*]+?\b(lb_\w+)\s*\(", h.read_text()))
    return names


@pytest.fixture(scope="module")
def lib():
    return _lib.load_library()


def test_header_declares_the_entry_points():
    assert {"lb_w4_gemv", "lb_w4_gemm_tc", "lb_w4_dequant", "lb_w4_quantize", "lb_w4_repack"} <= declared_symbols()


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(_lib.SIGNATURES) == declared_symbols()


def test_abi_version(lib):
    text = (ROOT / "include" / "lowbit_b200.h").read_text()
    assert lib.lb_abi_version() == int(re.search(r"#define LB_ABI_VERSION (\d+)", text).group(1))


def test_status_strings(lib):
    assert lib.lb_status_string(0) == b"ok"
    assert lib.lb_status_string(1) == b"invalid argument"
    assert lib.lb_status_string(99) == b"unknown status"


def test_options_round_trip(lib):
    prev = lib.lb_set_option(1, 1)
    assert lib.lb_get_option(1) == 1
    lib.lb_set_option(1, prev)
    assert lib.lb_set_option(42, 0) == -1


class FakePtr:
    """Addresses that are never dereferenced: the checks below fail before any CUDA call."""
    A = 0x10000       # 16-byte aligned
    U = 0x10001       # misaligned


def gemv(lib, x=FakePtr.A, w=FakePtr.A, s=FakePtr.A, y=FakePtr.A, m=1, n=64, k=256, g=128, v=6, r=0):
    return lib.lb_w4_gemv(x, w, s, y, m, n, k, g, v, r, None)


@pytest.mark.parametrize("kw,code,msg", [
    (dict(g=0), 1, b"group size must be positive"),
    (dict(g=48, k=96), 1, b"multiple of the group size"),
    (dict(k=200), 1, b"multiple of the group size"),
    (dict(m=9), 1, b"1..8 rows"),
    (dict(m=0), 1, b"1..8 rows"),
    (dict(v=5), 1, b"version is 1..4 or 6"),
    (dict(v=6, g=32, k=96), 1, b"multiples of 128"),
    (dict(r=3), 1, b"rows_per_warp"),
    (dict(x=FakePtr.U), 2, b"16-byte aligned"),
    (dict(w=FakePtr.U), 2, b"16-byte aligned"),
    (dict(s=0), 1, b"null pointer"),
])
def test_gemv_rejections(lib, kw, code, msg):
    assert gemv(lib, **kw) == code
    assert msg in lib.lb_last_error()


def test_gemm_tc_rejections(lib):
    A = FakePtr.A
    assert lib.lb_w4_gemm_tc(A, A, A, A, 65, 64, 256, 128, 0, None) == 1
    assert b"1..64 rows" in lib.lb_last_error()
    assert lib.lb_w4_gemm_tc(A, A, A, A, 4, 64, 96, 32, 0, None) == 1
    assert lib.lb_w4_gemm_tc(A, A, A, A, 4, 64, 256, 128, 3, None) == 1
    assert b"row_tiles" in lib.lb_last_error()


def test_dequant_rejections(lib):
    A = FakePtr.A
    assert lib.lb_w4_dequant(A, A, A, 4, 256, 0, 0, None) == 1
    assert lib.lb_w4_dequant(A, A, A, 4, 96, 32, 2, None) == 1
    assert b"v5 layout" in lib.lb_last_error()
    assert lib.lb_w4_dequant(FakePtr.U, A, A, 4, 256, 128, 0, None) == 2
    assert lib.lb_w4_dequant(A, A, A, 4, 256, 128, 3, None) == 1


def test_quantize_and_repack_rejections(lib):
    A = FakePtr.A
    grid = (ctypes.c_float * 2)(1.0, -0.5)
    assert lib.lb_w4_quantize(A, 0, A, A, 4, 100, 128, None, 0, None) == 1
    assert lib.lb_w4_quantize(A, 0, A, A, 4, 256, 128, ctypes.cast(grid, ctypes.c_void_p), 2, None) == 1
    assert b"positive" in lib.lb_last_error()
    assert lib.lb_w4_quantize(A, 0, A, A, 4, 256, 128, None, 33, None) == 1
    assert lib.lb_w4_repack(A, A + 0x100000, 4, 96, 2, None) == 1
    assert lib.lb_w4_repack(A, A + 8, 4, 256, 2, None) == 1
    assert b"overlap" in lib.lb_last_error()
    assert lib.lb_w4_repack(A, A + 0x100000, 4, 256, 0, None) == 1


@pytest.mark.parametrize("hd", [8, 16, 24])
def test_attention_refuses_head_dims_below_one_warp(lib, hd):
    """The combine step runs one thread per head dimension with full-warp shuffle reductions, so head dims below
    32 are refused up front by both attention entry points, before any CUDA call."""
    A = FakePtr.A
    assert lib.lb_decode_attention(A, None, A, A, A, A, A, A, A, 4, 2, hd, 64, None) == 1
    assert b"32..1024" in lib.lb_last_error()
    assert lib.lb_decode_attention_noalloc(A, None, A, A, A, A, A, 4, 2, hd, 64, None) == 1
    assert b"32..1024" in lib.lb_last_error()


def test_linear_rejections(lib):
    """lb_w4_linear: the checks of lb_w4_gemv (versions 1-4, 6) or lb_w4_gemm_tc (version 5), and a 2-byte aligned
    bias; all refused before any CUDA call."""
    A = FakePtr.A
    assert lib.lb_w4_linear(A, A, A, FakePtr.U, A, 1, 64, 256, 128, 6, None) == 2
    assert b"bias" in lib.lb_last_error()
    assert lib.lb_w4_linear(A, A, A, A, A, 9, 64, 256, 128, 6, None) == 1
    assert b"1..8 rows" in lib.lb_last_error()
    assert lib.lb_w4_linear(A, A, A, A, A, 65, 64, 256, 128, 5, None) == 1
    assert b"1..64 rows" in lib.lb_last_error()
    assert lib.lb_w4_linear(A, A, A, None, A, 2, 64, 256, 128, 7, None) == 1


def test_fastcall_extension_calls_the_same_library(lib):
    """lowbit/_fastcall.so (the decode call path without ctypes) reaches the same loaded library: its refusals
    come back with the C ABI's status codes and set the same lb_last_error() message."""
    from lowbit import _fastcall
    A = FakePtr.A
    assert _fastcall.gemv(A, A, A, A, 1, 64, 256, 0, 6, None) == 1
    assert b"group size must be positive" in lib.lb_last_error()
    assert _fastcall.gemv(A, A, A, A, 65, 64, 256, 128, 5, None) == 1
    assert b"1..64 rows" in lib.lb_last_error()
    assert _fastcall.linear(A, A, A, FakePtr.U, A, 1, 64, 256, 128, 6, None) == 2
    with pytest.raises(TypeError):
        _fastcall.gemv(A, A)
