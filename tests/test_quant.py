"""Format pins for lowbit.quant (host side, numpy only), restating what the reference's tests/test_quant.py pins:
error bound, nibble order and exact bytes, range, bad shapes, the bit logic each kernel layout relies on, the
magic-number trick, and that the interleaves are permutations."""
import numpy as np
import pytest

from lowbit import quant

RNG = np.random.default_rng(11)


def words(packed):
    return np.ascontiguousarray(packed).view("<u4")


def test_quantization_error_is_at_most_half_a_step():
    w = RNG.standard_normal((32, 384)).astype(np.float32)
    packed, scales = quant.quantize_w4(w, 128)
    err = np.abs(quant.dequantize_w4(packed, scales, 128) - w).reshape(32, 3, 128)
    step = scales.astype(np.float32)[..., None]
    # values clipped at -8 only ever gain precision (|w| <= 7 * scale up to fp16 rounding of the scale)
    assert np.all(err <= step / 2 + step * 2e-3)


def test_two_nibbles_per_byte_low_nibble_first():
    w = np.zeros((1, 128), np.float32)
    w[0, :6] = [7, -7, 1, 0, -3, 2]
    packed, scales = quant.quantize_w4(w, 128)
    assert scales[0, 0] == 1.0
    assert list(packed[0, :3]) == [15 | (1 << 4), 9 | (8 << 4), 5 | (10 << 4)]


def test_range_and_zero_group():
    w = RNG.standard_normal((6, 256)).astype(np.float32) * 100
    w[2] = 0
    packed, scales = quant.quantize_w4(w, 128)
    q = quant.unpack_w4(packed)
    assert q.min() >= -8 and q.max() <= 7
    assert np.all(scales[2] == 1.0)
    assert np.all(quant.dequantize_w4(packed, scales, 128)[2] == 0)


def test_round_half_to_even():
    w = np.zeros((1, 128), np.float32)
    w[0, 0] = 7.0                                  # scale 1.0
    w[0, 1:6] = [0.5, 1.5, 2.5, -0.5, -2.5]
    q = quant.unpack_w4(quant.quantize_w4(w, 128)[0])[0, :6]
    assert list(q) == [7, 0, 2, 2, 0, -2]


@pytest.mark.parametrize("k,g", [(100, 128), (96, 48), (128, 0), (256, 96)])
def test_rejects_bad_shapes(k, g):
    with pytest.raises(ValueError):
        quant.quantize_w4(np.zeros((4, k), np.float32), g)


def test_canonical_words_hold_k0_to_k7_in_nibble_order():
    packed, _ = quant.quantize_w4(RNG.standard_normal((5, 256)).astype(np.float32))
    u = quant.unpack_w4(packed) + 8
    wd = words(packed)
    for b in range(8):
        assert np.array_equal((wd >> (4 * b)) & 0xF, u[:, b::8])


def test_v3_words_give_consecutive_pairs_after_one_mask():
    packed, _ = quant.quantize_w4(RNG.standard_normal((5, 256)).astype(np.float32))
    u = quant.unpack_w4(packed) + 8
    wd = words(quant.interleave_for_gpu(packed)).astype(np.uint64)
    for j in range(4):
        t = (wd >> (4 * j)) & 0x000F000F
        assert np.array_equal(t & 0xFFFF, u[:, 2 * j::8])
        assert np.array_equal(t >> 16, u[:, 2 * j + 1::8])


def test_magic_number_conversion_is_exact():
    u = np.arange(16, dtype=np.uint16)
    lo = (u | 0x6400).view(np.float16)
    assert np.array_equal(lo - np.float16(1032), (u.astype(np.int16) - 8).astype(np.float16))
    # the high-nibble form used by the kernels: (1024 + 16u) / 16 - 72 = u - 8, exactly
    hi = ((u << 4) | 0x6400).view(np.float16)
    assert np.array_equal(hi * np.float16(1 / 16) - np.float16(72), (u.astype(np.int16) - 8).astype(np.float16))


def test_interleaves_are_permutations_of_each_row():
    packed, _ = quant.quantize_w4(RNG.standard_normal((3, 384)).astype(np.float32))
    for inter in (quant.interleave_for_gpu(packed), quant.interleave_for_mma(packed)):
        assert inter.shape == packed.shape
        for r in range(3):
            assert sorted(quant.unpack_w4(inter)[r]) == sorted(quant.unpack_w4(packed)[r])


def test_mma_layout_holds_each_lanes_fragment():
    """Lane t of a tensor-core quad reads 16-byte word t of a 64-byte chunk: pair j of its word i is
    k = 128c + 32i + 8j + 2t and k + 1."""
    packed, _ = quant.quantize_w4(RNG.standard_normal((2, 384)).astype(np.float32))
    u = quant.unpack_w4(packed) + 8
    wd = quant.interleave_for_mma(packed).reshape(2, 3, 4, 4, 4).view("<u4")[..., 0]   # [row, chunk, t, word i]
    for c in range(3):
        for t in range(4):
            for i in range(4):
                for j in range(4):
                    k = 128 * c + 32 * i + 8 * j + 2 * t
                    wv = int(wd[1, c, t, i])
                    assert (wv >> (4 * j)) & 0xF == u[1, k]
                    assert (wv >> (4 * j + 16)) & 0xF == u[1, k + 1]


def test_mma_layout_rejects_k_not_multiple_of_128():
    with pytest.raises(ValueError):
        quant.interleave_for_mma(np.zeros((1, 32), np.uint8))


def test_gemv_reference_is_x_times_dequantized_weights():
    w = RNG.standard_normal((16, 256)).astype(np.float32)
    x = RNG.standard_normal((3, 256)).astype(np.float32)
    packed, scales = quant.quantize_w4(w, 128)
    y = quant.gemv_reference(x, packed, scales, 128)
    assert y.shape == (3, 16) and y.dtype == np.float64
    np.testing.assert_allclose(y, x @ quant.dequantize_w4(packed, scales, 128).T, rtol=1e-5, atol=1e-4)
