"""The CPU oracle (oracle/) and the host format module (lowbit.quant) against golden vectors that the reference's
own Python produced (tests/golden/make_golden.py): quantize, both interleaves, fp32 and fp16 dequantize, the
fp64 GEMV, and the overflow known answer (bench/gpu_run.py:144-159 of the reference)."""
import numpy as np
import pytest

from lowbit import quant
from oracle import oracle as O


def tags(golden):
    return sorted({k.split("_")[0] for k in golden.files if not k.startswith("overflow")})


def bits16(a):
    return np.asarray(a, np.float16).view(np.uint16)


def test_golden_file_covers_every_group_size(golden):
    groups = {int(golden[f"{t}_group"]) for t in tags(golden)}
    assert groups == {32, 64, 128, 256}


@pytest.mark.parametrize("impl", ["c", "numpy"])
def test_quantize_matches_reference_bits(golden, impl):
    for t in tags(golden):
        w, g = golden[f"{t}_w"], int(golden[f"{t}_group"])
        packed, scales = O.c_quantize(w, g) if impl == "c" else quant.quantize_w4(w, g)
        assert np.array_equal(packed, golden[f"{t}_packed"]), t
        assert np.array_equal(bits16(scales), bits16(golden[f"{t}_scales"])), t


def test_interleaves_match_reference(golden):
    for t in tags(golden):
        p = golden[f"{t}_packed"]
        assert np.array_equal(O.c_interleave_gpu(p), golden[f"{t}_v3"]), t
        assert np.array_equal(quant.interleave_for_gpu(p), golden[f"{t}_v3"]), t
        if f"{t}_mma" in golden.files:
            assert np.array_equal(O.c_interleave_mma(p), golden[f"{t}_mma"]), t
            assert np.array_equal(quant.interleave_for_mma(p), golden[f"{t}_mma"]), t


def test_dequantize_matches_reference(golden):
    for t in tags(golden):
        p, s, g = golden[f"{t}_packed"], golden[f"{t}_scales"], int(golden[f"{t}_group"])
        assert np.array_equal(O.c_dequantize_f32(p, s, g), golden[f"{t}_deq32"]), t
        assert np.array_equal(quant.dequantize_w4(p, s, g), golden[f"{t}_deq32"]), t
        assert np.array_equal(O.np_dequantize_w4(p, s, g), golden[f"{t}_deq32"]), t
        want16 = bits16(golden[f"{t}_deq16"])
        assert np.array_equal(bits16(O.c_dequantize_f16(p, s, g)), want16), t
        assert np.array_equal(bits16(O.c_dequantize_f16(golden[f"{t}_v3"], s, g, "v3")), want16), t
        if f"{t}_mma" in golden.files:
            assert np.array_equal(bits16(O.c_dequantize_f16(golden[f"{t}_mma"], s, g, "mma")), want16), t


def test_torch_cpu_restatement_matches_reference_fp16(golden):
    torch = pytest.importorskip("torch")
    for t in tags(golden):
        p, s, g = golden[f"{t}_packed"], golden[f"{t}_scales"], int(golden[f"{t}_group"])
        got = O.torch_dequantize(torch.from_numpy(p), torch.from_numpy(s), g).numpy()
        assert np.array_equal(bits16(got), bits16(golden[f"{t}_deq16"])), t


@pytest.mark.parametrize("layout", ["canonical", "v3", "mma"])
def test_fp64_gemv_matches_reference(golden, layout):
    for t in tags(golden):
        key = {"canonical": "packed", "v3": "v3", "mma": "mma"}[layout]
        if f"{t}_{key}" not in golden.files:
            continue
        g = int(golden[f"{t}_group"])
        y = O.c_gemv_ref(golden[f"{t}_x16"], golden[f"{t}_{key}"], golden[f"{t}_scales"], g, layout)
        np.testing.assert_allclose(y, golden[f"{t}_y64"], rtol=1e-12, atol=1e-12)
        y2 = quant.gemv_reference(golden[f"{t}_x16"].astype(np.float64), golden[f"{t}_packed"], golden[f"{t}_scales"], g)
        np.testing.assert_allclose(y2, golden[f"{t}_y64"], rtol=1e-12, atol=1e-12)


def test_overflow_known_answer(golden):
    packed = np.full((16, 64), 0xFF, np.uint8)
    scales = np.full((16, 1), 2.0 ** -10, np.float16)
    for xv in (4096.0, -8192.0):
        want = golden[f"overflow_{int(xv)}_y64"]
        assert float(want[0, 0]) == 7 * 2.0 ** -10 * 128 * xv
        y = O.c_gemv_ref(np.full((1, 128), xv, np.float16), packed, scales, 128)
        assert np.array_equal(y, want)


def test_oracle_f16_conversion_is_round_to_nearest_even():
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-7, 1e-5, 1e-3, 1, 1e3, 6e4)]
                          + [np.array([65504, 65519.99, 65520, 1e9, -1e9, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26, 0.0,
                                       -0.0], np.float32)])
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    L = O.lib()
    got = np.array([L.lbo_f32_to_f16(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, want)
    back = np.array([L.lbo_f16_to_f32(int(h)) for h in want[:2000]], np.float32)
    assert np.array_equal(back, want[:2000].view(np.float16).astype(np.float32))


def test_oracle_rejects_bad_shapes():
    with pytest.raises(ValueError):
        O.c_quantize(np.zeros((4, 100), np.float32), 128)
    with pytest.raises(ValueError):
        O.c_interleave_mma(np.zeros((1, 32), np.uint8))
