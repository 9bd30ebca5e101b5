"""linear() routing and W4Weight validation on the CPU: gemv / dequant are stubbed, so no kernel runs.
Restates the reference's tests/test_dispatch.py pins under the reference's T4 constants, and checks the
same rule under the B200 table."""
import types

import numpy as np
import pytest

torch = pytest.importorskip("torch")
from lowbit import ops  # noqa: E402

REF = {"AUTO_GEMV_ROWS": 1, "AUTO_V5_ROWS": 32, "AUTO_V5_WIDE_ROWS": 64, "AUTO_WIDE_N": 3072}


def weight(n=1024, k=256, layouts=("mma",)):
    have = lambda name: object() if name in layouts else None  # noqa: E731
    return types.SimpleNamespace(n=n, k=k, group=128, packed=have("canonical"), packed_v3=have("v3"),
                                 packed_mma=have("mma"))


@pytest.fixture
def calls(monkeypatch):
    seen = []
    monkeypatch.setattr(ops, "gemv", lambda x, wq, v, rpw=0, out=None: seen.append(v) or
                        (torch.zeros(x.shape[0], wq.n) if out is None else out))
    monkeypatch.setattr(ops, "dequant", lambda wq, layout=None: seen.append("dequant") or torch.zeros(wq.n, wq.k))
    return seen


@pytest.fixture
def reference_constants(monkeypatch):
    for k, v in REF.items():
        monkeypatch.setattr(ops, k, v)


@pytest.mark.parametrize("m,n,want", [(1, 1024, 6), (2, 1024, 5), (32, 1024, 5), (33, 1024, "dequant"),
                                      (33, 4096, 5), (64, 4096, 5), (65, 4096, "dequant")])
def test_reference_rule_on_the_mma_layout(calls, reference_constants, m, n, want):
    ops.linear(torch.zeros(m, 256), weight(n))
    assert calls == [want]


@pytest.mark.parametrize("layouts,m,want", [(("canonical", "v3"), 1, 4), (("canonical", "v3"), 8, 4),
                                            (("canonical",), 3, 2), (("canonical", "v3"), 9, "dequant")])
def test_rule_without_the_mma_layout(calls, layouts, m, want):
    ops.linear(torch.zeros(m, 256), weight(layouts=layouts))
    assert calls == [want]


def test_b200_table_is_consistent():
    assert 1 <= ops.AUTO_GEMV_ROWS <= ops.MAX_ROWS[6]
    assert ops.AUTO_GEMV_ROWS <= ops.AUTO_V5_ROWS <= ops.MAX_ROWS[5]
    assert ops.AUTO_V5_ROWS <= ops.AUTO_V5_WIDE_ROWS <= ops.MAX_ROWS[5]
    assert "source" in ops.DISPATCH


@pytest.mark.parametrize("n", [128, 1024, 4096, 11008])
def test_b200_rule_boundaries(calls, n):
    limit = ops.AUTO_V5_WIDE_ROWS if n >= ops.AUTO_WIDE_N else ops.AUTO_V5_ROWS
    cases = [(1, 6), (ops.AUTO_GEMV_ROWS, 6), (limit + 1, "dequant")]
    if limit > ops.AUTO_GEMV_ROWS:
        cases += [(ops.AUTO_GEMV_ROWS + 1, 5), (limit, 5)]
    for m, want in cases:
        calls.clear()
        ops.linear(torch.zeros(m, 256), weight(n))
        assert calls == [want], (n, m)


def test_a_fixed_version_never_passes_its_row_limit(calls):
    ops.linear(torch.zeros(9, 256), weight(), max_gemv_rows=16, version=6)
    ops.linear(torch.zeros(64, 256), weight(), version=5)
    ops.linear(torch.zeros(65, 256), weight(), version=5)
    assert calls == ["dequant", 5, "dequant"]


def test_out_is_forwarded_and_returned(calls):
    buf = torch.empty(1, 1024)
    assert ops.linear(torch.zeros(1, 256), weight(), out=buf) is buf
    assert calls == [6]


def test_bad_versions_and_empty_input(calls):
    with pytest.raises(ValueError):
        ops.linear(torch.zeros(4, 256), weight(), version=7)
    assert ops.linear(torch.zeros(0, 256), weight()).shape == (0, 1024)
    assert calls == []


def test_gemv_refuses_a_layout_the_weight_does_not_keep():
    with pytest.raises(ValueError, match="packed_v3"):
        ops.gemv(torch.zeros(1, 256), weight(layouts=("mma",)), 4)
    with pytest.raises(ValueError):
        ops.gemv(torch.zeros(1, 256), weight(), 7)


def test_construction_checks_layouts_before_touching_the_gpu():
    packed, scales = np.zeros((4, 48), np.uint8), np.ones((4, 3), np.float16)       # K = 96, G = 32
    with pytest.raises(ValueError, match="multiples of 128"):
        ops.W4Weight(packed, scales, 32, ("mma",))
    with pytest.raises(ValueError, match="canonical or the mma"):
        ops.W4Weight(packed, scales, 32, ("v3",))
    with pytest.raises(ValueError, match="unknown layout"):
        ops.W4Weight(packed, scales, 32, ("nope",))


def test_dequant_refuses_a_layout_not_kept():
    with pytest.raises(ValueError, match="not kept"):
        ops.dequant(weight(layouts=("mma",)), "canonical")


def test_quantize_rejects_bad_shapes_before_the_gpu():
    with pytest.raises(ValueError):
        ops.quantize_w4_gpu(torch.zeros(4, 100), 128)


def test_pick_rows_matches_the_reference_rule():
    assert [ops.pick_rows(n, m) for n, m in ((512, 1), (511, 4), (511, 3), (128, 1))] == [4, 2, 1, 1]
