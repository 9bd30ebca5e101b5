"""linear()'s B200 dispatch table follows from a committed sweep record by the reference's rule structure
(lowbit/ops.py:136-142): the derivation on synthetic records, and the committed table against the committed record."""
import json
import pathlib

import pytest

from lowbit import dispatch

ROOT = pathlib.Path(__file__).resolve().parent.parent
RECORD = ROOT / "profiles" / "dispatch_sweep_b200.json"


def cell(n, m, v6=None, v5=None, dq=10.0):
    c = {"K": 1024, "N": n, "M": m, "dequant_cublas_us": dq}
    if v6 is not None:
        c["v6_us"] = v6
    if v5 is not None:
        c["v5_us"] = v5
    return c


def test_derive_takes_the_largest_prefix_each_kernel_wins():
    cells = []
    for n in (1024, 4096):
        for m in (1, 2, 4, 8):
            cells.append(cell(n, m, v6=1.0 + m, v5=1.0 + m))      # ties: the decode kernel keeps its rows
        for m in (16, 32):
            cells.append(cell(n, m, v5=5.0))
        # the tensor-core kernel loses at 48 rows on the narrow layer only
        cells.append(cell(n, 48, v5=12.0 if n == 1024 else 9.0))
        cells.append(cell(n, 64, v5=9.5))
    t = dispatch.derive(cells)
    assert t == {"AUTO_GEMV_ROWS": 8, "AUTO_V5_ROWS": 32, "AUTO_V5_WIDE_ROWS": 64, "AUTO_WIDE_N": 3072}


def test_derive_gives_rows_to_the_faster_kernel():
    cells = [cell(2048, m, v6=3.0, v5=2.0) for m in (1, 2)] + [cell(2048, 4, v5=20.0)]
    t = dispatch.derive(cells)
    assert t["AUTO_GEMV_ROWS"] == 1 and t["AUTO_V5_ROWS"] == 2


@pytest.mark.skipif(not RECORD.exists(), reason="no sweep record committed yet")
def test_committed_table_follows_from_the_committed_sweep():
    table = json.loads(dispatch.TABLE_PATH.read_text())
    derived = dispatch.table_from_record(RECORD)
    assert {k: table[k] for k in dispatch.KEYS} == derived
