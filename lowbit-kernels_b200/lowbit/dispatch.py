"""How linear()'s row-count dispatch table (dispatch_b200.json) follows from a B200 sweep.

The reference fixes its constants from its own A1 sweep on a T4 (lowbit/ops.py:136-142) with this rule structure:
up to AUTO_GEMV_ROWS rows the decode GEMV (version 6), up to AUTO_V5_ROWS rows the tensor-core kernel (version 5;
AUTO_V5_WIDE_ROWS on layers with N >= AUTO_WIDE_N), dequantize + cuBLAS above. ``derive`` applies the same rule to
a sweep record of this library's kernels on B200 -- one cell per (shape, M) with the per-call times of version 6
(M <= 8), version 5 (M <= 64) and dequantize + cuBLAS, all with cold weights -- so the table can be regenerated and
checked from the committed record (`python bench.py --sweep-dispatch` writes one).
"""
import json
import pathlib

TABLE_PATH = pathlib.Path(__file__).resolve().parent / "dispatch_b200.json"
KEYS = ("AUTO_GEMV_ROWS", "AUTO_V5_ROWS", "AUTO_V5_WIDE_ROWS", "AUTO_WIDE_N")


# Timing noise of a cell: the same kernel timed twice in one sweep (versions 5 and 6 share the decode kernel up to
# 8 rows) differs by up to 5 % on B200, so a kernel "wins" a cell when it is at most that much slower.
NOISE = 1.05


def _prefix_wins(cells, fast, slow, keep=lambda c: True, tol=NOISE):
    """The largest M such that, for every swept M' <= M, `fast` is no slower than `slow` (within `tol`) on every
    kept shape."""
    best = 0
    for m in sorted({c["M"] for c in cells if fast in c and slow in c}):
        row = [c for c in cells if c["M"] == m and fast in c and slow in c and keep(c)]
        if row and all(c[fast] <= c[slow] * tol for c in row):
            best = m
        else:
            break
    return best


def derive(cells, wide_n=3072):
    """The dispatch constants a sweep record implies: the reference's structure, each kernel taking the row counts
    up to which it wins every shape within timing noise. Ties between versions 6 and 5 (one kernel up to 8 rows)
    go to the decode GEMV up to its row limit."""
    v6_rows = max(c["M"] for c in cells if "v6_us" in c)
    gemv_rows = max(1, _prefix_wins(cells, "v6_us", "v5_us") or 1)
    if all(c["v6_us"] <= c["v5_us"] * NOISE for c in cells if "v6_us" in c and "v5_us" in c):
        gemv_rows = v6_rows
    v5_rows = _prefix_wins(cells, "v5_us", "dequant_cublas_us")
    v5_wide = _prefix_wins(cells, "v5_us", "dequant_cublas_us", lambda c: c["N"] >= wide_n)
    return {"AUTO_GEMV_ROWS": gemv_rows, "AUTO_V5_ROWS": max(v5_rows, gemv_rows),
            "AUTO_V5_WIDE_ROWS": max(v5_wide, v5_rows, gemv_rows), "AUTO_WIDE_N": wide_n}


def table_from_record(path):
    """The constants derived from a sweep record written by `bench.py --sweep-dispatch`."""
    rec = json.loads(pathlib.Path(path).read_text())
    return derive(rec["cells"], rec.get("wide_n", 3072))
