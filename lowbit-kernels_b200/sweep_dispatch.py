"""Derive the row-count dispatch table (lowbit/dispatch_b200.json) from a sweep on the current B200.

    python lowbit-kernels_b200/sweep_dispatch.py [--out sweep.json] [--write-table] [--quick]

For every Qwen2.5 0.5B/1.5B/3B projection shape and M in 1..64 plus the prefill range,
times with cold weights (>= 384 MiB of distinct copies per shape, one CUDA graph per measurement, median of 5
replays):
  * version 6 (decode GEMV, M <= 8), version 5 (tensor-core GEMM, M <= 64);
  * dequantize (mma layout) + cuBLAS fp16 GEMM -- the fallback linear() uses above the kernels' range;
  * fp16 cuBLAS on fp16 weights (for the record).
It then picks, like the reference's A1 sweep (lowbit/ops.py:136-142): AUTO_GEMV_ROWS = the largest M up to which
version 6 beats version 5 on every shape; AUTO_V5_ROWS = the largest M up to which version 5 beats
dequantize + cuBLAS on every shape; AUTO_WIDE_N / AUTO_V5_WIDE_ROWS the same restricted to wide layers.
"""
import argparse
import json
import pathlib
import statistics
import sys
import time

import torch

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from lowbit import ops  # noqa: E402

SHAPES = [  # (name, K, N)
    ("0.5b.q", 896, 896), ("0.5b.kv", 896, 128), ("0.5b.up", 896, 4864), ("0.5b.down", 4864, 896),
    ("1.5b.q", 1536, 1536), ("1.5b.kv", 1536, 256), ("1.5b.up", 1536, 8960), ("1.5b.down", 8960, 1536),
    ("3b.q", 2048, 2048), ("3b.kv", 2048, 256), ("3b.up", 2048, 11008), ("3b.down", 11008, 2048),
]
ROWS = (1, 2, 4, 8, 12, 16, 24, 32, 48, 64)
PREFILL_ROWS = (96, 128, 256)


def capture(fn):
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g):
        fn()
    return g


def timed(fn, copies, reps=5):
    """Median per-call microseconds of a graph that calls fn(c) once for every copy c."""
    g = capture(lambda: [fn(c) for c in range(copies)])
    for _ in range(2):
        g.replay()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1e3 / copies)
    del g
    return statistics.median(ts)


def sweep(shapes, rows, prefill):
    dev = torch.device("cuda")
    out = []
    for name, k, n in shapes:
        w4_bytes = n * k // 2 + 2 * n * (k // 128)
        copies = max(4, (384 << 20) // w4_bytes)
        wqs = [ops.W4Weight.from_float(torch.randn(n, k, device=dev) * 0.02, 128, ("mma",)) for _ in range(copies)]
        c16 = max(2, (384 << 20) // (2 * n * k))
        w16 = [ops.dequant(wqs[i], "mma") for i in range(min(c16, copies))]
        for m in rows + prefill:
            x = torch.randn(m, k, device=dev).half()
            r = {"shape": name, "K": k, "N": n, "M": m}
            if m <= ops.MAX_ROWS[6]:
                r["v6_us"] = timed(lambda c: ops.gemv(x, wqs[c], 6), copies)
            if m <= ops.MAX_ROWS[5]:
                r["v5_us"] = timed(lambda c: ops.gemv(x, wqs[c], 5), copies)
            r["dequant_cublas_us"] = timed(lambda c: torch.nn.functional.linear(x, ops.dequant(wqs[c], "mma")), copies)
            r["fp16_cublas_us"] = timed(lambda c: torch.nn.functional.linear(x, w16[c % len(w16)]), len(w16))
            r["bytes_int4"] = w4_bytes + 2 * (m * k + m * n)
            out.append(r)
            print(json.dumps(r), flush=True)
        del wqs, w16
        torch.cuda.empty_cache()
    return out


def derive(results, wide_n=3072):
    """The largest row counts at which each kernel wins on every shape (the reference's rule structure)."""
    def wins(a, b, pred):
        ms = sorted({r["M"] for r in results if a in r and b in r})
        best = 0
        for m in ms:
            rs = [r for r in results if r["M"] == m and a in r and b in r and pred(r)]
            if rs and all(r[a] <= r[b] for r in rs):
                best = m
            else:
                break
        return best
    # versions 6 and 5 run the same kernel up to 8 rows: ties go to version 6 up to its row limit
    gemv_rows = max(wins("v6_us", "v5_us", lambda r: True), max(r["M"] for r in results if "v6_us" in r))
    v5_rows = wins("v5_us", "dequant_cublas_us", lambda r: True)
    v5_wide = wins("v5_us", "dequant_cublas_us", lambda r: r["N"] >= wide_n)
    return {"AUTO_GEMV_ROWS": max(1, gemv_rows), "AUTO_V5_ROWS": max(v5_rows, gemv_rows),
            "AUTO_V5_WIDE_ROWS": max(v5_wide, v5_rows, gemv_rows), "AUTO_WIDE_N": wide_n}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    ap.add_argument("--write-table", action="store_true", help="overwrite lowbit/dispatch_b200.json")
    ap.add_argument("--quick", action="store_true", help="four shapes only")
    a = ap.parse_args()
    e = ops.ext()
    e.set_option("early_weights", 1)
    shapes = [SHAPES[i] for i in (0, 5, 10, 11)] if a.quick else SHAPES
    t0 = time.time()
    results = sweep(shapes, ROWS, PREFILL_ROWS)
    table = derive(results)
    table["source"] = (f"sweep_dispatch.py on {torch.cuda.get_device_name()} "
                       f"({time.strftime('%Y-%m-%d')}): {len(results)} cells, {time.time() - t0:.0f} s")
    print(json.dumps(table), flush=True)
    if a.out:
        pathlib.Path(a.out).write_text(json.dumps({"table": table, "results": results}, indent=1))
    if a.write_table:
        (ROOT / "lowbit" / "dispatch_b200.json").write_text(json.dumps(table, indent=2) + "\n")


if __name__ == "__main__":
    main()
