"""Benchmark: W4A16 GEMV HBM throughput on the Qwen2.5 decode projections, B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-per-shape] [--no-skinny]
                    [--no-dequant] [--no-decode] [--no-cpu]

A step is one decode pass (M = 1) over every projection of Qwen2.5-0.5B, 1.5B and 3B: q, k, v, o, gate, up,
down -- 21 GEMV calls. Weights are cold: the step cycles through enough distinct copies of the 21 weights
(>= 1 GiB, 8x the 126 MB L2) that every call reads its weights from HBM. The metric is the reference's
effective bandwidth (bench/gpu_run.py:255,267): bytes = N*K/2 + 2*N*K/128 + 2*(M*K + M*N) per call, divided
by time.

  value   whole-job GB/s with everything resident in HBM: K steps captured as CUDA graphs (one kernel launch per
          call, programmatic dependent launch between them), timed with CUDA events on the launching stream,
          max over ranks;
  e2e     the same metric through the public API (lowbit.ops.linear), eager, with each step's activations copied
          from pinned host memory to the GPU (one copy) and its outputs copied back (one copy) inside the timed
          region, the stream synchronized at the end of every step;
  e2e_graph
          the same step -- both copies and the public calls -- captured once in a CUDA graph, as a decode loop
          captures its step, and replayed every step with a synchronize: the host cost of eager calls (one CUDA
          launch, ~2.5 us on the B200 hosts, per call) taken out;
  cpu_baseline / --impl reference
          the reference's CPU path (dequantize on CPU tensors + fp32 F.linear, lowbit/ops.py:119-123) restated in
          oracle/oracle.py, timed on the host cores of this machine.

The same line carries the other BASELINE configurations, measured after the timed sweep in the same run:
  per_shape   each config-1 projection alone (cold copies), with the reference's own gemv_v6 on the same copies
              (ref_us; the reference's csrc/w4_gemv.cu built unchanged for sm_100a into oracle/_ref/);
  skinny      config 2: M = 2..64 over the config-1 and tail shapes -- the kernel linear() picks, the INT4
              tensor-core kernel, dequantize + cuBLAS and fp16 cuBLAS in the same run, and the reference's gemm_v5;
  dequant     north-star subsystem 3: the prefill dequantize kernel per shape, and dequantize + cuBLAS against
              fp16 cuBLAS at 128-1024 rows;
  decode_3b   config 3: Qwen2.5-3B batch-1 decode tok/s, one CUDA graph per step (replicas at N > 1);
  tp_decode   config 4: Qwen2.5-7B tensor-parallel decode tok/s over all ranks (the unsharded model at N = 1).
The kernel legs run at N = 1 only; the decoder legs at every N.

Under torchrun (--gpus N > 1) each rank runs the same sweep on its own GPU (the single-layer benchmark has no
exchange step: replicas, weak scaling); value sums all ranks' bytes over the slowest rank's time.
"""
import argparse
import itertools
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
for p in (ROOT / "lowbit-kernels_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import faulthandler  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402

faulthandler.enable()   # a crash in native code prints the Python stack

METRIC = "W4A16 GEMV HBM GB/s (% of ~8 TB/s) at M=1-64; Qwen2.5-3B decode tok/s"
MODELS = {  # hidden, intermediate, q width, kv width
    "qwen2.5-0.5b": (896, 4864, 896, 128),
    "qwen2.5-1.5b": (1536, 8960, 1536, 256),
    "qwen2.5-3b": (2048, 11008, 2048, 256),
}
GROUP = 128
ROTATION_BYTES = 1 << 30
L2_BYTES = 126 * 10 ** 6
FALLBACK_HBM_GBS = 6650.0


def projections():
    """[(model, proj, K, N)] in decode order."""
    out = []
    for name, (h, inter, q, kv) in MODELS.items():
        out += [(name, "q", h, q), (name, "k", h, kv), (name, "v", h, kv), (name, "o", q, h),
                (name, "gate", h, inter), (name, "up", h, inter), (name, "down", inter, h)]
    return out


def call_bytes(k, n, m=1):
    return n * k // 2 + 2 * n * (k // GROUP) + 2 * (m * k + m * n)


def rank_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def measured_peak():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        if d.get("hbm_gbs"):
            return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy read+write)"
    return FALLBACK_HBM_GBS, "fallback (6.65 TB/s, earlier measurement on this pool)"


def profiled_traffic():
    """DRAM bytes (read + write) per launch of the decode GEMV over one sweep step, as last measured by ncu on this
    build's kernel (profiles/traffic.json: the figure, the kernel and the capture command), or None."""
    f = ROOT / "profiles" / "traffic.json"
    if not f.exists():
        return None
    try:
        return float(json.loads(f.read_text())["traffic_bytes_per_launch"])
    except (ValueError, KeyError):
        return None


# ------------------------------------------------------------------------------------------------ clocks

class ClockSampler:
    """SM clock, power and throttle reasons sampled through NVML in a thread (~10 ms period)."""

    REASONS = {  # NVML clocks-event reason bits
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index):
        self.samples, self.stop_evt, self.ok = [], threading.Event(), False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # noqa: BLE001 - clocks are reported as unavailable, the bench still runs
            self.err = str(e)

    def _run(self):
        while not self.stop_evt.is_set():
            self.sample()
            time.sleep(0.01)

    def sample(self):
        try:
            mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
            reasons = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            self.samples.append((time.perf_counter(), mhz, reasons))
        except Exception:  # noqa: BLE001
            pass

    def __enter__(self):
        if self.ok:
            self.sample()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self.stop_evt.set()
            self.t.join()
            self.sample()

    def summary(self, t0, t1):
        if not self.ok:
            return {"unavailable": getattr(self, "err", "nvml")}
        win = [s for s in self.samples if t0 <= s[0] <= t1] or self.samples[-2:]
        mhz = [s[1] for s in win]
        bits = 0
        for s in win:
            bits |= s[2]
        reasons = [v for k, v in self.REASONS.items() if bits & k and v != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(win), "source": "nvml, ~10 ms period, during the timed region"}


# ------------------------------------------------------------------------------------------------ our arm

def build_sets(ops, quant, device, n_sets, seed=0):
    """n_sets independent copies of the 21 projection weights (mma layout only, as a model keeps them)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    sets = []
    for _ in range(n_sets):
        layer = []
        for _, _, k, n in projections():
            w = torch.randn(n, k, device=device, generator=gen) * 0.02
            packed, scales = ops.quantize_w4_gpu(w, GROUP)
            layer.append(ops.W4Weight(packed, scales, GROUP, ("mma",)))
            del w, packed
        sets.append(layer)
    return sets


def capture(fn):
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g):
        out = fn()
    return g, out


_T0 = time.perf_counter()


def progress(rank, what):
    """One line per benchmark leg on stderr (rank 0), so a run that dies shows where."""
    if rank == 0:
        print(f"[bench {time.perf_counter() - _T0:7.1f} s] {what}", file=sys.stderr, flush=True)


def graph_us(run, calls, reps=5, warm=3):
    """Capture `run` (which makes `calls` kernel calls) as one CUDA graph, replay it `warm` times untimed, then
    `reps` times between CUDA events on the current stream; the median time per call in microseconds."""
    g, _ = capture(run)
    for _ in range(warm):
        g.replay()
    st = torch.cuda.current_stream()
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        g.replay()
        b.record(st)
        b.synchronize()
        times.append(a.elapsed_time(b) * 1e3 / calls)
    del g
    return statistics.median(times)


def reference_kernels():
    """The reference's own extension (csrc/w4_gemv.cu), built unchanged for sm_100a into oracle/_ref/ -- the
    per-shape speed bar -- or None when it was not built."""
    try:
        from oracle import ref_kernel
        return ref_kernel.load() if ref_kernel.available() else None
    except Exception as ex:  # noqa: BLE001 - the bar is reported as missing, the bench still runs
        print(f"reference kernels unavailable: {ex}", file=sys.stderr)
        return None


MAX_COPIES = 8192   # calls per timed graph: tiny layers (the N = 1 tail: 66 bytes) would otherwise ask for millions


def cold_copies(k, n, device, seed, min_bytes=512 << 20):
    """Enough distinct packed weight + scale copies of an [n, k] layer (mma layout bytes, seeded) that cycling
    through them reads every call's weights from HBM -- at most MAX_COPIES, which bounds the graph of a tiny layer
    (whose copies then fit in L2: its time is the call's latency, not its bytes)."""
    b = n * k // 2 + 2 * n * (k // GROUP)
    copies = min(MAX_COPIES, max(4, -(-min_bytes // b)))
    gen = torch.Generator(device=device).manual_seed(seed)
    packed = torch.randint(0, 256, (copies, n, k // 2), dtype=torch.uint8, device=device, generator=gen)
    scales = (torch.rand(copies, n, k // GROUP, device=device, generator=gen) * 0.01 + 1e-3).half()
    return packed, scales, copies


def per_shape(ops, quant, device, peak, ref=None):
    """Each projection alone: one graph of calls over >= 512 MiB of distinct copies (4x L2), replayed 5 times;
    the median per-call time. A model keeps every layer's weights, so copies stand for the layers in between.
    `ref_us`: the reference's gemv_v6 (csrc/w4_gemv.cu:327-391) on the same copies, timed the same way."""
    rows = []
    seen = {}
    e = ops.ext()
    for model, proj, k, n in projections():
        if (k, n) in seen:
            rows.append(dict(seen[(k, n)], model=model, proj=proj))
            continue
        b = call_bytes(k, n)
        packed, scales, copies = cold_copies(k, n, device, k * 31 + n)
        x = torch.randn(1, k, device=device).half()
        y = torch.empty(copies, 1, n, dtype=torch.half, device=device)

        def run():
            for c in range(copies):   # direct C-ABI calls: no host work inside the graph
                rc = e.lib.lb_w4_gemv(x.data_ptr(), packed[c].data_ptr(), scales[c].data_ptr(), y[c].data_ptr(), 1,
                                      n, k, GROUP, 6, 0, torch.cuda.current_stream().cuda_stream)
                if rc:
                    raise RuntimeError(e.lib.lb_last_error().decode())
        us = graph_us(run, copies)
        row = {"model": model, "proj": proj, "K": k, "N": n, "bytes": b, "us": round(us, 3),
               "gbs": round(b / (us * 1e-6) / 1e9, 1), "frac": round(b / (us * 1e-6) / 1e9 / peak, 3),
               "copies": copies}
        if ref is not None:
            rus = graph_us(lambda: [ref.w4_gemv(x, packed[c], scales[c], GROUP, 6, 0) for c in range(copies)], copies)
            row["ref_us"] = round(rus, 3)
            row["speedup_vs_ref"] = round(rus / us, 2)
        seen[(k, n)] = row
        rows.append(row)
        del packed, scales, y
        torch.cuda.empty_cache()
    return rows


SKINNY_M = (2, 4, 8, 16, 32, 48, 64)
# the reference's tail shapes (K, N): N not a multiple of a tile, K of 128 / 256 / 384 (bench/gpu_run.py:31)
EDGE_SHAPES = ((128, 1), (256, 1001), (384, 37))
PREFILL_ROWS = (128, 256, 512, 1024)
PREFILL_SHAPES = ((2048, 11008), (11008, 2048), (1536, 8960))


def unique_shapes():
    out = []
    for _, _, k, n in projections():
        if (k, n) not in out:
            out.append((k, n))
    return out


def _abi(e, rc):
    if rc:
        raise RuntimeError(e.lib.lb_last_error().decode())


def skinny(ops, device, peak, ref=None, rows=SKINNY_M, shapes=None):
    """M in {2, ..., 64} over the config-1 shapes and the tail shapes, every call's weights cold
    (>= 256 MiB of copies, 2x L2). Per (shape, M): the kernel linear() picks (auto_version), the INT4 tensor-core
    kernel (version 5) whatever the rule picks, and in the same run the paths it replaces -- dequantize + cuBLAS
    (the fp16 weight written and read back each call) and cuBLAS on resident fp16 weights -- plus the reference's
    gemm_v5 (csrc/w4_gemv.cu:215-294) on the same copies (bench/gpu_run.py:250-301)."""
    from types import SimpleNamespace
    e = ops.ext()
    out = []
    for k, n in shapes or (unique_shapes() + list(EDGE_SHAPES)):
        progress(0, f"skinny K={k} N={n}")
        packed, scales, copies = cold_copies(k, n, device, 3 * k + n, min_bytes=256 << 20)
        c16 = min(MAX_COPIES, max(2, -(-(256 << 20) // (2 * n * k))))
        w16 = torch.empty(c16, n, k, dtype=torch.half, device=device)
        for c in range(c16):
            _abi(e, e.lib.lb_w4_dequant(packed[c].data_ptr(), scales[c].data_ptr(), w16[c].data_ptr(), n, k, GROUP, 2,
                                        torch.cuda.current_stream().cuda_stream))
        wbuf = torch.empty(n, k, dtype=torch.half, device=device)      # the dequantize path's fp16 weight
        proxy = SimpleNamespace(packed_mma=True, packed_v3=None, packed=None, n=n)
        for m in rows:
            x = torch.randn(m, k, device=device).half()
            y = torch.empty(max(copies, c16), m, n, dtype=torch.half, device=device)
            st = lambda: torch.cuda.current_stream().cuda_stream   # noqa: E731

            def int4(version):
                fn = e.lib.lb_w4_gemv if version == 6 else e.lib.lb_w4_gemm_tc
                extra = (6, 0) if version == 6 else (0,)
                return lambda: [_abi(e, fn(x.data_ptr(), packed[c].data_ptr(), scales[c].data_ptr(), y[c].data_ptr(),
                                          m, n, k, GROUP, *extra, st())) for c in range(copies)]

            def deq_cublas():
                for c in range(copies):
                    _abi(e, e.lib.lb_w4_dequant(packed[c].data_ptr(), scales[c].data_ptr(), wbuf.data_ptr(), n, k,
                                                GROUP, 2, st()))
                    torch.mm(x, wbuf.t(), out=y[c])
            path = ops.auto_version(m, proxy)
            arms = {}
            if m <= ops.MAX_ROWS[6]:
                arms[6] = graph_us(int4(6), copies)
            if m <= ops.MAX_ROWS[5]:
                arms[5] = graph_us(int4(5), copies)
            dq = graph_us(deq_cublas, copies)
            cb = graph_us(lambda: [torch.mm(x, w16[c].t(), out=y[c]) for c in range(c16)], c16)
            us = dq if path is None else arms[path]
            b = call_bytes(k, n, m)
            row = {"K": k, "N": n, "M": m, "path": {5: "v5 tensor-core", 6: "v6 GEMV", None: "dequant+cublas"}[path],
                   "us": round(us, 3), "gbs": round(b / (us * 1e-6) / 1e9, 1),
                   "frac": round(b / (us * 1e-6) / 1e9 / peak, 3)}
            row.update({f"v{v}_us": round(t, 3) for v, t in arms.items()})
            row.update({"dequant_cublas_us": round(dq, 3), "cublas_fp16_us": round(cb, 3),
                        "vs_dequant_cublas": round(dq / us, 2), "vs_cublas_fp16": round(cb / us, 2),
                        "tflops": round(2 * m * n * k / (us * 1e-6) / 1e12, 2)})
            if ref is not None and m <= 64:
                rus = graph_us(lambda: [ref.w4_gemm_tc(x, packed[c], scales[c], GROUP, 0) for c in range(copies)],
                               copies)
                row["ref_us"] = round(rus, 3)
                row["speedup_vs_ref"] = round(rus / us, 2)
            out.append(row)
            del y
        del packed, scales, w16, wbuf
        torch.cuda.empty_cache()
    return out


SWEEP_ROWS = (1, 2, 4, 8, 12, 16, 24, 32, 48, 64, 96, 128, 256)


def sweep_dispatch(out_path):
    """The record linear()'s dispatch table is derived from (lowbit/dispatch.py): every config-1 shape at M = 1..256,
    cold weights, version 6 / version 5 / dequantize + cuBLAS / fp16 cuBLAS per cell. Writes the record and prints
    the table it implies."""
    from lowbit import dispatch, ops
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    e = ops.ext()
    e.set_option("pdl", 1)
    e.set_option("early_weights", 1)
    peak, _ = measured_peak()
    t0 = time.time()
    cells = skinny(ops, device, peak, None, rows=SWEEP_ROWS, shapes=unique_shapes())
    table = dispatch.derive(cells)
    rec = {"device": torch.cuda.get_device_name(), "date": time.strftime("%Y-%m-%d"), "wide_n": 3072,
           "seconds": round(time.time() - t0), "table": table,
           "how": "bench.py --sweep-dispatch: per (shape, M) the per-call time with cold weights (>= 256 MiB of "
                  "copies, one CUDA graph per cell, median of 5 replays)", "cells": cells}
    pathlib.Path(out_path).write_text(json.dumps(rec, indent=1) + "\n")
    print(json.dumps(table))


def dequant_leg(ops, device, peak):
    """North-star subsystem 3, the prefill path: the dequantize kernel alone on every config-1 shape (bytes
    N*K/2 + N*K/64 read + 2*N*K written, cold copies), and at 128..1024 rows linear() -- dequantize + cuBLAS --
    against cuBLAS on resident fp16 weights (the reference's prefill table, results/RESULTS.md:97-108)."""
    e = ops.ext()
    kern = []
    for k, n in unique_shapes():
        packed, scales, copies = cold_copies(k, n, device, 5 * k + n, min_bytes=256 << 20)
        wbuf = torch.empty(2, n, k, dtype=torch.half, device=device)
        us = graph_us(lambda: [_abi(e, e.lib.lb_w4_dequant(packed[c].data_ptr(), scales[c].data_ptr(),
                                                           wbuf[c & 1].data_ptr(), n, k, GROUP, 2,
                                                           torch.cuda.current_stream().cuda_stream))
                               for c in range(copies)], copies)
        b = n * k // 2 + n * k // 64 + 2 * n * k
        kern.append({"K": k, "N": n, "bytes": b, "us": round(us, 3), "gbs": round(b / (us * 1e-6) / 1e9, 1),
                     "frac": round(b / (us * 1e-6) / 1e9 / peak, 3)})
        del packed, scales, wbuf
        torch.cuda.empty_cache()
    prefill = []
    for k, n in PREFILL_SHAPES:
        wq = ops.W4Weight.from_float(torch.randn(n, k, device=device) * 0.02, GROUP, ("mma",))
        w16 = ops.dequant(wq, "mma")
        for m in PREFILL_ROWS:
            x = torch.randn(m, k, device=device).half()
            lin = graph_us(lambda: [ops.linear(x, wq) for _ in range(8)], 8)
            cb = graph_us(lambda: [torch.nn.functional.linear(x, w16) for _ in range(8)], 8)
            prefill.append({"K": k, "N": n, "M": m, "dequant_cublas_us": round(lin, 2), "cublas_fp16_us": round(cb, 2),
                            "ratio": round(lin / cb, 3)})
        del wq, w16
        torch.cuda.empty_cache()
    return {"kernel": kern, "prefill": prefill,
            "note": "prefill rows: one weight, back-to-back calls (the fp16 weight of cuBLAS stays partly in L2, as in "
                    "a prefill that reuses it); kernel rows: cold copies"}


def run_ours(args, rank, world, local):
    from lowbit import ops, quant

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_dist(device) if world > 1 else None

    e = ops.ext()
    e.set_option("pdl", 1)
    e.set_option("early_weights", 1)   # the weights are static model state: fetch them before the wait
    peak, peak_src = measured_peak()
    projs = projections()
    step_bytes = sum(call_bytes(k, n) for _, _, k, n in projs)
    set_bytes = sum(n * k // 2 + 2 * n * (k // GROUP) for _, _, k, n in projs)
    n_sets = -(-ROTATION_BYTES // set_bytes)
    sets = build_sets(ops, quant, device, n_sets, seed=1234 + rank)
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    xs = [torch.randn(1, k, device=device, generator=gen).half() for _, _, k, _ in projs]

    # one graph per copy set (21 launches) and one graph over all sets (bulk replay: one host launch per
    # n_sets steps, so the timed region is never host-bound)
    def step_fn(layer):
        return lambda: [ops.linear(x, wq) for x, wq in zip(xs, layer)]
    set_graphs = [capture(step_fn(layer))[0] for layer in sets]
    all_graph, _ = capture(lambda: [ops.linear(x, wq) for layer in sets for x, wq in zip(xs, layer)])
    launches_per_step = len(projs)

    def run_steps(k0, count):
        i = 0
        while i < count:
            if (k0 + i) % n_sets == 0 and count - i >= n_sets:
                all_graph.replay()
                i += n_sets
            else:
                set_graphs[(k0 + i) % n_sets].replay()
                i += 1

    # up to four rotations, the timed steps are one graph of their own (steps warmup .. warmup + steps - 1 of the
    # rotation): a graph boundary breaks the programmatic-launch chain between two calls, so the timed region
    # should not have one per step
    timed = None
    if args.steps <= 4 * n_sets:
        timed, _ = capture(lambda: [ops.linear(x, wq) for i in range(args.steps)
                                    for x, wq in zip(xs, sets[(args.warmup + i) % n_sets])])

    st = torch.cuda.current_stream()
    run_steps(0, args.warmup)
    if timed is not None:
        timed.replay()   # warms the timed graph itself (untimed)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    with sampler:
        time.sleep(0.05)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        t_host0 = time.perf_counter()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(st)
        if timed is not None:
            timed.replay()
        else:
            run_steps(args.warmup, args.steps)
        ev1.record(st)
        ev1.synchronize()
        torch.cuda.synchronize()
        t_host1 = time.perf_counter()
        if dist:
            dist.barrier()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clocks = sampler.summary(t_host0, t_host1)
    value = world * step_bytes * args.steps / (ms * 1e-3) / 1e9
    ms_per_step = ms / args.steps

    # the timed region lasts about a millisecond, under NVML's sampling period: the same rotation replayed for
    # ~0.4 s afterwards (not part of `value`) gives the clock record under sustained load and a cross-check of
    # the rate
    reps = max(1, min(4096, int(400.0 / max(ms_per_step * n_sets, 1e-3))))
    sustained = ClockSampler(local)
    with sustained:
        ts0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            all_graph.replay()
        e1.record(st)
        e1.synchronize()
        ts1 = time.perf_counter()
    s_ms = e0.elapsed_time(e1)
    if sustained.ok:
        clocks["sustained"] = {k: v for k, v in sustained.summary(ts0, ts1).items() if k != "source"}
        clocks["sustained"].update({"seconds": round(s_ms / 1e3, 3),
                                    "gbs": round(step_bytes * n_sets * reps / (s_ms * 1e-3) / 1e9, 1),
                                    "how": "the step rotation replayed back to back after the timed region, "
                                           "this rank's GB/s"})

    # e2e: the public API (lowbit.ops.linear), eager, from pinned host memory and back every step: one host-to-
    # device copy of the step's 21 activation rows, the 21 calls writing into one device buffer, one copy of the 21
    # outputs back to the host, then a synchronize
    ks, ns = [k for _, _, k, _ in projs], [n for _, _, _, n in projs]
    x_host = torch.cat([x.reshape(-1).cpu() for x in xs]).pin_memory()
    y_host = torch.empty(sum(ns), dtype=torch.half).pin_memory()
    x_dev = torch.empty(sum(ks), dtype=torch.half, device=device)
    y_dev = torch.empty(sum(ns), dtype=torch.half, device=device)
    x_views = [x_dev[a:a + k].view(1, k) for a, k in zip(itertools.accumulate([0] + ks[:-1]), ks)]
    y_views = [y_dev[a:a + n].view(1, n) for a, n in zip(itertools.accumulate([0] + ns[:-1]), ns)]
    h2d, d2h = x_host.numel() * 2, y_host.numel() * 2
    e2e_steps = max(3, min(args.steps, 200))

    def e2e_step(layer):
        x_dev.copy_(x_host, non_blocking=True)
        for xv, yv, wq in zip(x_views, y_views, layer):
            ops.linear(xv, wq, out=yv)
        y_host.copy_(y_dev, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    for i in range(3):
        e2e_step(sets[i % n_sets])
    if dist:
        dist.barrier()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(st)
    for i in range(e2e_steps):
        e2e_step(sets[i % n_sets])
    eb.record(st)
    eb.synchronize()
    e2e_ms = ea.elapsed_time(eb)
    if dist:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_val = world * step_bytes * e2e_steps / (e2e_ms * 1e-3) / 1e9

    # e2e_graph: the step as a decode loop runs it -- the pinned-host input copy, the same public calls and the
    # copy of the outputs back to pinned host memory captured once per weight set in a CUDA graph -- replayed every
    # step, then a synchronize
    def eg_body(layer):
        x_dev.copy_(x_host, non_blocking=True)
        for xv, yv, wq in zip(x_views, y_views, layer):
            ops.linear(xv, wq, out=yv)
        y_host.copy_(y_dev, non_blocking=True)
    eg = [capture(lambda layer=layer: eg_body(layer))[0] for layer in sets]

    def eg_step(i):
        eg[i % n_sets].replay()
        torch.cuda.current_stream().synchronize()
    for i in range(3):
        eg_step(i)
    if dist:
        dist.barrier()
    ea.record(st)
    for i in range(e2e_steps):
        eg_step(i)
    eb.record(st)
    eb.synchronize()
    eg_ms = ea.elapsed_time(eb)
    if dist:
        t = torch.tensor([eg_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        eg_ms = float(t.item())
    e2e_graph_val = world * step_bytes * e2e_steps / (eg_ms * 1e-3) / 1e9
    del eg

    # the other configurations, measured after the timed sweep in the same run: the single-GPU kernel legs
    # (per-shape M = 1, config 2, prefill dequantize) at one GPU; the decoders at every N (config 3 as replicas,
    # config 4 sharded over all ranks)
    del set_graphs, all_graph, timed
    sets = None
    torch.cuda.empty_cache()
    extras = {}
    ref = reference_kernels() if world == 1 else None
    if world == 1 and not args.no_per_shape:
        progress(rank, "per_shape")
        extras["per_shape"] = per_shape(ops, quant, device, peak, ref)
    if world == 1 and not args.no_skinny:
        progress(rank, "skinny")
        extras["skinny"] = skinny(ops, device, peak, ref)
    if world == 1 and not args.no_dequant:
        progress(rank, "dequant")
        extras["dequant"] = dequant_leg(ops, device, peak)
    if not args.no_decode:
        progress(rank, "decode_3b")
        extras["decode_3b"] = decode_summary(run_decode(args, rank, world, local, dist, steps=128, warm=16))
        progress(rank, "tp_decode")
        extras["tp_decode"] = decode_summary(run_tp_decode(args, rank, world, local, dist, steps=128, warm=16))
    progress(rank, "legs done")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(budget_s=args.cpu_seconds)

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    achieved = step_bytes / (ms_per_step * 1e-3) / 1e9 / 1.0
    traffic = profiled_traffic()
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16 activations x int4 weights, fp32 accumulate",
        "data": "synthetic: seeded N(0, 0.02) weights quantized by lowbit's format, N(0, 1) activations",
        "config": {
            "workload": "BASELINE config 1: M=1 GEMV over every q/k/v/o/gate/up/down projection of Qwen2.5-0.5B, "
                        "1.5B and 3B (21 calls per step), group 128, mma layout",
            "M": 1, "calls_per_step": launches_per_step, "bytes_per_step": step_bytes,
            "l2": f"cold weights: rotating {n_sets} copy sets = {n_sets * set_bytes / 1e9:.2f} GB "
                  f"({n_sets * set_bytes / L2_BYTES:.1f}x L2)",
            "timing": "CUDA graphs (the timed steps one graph of their own up to 60 steps; one launch per call, "
                      "programmatic dependent launch, early weight fetch), "
                      "CUDA events on the launching stream, max over ranks",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
        },
        "roofline": {
            "bound": "hbm", "kernel": "gemv_tile_kernel (M=1 decode GEMV)",
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "algorithmic_bytes_per_launch": round(step_bytes / launches_per_step),
            "frac": round(achieved / peak, 4), "peak_source": peak_src,
            "traffic": traffic,
            "note": "achieved = algorithmic bytes per launch / average launch duration over the timed region "
                    "(every launch in the step is this kernel)",
        },
        "clocks": clocks,
        "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps,
                "how": "lowbit.ops.linear eager per call (out= slices of one device buffer); the step's 21 "
                       "activation rows pinned-host -> GPU in one copy and its 21 outputs -> pinned host in one "
                       "copy inside the timed region; stream synchronized at the end of each step"},
        "e2e_graph": {"value": round(e2e_graph_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                      "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                      "how": "the step captured once per weight set in a CUDA graph, as a decode loop captures "
                             "its step: the pinned-host copy of the 21 activation rows, the same 21 "
                             "lowbit.ops.linear calls, the copy of the 21 outputs to pinned host memory; each step "
                             "replays the graph (both copies included) and synchronizes the stream"},
        "gpu_launches": launches_per_step * args.steps,
    }
    line.update({k: v for k, v in extras.items() if v is not None})
    if ref is None and world == 1:
        line["reference_kernels"] = "unavailable: oracle/_ref was not built (no reference checkout at build time)"
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def decode_summary(line):
    """The sub-record of a decoder run (configs 3 and 4) inside the headline line (rank 0; None elsewhere)."""
    if line is None:
        return None
    rf = line["roofline"]
    return {"metric": line["metric"], "value": line["value"], "unit": line["unit"], "n_gpus": line["n_gpus"],
            "ms_per_token": line["ms_per_step"], "steps": line["steps"], "warmup": line["warmup"],
            "scaling": line["scaling"], "parallelism": line["config"]["parallelism"], "fuse": line["config"]["fuse"],
            "roofline": {k: rf[k] for k in rf if k != "traffic"}, "e2e": line["e2e"], "clocks": line["clocks"],
            "gpu_launches": line["gpu_launches"]}


# ------------------------------------------------------------------------------------------------ CPU arm

def cpu_sweep_inputs(seed=0):
    """The same workload on the host: the 21 projections, packed canonical weights + scales (CPU tensors)."""
    from lowbit import quant
    g = torch.Generator().manual_seed(seed)
    out = []
    for _, _, k, n in projections():
        # the GPU arm's weights: N(0, 0.02), quantized to the lowbit format (absmax, group 128)
        packed, scales = quant.quantize_w4((torch.randn(n, k, generator=g) * 0.02).numpy(), GROUP)
        x = torch.randn(1, k, generator=g).half()
        out.append((x, torch.from_numpy(packed), torch.from_numpy(scales), k, n))
    return out


def cpu_pass(inputs):
    from oracle import oracle
    done = 0
    for x, packed, scales, k, n in inputs:
        y = oracle.torch_linear(x, packed, scales, GROUP)
        assert y.shape == (1, n)
        done += call_bytes(k, n)
    return done


def cpu_baseline(budget_s=10.0):
    """The reference's CPU path timed on this host's cores: a bounded sample of the workload (whole sweep
    passes until `budget_s` has elapsed, at least one)."""
    from oracle import oracle
    threads = oracle.cpu_threads()
    torch.set_num_threads(threads)
    inputs = cpu_sweep_inputs()
    cpu_pass(inputs[:3])                                     # warm-up (thread pool, allocator)
    t0 = time.perf_counter()
    done, passes = 0, 0
    while passes == 0 or time.perf_counter() - t0 < budget_s:
        done += cpu_pass(inputs)
        passes += 1
    dt = time.perf_counter() - t0
    return {"value": round(done / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{passes} full sweep pass(es) of the 21 projections (M=1) in {dt:.1f} s: "
                      "oracle.torch_linear = lowbit/ops.py:119-123 dequantize on CPU tensors + fp32 F.linear",
            "cpu": platform_cpu()}


def platform_cpu():
    try:
        for line in pathlib.Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args, rank, world):
    """--impl reference: the reference's own CPU implementation (restated in oracle/, the reference ships no
    compiled CPU code and has no installable package) on this host's cores, same metric and config."""
    if rank != 0:
        return None
    from oracle import oracle
    threads = oracle.cpu_threads()
    torch.set_num_threads(threads)
    inputs = cpu_sweep_inputs()
    for _ in range(args.warmup):
        cpu_pass(inputs)
    steps = args.steps if args.steps <= 50 else 50
    t0 = time.perf_counter()
    done = 0
    for _ in range(steps):
        done += cpu_pass(inputs)
    dt = time.perf_counter() - t0
    val = done / dt / 1e9
    step_bytes = sum(call_bytes(k, n) for _, _, k, n in projections())
    return {
        "impl": "reference",
        "metric": METRIC, "value": round(val, 4), "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(dt / steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (dequantize to fp16, fp32 matmul)",
        "data": "synthetic: seeded N(0, 0.02) weights quantized by lowbit's format, N(0, 1) activations",
        "config": {"workload": "BASELINE config 1 on the host: the 21 Qwen2.5 projections, M=1", "M": 1,
                   "bytes_per_step": step_bytes, "parallelism": "host cores, rank 0 only"},
        "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{steps} sweep pass(es); steps capped at 50 to bound the run",
                         "cpu": platform_cpu()},
        "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def profile_case(k, n, m, copies=8, calls=6):
    """A handful of cold calls of one shape (8 distinct weight copies, each > L2 / 8 for the large layers) for
    `ncu -k regex:gemv -s 2 -c 3`: small enough that a --set full capture ends in about a minute."""
    from lowbit import ops
    torch.cuda.set_device(0)
    ops.ext().set_option("early_weights", 1)
    wqs = [ops.W4Weight.from_float(torch.randn(n, k, device="cuda") * 0.02, GROUP, ("mma",)) for _ in range(copies)]
    x = torch.randn(m, k, device="cuda").half()
    for i in range(calls):
        ops.linear(x, wqs[i % copies])
    torch.cuda.synchronize()
    print(f"profile case K={k} N={n} M={m}: {calls} calls done", file=sys.stderr)


# ------------------------------------------------------------------------------------------------ config 3

DECODE_CONTEXT = 512


def init_dist(device, timeout_s=600):
    """The NCCL process group of a torchrun job (one rank per GPU), with a bounded timeout."""
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=device)
    return dist


def run_decode(args, rank, world, local, dist=None, steps=None, warm=None):
    """Config 3: random-init Qwen2.5-3B architecture, all 252 projections INT4 group-128, batch-1 greedy decode with
    one CUDA graph per step (embedding -> 36 layers -> tied fp16 lm_head -> argmax) after a 512-token prompt of
    ids uniform over the vocabulary. value = tokens/s on the device; e2e also reads every token back to the host,
    as a streaming generator does. N > 1: independent replicas (the model fits one GPU; config 4 is the sharded
    one). `dist`: an initialized torch.distributed module (None: this call makes and ends its own group)."""
    from lowbit import decode

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    own = dist is None and world > 1
    if own:
        dist = init_dist(device)
    decode.enable_decode_options()
    steps = steps or min(args.steps, 256)
    warm = warm or min(args.warmup, 64)
    fuse = fuse_arg(args, 3)
    m = decode.build(decode.QWEN25_3B, seed=rank)
    dec = decode.Int4Decoder(m, DECODE_CONTEXT + warm + 2 * steps + 16, fuse=fuse)
    del m
    torch.cuda.empty_cache()
    int4_bytes = dec.int4_bytes
    gen = torch.Generator().manual_seed(7 + rank)
    prompt = torch.randint(0, decode.QWEN25_3B["vocab_size"], (DECODE_CONTEXT,), generator=gen)
    dec.prefill(prompt)
    for _ in range(warm):
        dec.step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        a.record(st)
        for _ in range(steps):
            dec.step()
        b.record(st)
        b.synchronize()
        t1 = time.perf_counter()
    ms = a.elapsed_time(b)
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    tok_s = steps / (ms / 1e3)
    # e2e: every step's token read back into pinned host memory before the next step is launched
    host = torch.empty(1, 1, dtype=torch.long, pin_memory=True)
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    for _ in range(steps):
        dec.step()
        host.copy_(dec.tok, non_blocking=True)
        st.synchronize()
    e2e_s = time.perf_counter() - t2
    ctx_mid = DECODE_CONTEXT + warm + steps // 2
    per_tok = int4_bytes + dec.head_bytes() + dec.kv_bytes(ctx_mid)
    peak, peak_src = measured_peak()
    achieved = per_tok * tok_s / 1e9
    line = {
        "metric": "Qwen2.5-3B decode tokens/s (batch 1, greedy, one CUDA graph per step, 512-token context)",
        "value": round(tok_s * world, 2), "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": round(ms / steps, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4 weights x fp16 activations, fp32 accumulate",
        "data": "synthetic: random-init weights (N(0, 0.02)), prompt ids uniform over the vocabulary",
        "config": {"workload": "config 3: Qwen2.5-3B architecture, 36 layers, 252 INT4 projections, tied fp16 lm_head",
                   "model": "Qwen2.5-3B (random init)", "global_batch": world, "seq_len": DECODE_CONTEXT,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "weights 2 GB per token >> 126 MB L2", "fuse": list(fuse)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_src,
                     "algorithmic_bytes_per_token": per_tok,
                     "bytes": "INT4 projections + fp16 lm_head + KV cache at the mean context"},
        "e2e": {"value": round(steps / e2e_s * world, 2), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 8, "note": "token read back to pinned host memory after every step"},
        "clocks": clk.summary(t0, t1),
        "gpu_launches": dec.launches_per_step() * steps,
        "cpu_baseline": None,
    }
    if dist:
        dist.barrier()
    dec.graph = None
    del dec
    torch.cuda.empty_cache()
    if own:
        dist.destroy_process_group()
    return line if rank == 0 else None


# ------------------------------------------------------------------------------------------------ config 4

TP_CONTEXT = 1024


def run_tp_decode(args, rank, world, local, dist=None, steps=None, warm=None):
    """Config 4: random-init Qwen2.5-7B architecture, INT4 group-128, tensor-parallel over the torchrun ranks
    (column-parallel q|k|v and gate|up, row-parallel o and down + allreduce, vocabulary-parallel lm_head),
    batch-1 greedy decode with one CUDA graph per step after a 1024-token prompt. value = tokens/s of the whole
    job (strong scaling: the same model split over more GPUs), timed on the device, max over ranks. At one GPU the
    unsharded model. `dist`: an initialized torch.distributed module (None: this call makes and ends its own)."""
    from lowbit import decode

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    own = dist is None and world > 1
    if own:
        dist = init_dist(device)
    decode.enable_decode_options()
    steps = steps or min(args.steps, 256)
    warm = warm or min(args.warmup, 64)
    fuse = fuse_arg(args, 4, world)
    allreduce = getattr(args, "allreduce", "oneshot")
    m = decode.build(decode.QWEN25_7B, seed=0, device=device)
    dec = decode.Int4Decoder(m, TP_CONTEXT + warm + steps + 16, world=world, rank=rank,
                             pg=dist.group.WORLD if dist else None, allreduce=allreduce, fuse=fuse)
    del m
    torch.cuda.empty_cache()
    gen = torch.Generator().manual_seed(7)
    prompt = torch.randint(0, decode.QWEN25_7B["vocab_size"], (TP_CONTEXT,), generator=gen)
    dec.prefill(prompt)
    for _ in range(warm):
        dec.step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        a.record(st)
        for _ in range(steps):
            dec.step()
        b.record(st)
        b.synchronize()
        t1 = time.perf_counter()
    ms = a.elapsed_time(b)
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    tok_s = steps / (ms / 1e3)
    ctx_mid = TP_CONTEXT + warm + steps // 2
    per_rank = dec.int4_bytes + dec.head_bytes() + dec.kv_bytes(ctx_mid)
    peak, peak_src = measured_peak()
    achieved = per_rank * tok_s / 1e9       # one rank's HBM traffic rate; every rank reads its own shard
    line = {
        "metric": "Qwen2.5-7B tensor-parallel decode tokens/s (batch 1, greedy, one CUDA graph per step, 1024-token context)",
        "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": round(ms / steps, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 weights x fp16 activations, fp32 accumulate",
        "data": "synthetic: random-init weights (N(0, 0.02)), prompt ids uniform over the vocabulary",
        "config": {"workload": "config 4: Qwen2.5-7B architecture, 28 layers, INT4 group-128, untied fp16 lm_head",
                   "model": "Qwen2.5-7B (random init)", "global_batch": 1, "seq_len": TP_CONTEXT,
                   "parallelism": (f"tp{world}: column q|k|v, gate|up; row o, down + "
                                   f"{'one-shot peer-memory' if allreduce == 'oneshot' else 'NCCL'} allreduce; "
                                   "vocab lm_head") if world > 1 else "single GPU (unsharded)",
                   "fuse": list(fuse)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_src,
                     "algorithmic_bytes_per_token_per_rank": per_rank,
                     "bytes": "this rank's INT4 shard + fp16 lm_head rows + KV cache at the mean context"},
        "e2e": None,
        "clocks": clk.summary(t0, t1),
        "gpu_launches": dec.launches_per_step() * steps,
        "cpu_baseline": None,
    }
    if dist:
        dist.barrier()
    dec.graph = None
    del dec
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if own:
        dist.destroy_process_group()
    return line if rank == 0 else None


def profile_sweep(passes=2):
    """No timing: `passes` eager passes over the 21 config-1 projections, each pass on its own weight set (cold:
    15 sets rotate as in the benchmark), for an ncu capture of one whole step's launches (-s 21 -c 21)."""
    from lowbit import ops, quant
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    e = ops.ext()
    e.set_option("pdl", 1)
    e.set_option("early_weights", 1)
    projs = projections()
    set_bytes = sum(n * k // 2 + 2 * n * (k // GROUP) for _, _, k, n in projs)
    sets = build_sets(ops, quant, device, -(-ROTATION_BYTES // set_bytes), seed=1234)
    gen = torch.Generator(device=device).manual_seed(99)
    xs = [torch.randn(1, k, device=device, generator=gen).half() for _, _, k, _ in projs]
    for p in range(passes):
        for x, wq in zip(xs, sets[p % len(sets)]):
            ops.linear(x, wq)
    torch.cuda.synchronize()
    print(f"profile sweep: {passes} passes x {len(projs)} calls", file=sys.stderr)


# measured defaults (B200): config 3 runs fastest with the separate kernels; config 4 with the o and down GEMVs
# fused with their allreduce, residual add and RMSNorm (TP2 488 tok/s against 474 for GEMV then allreduce + norm)
DEFAULT_FUSE = {3: "", 4: "epilogue"}
# config 4 at two ranks: the o and down GEMVs also fused with their allreduce (measured at TP2: 610 against 543
# tok/s); at eight the fused kernel's last CTA, polling every rank's region, made the step slower than separate
# GEMV + one-shot allreduce kernels (3121 against 1921 us per token, `--tp-timeline`)
DEFAULT_FUSE_TP2 = "epilogue,gemv_allreduce"


def fuse_arg(args, config=None, world=1):
    """--fuse: comma-separated kernel fusions of the decode step (Int4Decoder's `fuse`); the config's measured
    default at this world size when not given."""
    f = getattr(args, "fuse", None)
    if f is None:
        cfg = config or getattr(args, "config", 3)
        f = DEFAULT_FUSE_TP2 if cfg == 4 and world == 2 else DEFAULT_FUSE.get(cfg, "")
    return tuple(x for x in f.split(",") if x)


def tp_timeline(args, rank, world, local, steps=16):
    """No headline: where the time of one config-4 decode step goes at this world size. The step graph is replayed
    `steps` times under torch's CUPTI profiler on every rank; rank 0 prints one JSON line with each kernel's GPU
    time per step and share, plus the graph-timed step. A kernel that waits on its peers (the fused GEMV +
    allreduce, the one-shot allreduce, NCCL) is charged its waiting time, so the table names the collective or
    kernel that bounds the tensor-parallel step. Kernels overlap under programmatic dependent launch, so the
    per-kernel times add up to more than the step."""
    from torch.profiler import ProfilerActivity, profile
    from lowbit import decode
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_dist(device) if world > 1 else None
    decode.enable_decode_options()
    allreduce = getattr(args, "allreduce", "oneshot")
    m = decode.build(decode.QWEN25_7B, seed=0, device=device)
    dec = decode.Int4Decoder(m, TP_CONTEXT + 3 * steps + 16, world=world, rank=rank,
                             pg=dist.group.WORLD if dist else None, allreduce=allreduce, fuse=fuse_arg(args, 4, world))
    del m
    torch.cuda.empty_cache()
    prompt = torch.randint(0, decode.QWEN25_7B["vocab_size"], (TP_CONTEXT,), generator=torch.Generator().manual_seed(7))
    dec.prefill(prompt)
    for _ in range(steps):
        dec.step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        dec.step()
    b.record()
    b.synchronize()
    step_us = a.elapsed_time(b) * 1e3 / steps
    if dist:
        dist.barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            dec.step()
        torch.cuda.synchronize()
    kern = {}
    for ev in prof.key_averages():
        if ev.device_type == torch.autograd.DeviceType.CUDA and ev.count:
            k = kern.setdefault(ev.key[:90], [0, 0.0])
            k[0] += ev.count
            k[1] += ev.device_time_total
    total = sum(v[1] for v in kern.values()) or 1.0
    rows = sorted(kern.items(), key=lambda kv: -kv[1][1])
    line = {"tp_timeline": world, "fuse": list(fuse_arg(args, 4, world)), "allreduce": allreduce,
            "step_us_graph": round(step_us, 1), "kernel_us_per_step": round(total / steps, 1),
            "kernels": [{"kernel": k, "launches_per_step": round(c / steps, 2), "us_per_step": round(t / steps, 1),
                         "share": round(t / total, 3)} for k, (c, t) in rows[:25]]}
    if dist:
        dist.barrier()
        del dec
        dist.destroy_process_group()
    return line if rank == 0 else None


def profile_decode(fuse=(), steps=3, prompt_len=8):
    """No timing: the config-3 decoder (Qwen2.5-3B, INT4) with a short prompt, then a few graph steps, for an ncu
    launch list of whole decode steps."""
    from lowbit import decode
    torch.cuda.set_device(0)
    decode.enable_decode_options()
    dec = decode.Int4Decoder(decode.build(decode.QWEN25_3B, seed=0), 64, fuse=fuse)
    dec.prefill(torch.arange(prompt_len) * 9973 % 151936)
    for _ in range(steps):
        dec.step()
    torch.cuda.synchronize()
    print(f"profile decode: {dec.launches_per_step()} library launches per step", file=sys.stderr)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30000)
    ap.add_argument("--warmup", type=int, default=1500)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, choices=(1, 3, 4), default=1,
                    help="1: M=1 GEMV sweep over the Qwen2.5 projections (headline); 3: Qwen2.5-3B decode tok/s; "
                         "4: Qwen2.5-7B tensor-parallel decode tok/s over the torchrun ranks")
    ap.add_argument("--no-per-shape", action="store_true")
    ap.add_argument("--no-skinny", action="store_true", help="skip the config-2 sweep (M = 2..64)")
    ap.add_argument("--no-dequant", action="store_true", help="skip the prefill dequantize leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-3 and config-4 decoder legs")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--allreduce", choices=("oneshot", "nccl"), default="oneshot",
                    help="config 4: row-parallel sums by the library's one-shot kernel or by NCCL")
    ap.add_argument("--fuse", default=None,
                    help="configs 3, 4: decode-step fusions, comma-separated: epilogue (norms and SwiGLU in the "
                         "GEMV / allreduce epilogues), gemv_allreduce (config 4: o and down GEMVs fused with their "
                         "allreduce) or any of qkv, gu, down (GEMV prologues); --fuse= for none")
    ap.add_argument("--sweep-dispatch", default=None, metavar="OUT.json",
                    help="sweep the config-1 shapes at M = 1..256 and write the record the dispatch table follows from")
    ap.add_argument("--profile-decode", action="store_true", help="no timing: a few config-3 decode steps, for ncu")
    ap.add_argument("--profile-sweep", action="store_true", help="no timing: two cold passes over the config-1 calls")
    ap.add_argument("--tp-timeline", action="store_true",
                    help="no headline: per-kernel GPU time of one config-4 decode step at this world size (CUPTI)")
    ap.add_argument("--profile-case", default=None, metavar="K,N,M",
                    help="no timing: a few launches of one GEMV shape, for a small ncu capture")
    args = ap.parse_args()
    if args.sweep_dispatch:
        sweep_dispatch(args.sweep_dispatch)
        return
    if args.profile_decode:
        profile_decode(fuse_arg(args))
        return
    if args.profile_sweep:
        profile_sweep()
        return
    if args.profile_case:
        profile_case(*(int(v) for v in args.profile_case.split(",")))
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, local = rank_env()
    if world != args.gpus and world > 1:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    if args.tp_timeline:
        line = tp_timeline(args, rank, world, local)
    elif args.impl == "reference":
        line = run_reference(args, rank, world)
    elif args.config == 3:
        line = run_decode(args, rank, world, local)
    elif args.config == 4:
        line = run_tp_decode(args, rank, world, local)
    else:
        line = run_ours(args, rank, world, local)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
