"""Benchmark of the B200 attention backend (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

A step is one forward pass of the hot path over one batch of the workload's
seeded synthetic inputs (shapes, seeds and value distributions of the
portable-attention benchmark configurations, ``pa_b200.workloads``). The
default workload is the fp16 causal grouped-query prefill forward, q
(8, 32, 4096, 128), k/v (8, 8, 4096, 128): its inputs (512 MiB) exceed the
126 MB L2, so no flush is needed between iterations.

* ``value``: whole-job TFLOP/s (or GB/s for decode) with inputs resident in
  HBM, timed with CUDA events on the launching stream over exactly K steps,
  max over ranks.
* ``e2e``: the same metric through the public SdpaBackend call on NumPy arrays
  in page-locked host memory, host->device and device->host copies included;
  ``e2e.pageable`` is the same call on ordinary NumPy arrays.
* ``roofline``: the dominant kernel's algorithmic FLOPs (bytes) per launch
  over its average CUDA-event launch time, against MEASURED_PEAKS.json (the
  fp32 workload against the theoretical FFMA rate: no measured fp32 peak).
* ``workloads`` (default workload only): device-timed lines for the other
  benchmark configurations -- fp32 exact forward, masked cross-attention,
  split-KV decode and long-context forward + backward at N = 1; the decode
  with its batch split over the ranks at N > 1.
* ``cpu_baseline``: the reference's own ``fused`` CPU backend (byte-compiled
  by ``oracle/build_ref.py``; the oracle's restatement, labelled ``port``,
  only when that is missing) on a bounded sample of the same workload, all
  host threads, BLAS pinned to one thread per worker, plus ``fused`` and
  ``reference`` on one item at default BLAS threads and at one (rank 0, N=1).

Multi-GPU (torchrun): the one global problem is cut into N parts (batch rows,
or whole grouped-query KV-head groups), one per rank, with no data-path
collective (strong scaling); torch.distributed provides the barrier and the
max-over-ranks timing. ``ring`` adds the long-context forward + backward as
ring attention over the same ranks, with a per-phase split of one profiled
step.

``--impl reference`` times the reference's CPU ``fused`` backend the same way
on the box's host cores, a bounded sample per step.

KV-cache decode workloads (``--workload kv_fp8_decode_gqa``,
``kv_paged_decode_gqa``, ``kv_paged_fp8_decode_gqa``) run the decode shapes
(q (64, 32, 1, 128), caches for 64 sequences x 8 KV heads x 32768 keys) from
an fp8 e4m3 cache and/or a paged cache (16-key pages in a seeded random
order). ``value`` is GB/s of the bytes the kernel must read (cache in its
storage type, block table, q) and write (out); ``e2e`` is a serving step:
the query copied in from page-locked memory, the decode on the resident
cache, the output copied back.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "portable-attention_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "SDPA TFLOP/s (fwd, fwd+bwd) at 1/2/4/8 B200; decode HBM GB/s; %peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def clock_log(args, rank: int, tag: str = "") -> Path:
    """CSV file for this rank's nvidia-smi clock samples.

    ``--clock-dir`` when given; otherwise a fresh private folder per run and
    rank (``tempfile.mkdtemp``), so concurrent runs never share a file.
    """
    if args.clock_dir:
        out_dir = Path(args.clock_dir)
        out_dir.mkdir(parents=True, exist_ok=True)
    else:
        out_dir = Path(tempfile.mkdtemp(prefix=f"pa_b200_bench_r{rank}_"))
    return out_dir / f"clocks{tag}_rank{rank}.csv"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples (every 20 ms, to a file) around the timed region.

    Sampling starts before warm-up (nvidia-smi takes a moment to start) and
    :meth:`mark` brackets the timed region; the summary keeps the samples
    inside it, or the nearest ones when the region is shorter than a period.
    """

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, path: Path):
        self.index = index
        self.path = path
        self.proc = None
        self.window = [None, None]

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20", "-f", str(self.path)],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def mark(self, which: int):
        self.window[which] = time.time()

    def stop(self):
        if self.proc is not None:
            time.sleep(0.05)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        import datetime

        rows = []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        try:
            text = self.path.read_text()
        except OSError:
            text = ""
        for line in text.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]), float(parts[4]),
                             [n for n, v in zip(names, parts[6:10]) if v.lower() == "active"]))
            except ValueError:
                continue
        t0, t1 = self.window
        inside = [r for r in rows if t0 is not None and t0 - 0.02 <= r[0] <= (t1 or t0) + 0.02]
        how = "inside timed region"
        if not inside and rows and t0 is not None:
            inside = sorted(rows, key=lambda r: abs(r[0] - t0))[:3]
            how = "nearest samples (timed region shorter than the 20 ms period)"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": inside[0][2],
                "power_w_max": max(r[3] for r in inside),
                "reasons": sorted({n for r in inside for n in r[4]}), "samples": len(inside),
                "window": how}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    pg = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    return rank, local, world, pg


def barrier(pg):
    if pg is not None:
        pg.barrier()


def sum_over_ranks(pg, value: float, local: int) -> float:
    if pg is None:
        return value
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=f"cuda:{local}")
    pg.all_reduce(t, op=pg.ReduceOp.SUM)
    return float(t.item())


def max_over_ranks(pg, value: float, local: int) -> float:
    if pg is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=f"cuda:{local}")
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- CPU leg

def cpu_backends():
    """The reference's CPU backends: ``(fused, reference, benchmark module, kind)``.

    The real package (byte-compiled into ``oracle/_ref`` by
    ``oracle/build_ref.py``, or ``$PA_REFERENCE_SRC``) when it imports; else the
    oracle's restatement of the same two algorithms, labelled ``port``.
    """
    from oracle import build_ref

    pa = build_ref.import_reference()
    if pa is not None:
        from portable_attention import benchmark as bm

        return pa.get_backend("fused"), pa.get_backend("reference"), bm, "reference"
    from oracle.sdpa import fused_sdpa, reference_sdpa

    return fused_sdpa, reference_sdpa, None, "port"


def cpu_jobs(name, x=None):
    """Work items of the workload for the CPU backends: ``([(args, kwargs, work)], what)``.

    Items are whole (batch, head) slices, except for decode (whole batch rows)
    and the 131072-long causal workload (64-row query blocks against the keys
    they see, with the causal mask as an explicit boolean slice); the
    reference has no backward, so that baseline is forward-only.
    """
    from pa_b200 import workloads

    w = workloads.WORKLOADS[name]
    threads = os.cpu_count() or 1
    group = w.q_shape[1] // w.kv_shape[1]
    D = w.q_shape[3]
    if name == "fp16_decode_gqa":
        gen = np.random.default_rng(3)
        q = (gen.standard_normal((1, w.q_shape[1], 1, D)) * 0.5).astype(np.float16)
        kv = [(gen.standard_normal((1, w.kv_shape[1], w.kv_shape[2], D)) * 0.5).astype(np.float16)
              for _ in range(2)]
        jobs = [((q, kv[0], kv[1]), {"enable_gqa": True}, 2 * kv[0].nbytes)] * max(threads, 8)
        return jobs, "batch rows of q (1,32,1,128) vs k/v (1,8,32768,128)"
    if name == "fp16_long_causal":
        if x is None:
            x = workloads.make(name)
        jobs = []
        rng = np.random.default_rng(0)
        for r0 in sorted(rng.integers(0, x["q"].shape[2] // 64, size=4 * threads) * 64):
            h = int(rng.integers(0, x["q"].shape[1]))
            rows = np.arange(r0, r0 + 64)
            keys = r0 + 64
            m = np.arange(keys)[None, :] <= rows[:, None]
            jobs.append(((x["q"][0, h, r0:r0 + 64], x["k"][0, h, :keys], x["v"][0, h, :keys]),
                         {"attn_mask": m}, 4.0 * D * float(np.sum(rows + 1))))
        return jobs, "64-row query blocks (random heads/offsets) vs their visible keys, forward only"
    if x is None:
        x = workloads.make(name, batch_rows=slice(0, 1))
    L, S = w.q_shape[2], w.kv_shape[2]
    unit = 4.0 * L * S * D * (0.5 if w.is_causal else 1.0)
    jobs = []
    for h in range(w.q_shape[1]):
        kw = {"is_causal": True} if w.is_causal else {}
        if w.masked:
            kw["attn_mask"] = x["mask"][0, 0]
        jobs.append(((x["q"][0, h], x["k"][0, h // group], x["v"][0, h // group]), kw, unit))
    return jobs, "(b,h) slices of the workload"


def cpu_sample(name, budget_s=12.0, x=None):
    """Time the reference's ``fused`` CPU backend on a bounded sample of the workload.

    Returns (rate in the metric's unit, threads, description, kind). Work
    items run in a thread pool, one per host core (NumPy releases the GIL in
    its GEMMs), each with BLAS pinned to one thread -- the ``fused`` backend's
    own policy (``fused.py``: one BLAS thread for the compute region), spread
    over every core.
    """
    import threadpoolctl

    fused, _, _, kind = cpu_backends()
    jobs, what = cpu_jobs(name, x)
    threads = os.cpu_count() or 1
    done, work = 0, 0.0
    t0 = time.perf_counter()
    with threadpoolctl.threadpool_limits(limits=1), ThreadPoolExecutor(threads) as ex:
        pos = 0
        while True:
            batch = [jobs[(pos + i) % len(jobs)] for i in range(threads)]
            pos += threads
            list(ex.map(lambda j: fused(*j[0], **j[1]), batch))
            done += len(batch)
            work += sum(j[2] for j in batch)
            if time.perf_counter() - t0 > budget_s or done >= 4 * threads:
                break
    dt = time.perf_counter() - t0
    rate = work / dt / (1e9 if name == "fp16_decode_gqa" else 1e12)
    src = "the reference's fused backend" if kind == "reference" else "oracle port of the fused backend"
    return rate, threads, f"{done} {what}, {dt:.1f}s wall; {src}", kind


def cpu_thread_settings(name, x=None, repeats=3):
    """One work item through each reference CPU backend, at default BLAS threads and at one.

    The reference's benchmark harness measures exactly these two settings
    (``benchmark.py:170-188`` ``_limit_threads``, ``:126-149``
    ``describe_threads``). Each figure is the median of ``repeats`` calls
    after one warm-up, as the rate of the metric's unit.
    """
    import threadpoolctl

    fused, reference, bm, kind = cpu_backends()
    jobs, what = cpu_jobs(name, x)
    args, kw, work = jobs[0]
    unit = 1e9 if name == "fp16_decode_gqa" else 1e12

    def limit(n):
        if bm is not None:
            return bm._limit_threads(n)
        return threadpoolctl.threadpool_limits(limits=n) if n else contextlib.nullcontext()

    out = {"cpu_count": os.cpu_count(), "kind": kind,
           "item": what.split(" of ")[0] + f" (first item, shapes q {args[0].shape} k {args[1].shape})"}
    if bm is not None:
        out["describe_threads"] = bm.describe_threads().summary
    else:
        out["describe_threads"] = ", ".join(f"{i.get('internal_api')}={i.get('num_threads')}"
                                            for i in threadpoolctl.threadpool_info())
    for bname, fn in (("fused", fused), ("reference", reference)):
        for label, n in (("default", None), ("1", 1)):
            with limit(n):
                fn(*args, **kw)
                times = []
                for _ in range(repeats):
                    t0 = time.perf_counter()
                    fn(*args, **kw)
                    times.append(time.perf_counter() - t0)
            ms = statistics.median(times) * 1e3
            out[f"{bname}_blas_{label}"] = {"ms": ms, "rate": work / (ms * 1e-3) / unit}
    return out


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from pa_b200 import workloads

    if args.workload in KV_WORKLOADS:
        return run_reference_kv(args)
    w = workloads.WORKLOADS[args.workload]
    # Each step is a bounded sample, sized so the whole run stays within ~2.5 minutes.
    budget = max(0.5, min(4.0, 150.0 / (args.warmup + args.steps)))
    rates = []
    for i in range(args.warmup + args.steps):
        rate, threads, desc, kind = cpu_sample(args.workload, budget_s=budget)
        if i >= args.warmup:
            rates.append(rate)
    value = statistics.median(rates)
    unit = "GB/s" if args.workload == "fp16_decode_gqa" else "TFLOP/s"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32" if w.dtype == "float16" else w.dtype.replace("float", "f"),
        "data": "synthetic", "config": workload_config(args.workload, args.gpus),
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": kind,
                         "sample": desc + " per step",
                         "thread_settings": cpu_thread_settings(args.workload)},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_kv(args):
    """The reference arm for the KV-cache workloads: the oracle's decode on whole sequences."""
    rates = []
    for i in range(args.warmup + args.steps):
        rate, threads, desc = kv_cpu_sample(args.workload, budget_s=4.0)
        if i >= args.warmup:
            rates.append(rate)
    value = statistics.median(rates)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic", "config": {"workload": args.workload + " (decode shapes, one sequence per item)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": desc + " per step"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(name, n, x=None):
    """The ``config`` of a line: the global workload (``x``: a profiling cut of it)."""
    from pa_b200 import workloads

    w = workloads.WORKLOADS[name]
    qs = tuple(x["q"].shape) if x is not None else w.q_shape
    ks = tuple(x["k"].shape) if x is not None else w.kv_shape
    axis = split_axis(w, n)
    return {"workload": f"{name}: q {qs} k/v {ks} {w.dtype}"
                        f"{' causal' if w.is_causal else ''}{' gqa' if w.enable_gqa else ''}"
                        f"{' key-padding mask' if w.masked else ''}",
            "global_batch": qs[0], "seq_len": qs[2],
            "parallelism": (f"{axis}-shard x{n}: one global problem split over {n} GPUs, "
                            "no data-path collective" if n > 1 else "single"),
            "l2": "inputs larger than L2 (no flush)"}


def split_axis(w, n):
    """Axis the global problem is cut along for ``n`` ranks: batch rows, else whole KV-head groups."""
    if n <= 1 or w.q_shape[0] >= n:
        return "batch"
    return "head"


def rank_part(x, w, n, rank):
    """This rank's contiguous part of the global inputs (batch rows, or whole grouped-query groups)."""
    if n <= 1:
        return x
    group = w.q_shape[1] // w.kv_shape[1]
    if split_axis(w, n) == "batch":
        b = np.array_split(np.arange(x["q"].shape[0]), n)[rank]
        sl_q = sl_kv = (slice(int(b[0]), int(b[-1]) + 1),)
        sl_m = sl_q
    else:
        kvh = np.array_split(np.arange(x["k"].shape[1]), n)[rank]
        sl_kv = (slice(None), slice(int(kvh[0]), int(kvh[-1]) + 1))
        sl_q = (slice(None), slice(int(kvh[0]) * group, (int(kvh[-1]) + 1) * group))
        sl_m = None
    out = {}
    for key, val in x.items():
        if key in ("q", "dout"):
            out[key] = np.ascontiguousarray(val[sl_q])
        elif key in ("k", "v"):
            out[key] = np.ascontiguousarray(val[sl_kv])
        elif key == "mask":
            out[key] = np.ascontiguousarray(val[sl_m]) if sl_m is not None and val.shape[0] > 1 else val
        elif key == "keep":
            out[key] = val[sl_m] if sl_m is not None else val
    return out


# ---------------------------------------------------------------- GPU leg

def shrink(x, w, batch=None, heads=None):
    """Keep the first ``batch`` rows / ``heads`` query heads (and their KV heads) of a workload."""
    if not batch and not heads:
        return x
    group = w.q_shape[1] // w.kv_shape[1]
    b = slice(0, batch) if batch else slice(None)
    hq = slice(0, heads) if heads else slice(None)
    hk = slice(0, max(1, heads // group)) if heads else slice(None)
    out = {}
    for key, val in x.items():
        if key in ("q", "dout"):
            out[key] = np.ascontiguousarray(val[b, hq])
        elif key in ("k", "v"):
            out[key] = np.ascontiguousarray(val[b, hk])
        elif key == "mask":
            out[key] = np.ascontiguousarray(val[b])
        elif key == "keep":
            out[key] = val[b]
    return out


def fwd_flops(x, w):
    """Algorithmic forward FLOPs of the (possibly shrunk) inputs: 4 B Hq Lq Lk D, halved if causal."""
    bq, hq, lq, d = x["q"].shape
    f = 4.0 * bq * hq * lq * x["k"].shape[2] * d
    return f / 2 if w.is_causal else f


def run_gpu(args):
    rank, local, world, pg = dist_setup(args.gpus)
    import ctypes

    import pa_b200
    from pa_b200 import workloads
    from pa_b200._lib import check, lib
    from pa_b200.backend import sdpa_device, use_decode_kernel
    from pa_b200.device import DeviceBuffer, Event, Stream

    pa_b200.set_device(local)
    w = workloads.WORKLOADS[args.workload]
    if w.backward and world > 1:
        return run_ring(args, rank, local, world, pg)
    x = shrink(workloads.make(args.workload), w, args.batch, args.heads)
    x_global = {key: x[key] for key in ("q", "k", "v")}
    global_flops = fwd_flops(x, w)
    global_bytes = float(2 * x["k"].nbytes + 2 * x["q"].nbytes)
    # N > 1: the one global problem is cut into N parts (strong scaling).
    x = rank_part(x, w, world, rank)
    mask = x.get("mask")
    plan = pa_b200.plan_call(x["q"].shape, x["k"].shape, x["v"].shape, x["q"].dtype, x["k"].dtype,
                             x["v"].dtype, None if mask is None else mask.shape,
                             None if mask is None else mask.dtype, w.is_causal, None,
                             x["q"].shape[1] // x["k"].shape[1])
    decode = use_decode_kernel(plan)
    backward = w.backward
    stream = Stream()
    bufs = {}

    def upload(key, arr):
        a = np.ascontiguousarray(arr)
        bufs[key] = DeviceBuffer(a.nbytes)
        check(lib().pa_memcpy_h2d(bufs[key].ptr, a.ctypes.data, a.nbytes, stream.handle))

    for key in ("q", "k", "v"):
        upload(key, x[key])
    if mask is not None:
        upload("mask", np.ascontiguousarray(mask).view(np.uint8))
    out_bytes = int(np.prod(plan.out_shape)) * plan.cdt.itemsize
    bufs["out"] = DeviceBuffer(out_bytes)
    if backward:
        upload("dout", x["dout"])
        bufs["lse"] = DeviceBuffer(int(np.prod(plan.out_shape[:-1])) * 4)
        for key in ("dq", "dk", "dv"):
            bufs[key] = DeviceBuffer(x[key[1]].nbytes)
    stream.synchronize()
    desc = ctypes.byref(plan.desc)
    mid = Event() if backward else None

    def step(mark=None):
        if backward:
            check(lib().pa_sdpa_fwd(desc, bufs["q"].ptr, bufs["k"].ptr, bufs["v"].ptr, None,
                                    bufs["out"].ptr, bufs["lse"].ptr, stream.handle))
            if mark is not None:
                mark.record(stream)
            check(lib().pa_sdpa_bwd(desc, bufs["q"].ptr, bufs["k"].ptr, bufs["v"].ptr,
                                    bufs["out"].ptr, bufs["dout"].ptr, bufs["lse"].ptr,
                                    bufs["dq"].ptr, bufs["dk"].ptr, bufs["dv"].ptr, stream.handle))
            return
        sdpa_device(plan, bufs["q"].ptr, bufs["k"].ptr, bufs["v"].ptr, bufs["out"].ptr,
                    mask_ptr=bufs["mask"].ptr if "mask" in bufs else None, stream=stream,
                    decode=decode)

    clocks = ClockSampler(local, clock_log(args, rank)).start()
    for _ in range(args.warmup):
        step()
    stream.synchronize()
    pa_b200.sync_device_status()
    events = [Event() for _ in range(args.steps + 1)]
    mids = [Event() for _ in range(args.steps)] if backward else None
    barrier(pg)
    stream.synchronize()
    clocks.mark(0)
    events[0].record(stream)
    for i in range(args.steps):
        step(mids[i] if mids else None)
        events[i + 1].record(stream)
    stream.synchronize()
    clocks.mark(1)
    clocks.stop()
    barrier(pg)
    pa_b200.sync_device_status()
    per = [events[i].elapsed_ms(events[i + 1]) for i in range(args.steps)]
    ms_local = events[0].elapsed_ms(events[-1]) / args.steps
    ms = max_over_ranks(pg, ms_local, local)

    pk, pk_kind = peaks()
    extra = {}
    if decode:
        unit = "GB/s"
        work = float(2 * x["k"].nbytes + x["q"].nbytes + out_bytes)
        value = global_bytes / (ms * 1e-3) / 1e9
        achieved = work / (statistics.mean(per) * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "traffic": traffic_for(args.workload),
                "peak_kind": pk_kind, "kernel": "decode_partial + decode_combine"}
        launches = 2
    elif backward:
        unit = "TFLOP/s"
        work = 3.5 * fwd_flops(x, w)
        value = world * work / (ms * 1e-3) / 1e12
        fwd_ms = statistics.mean(events[i].elapsed_ms(mids[i]) for i in range(args.steps))
        bwd_ms = statistics.mean(mids[i].elapsed_ms(events[i + 1]) for i in range(args.steps))
        peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
        achieved = 2.5 * fwd_flops(x, w) / (bwd_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic_for(args.workload),
                "peak_kind": pk_kind + " (sustained: seconds-long step)",
                "kernel": "backward: bwd_prep + bwd_dkdv + bwd_dq (2.5x forward FLOPs)"}
        extra = {"fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
                 "fwd_tflops": fwd_flops(x, w) / (fwd_ms * 1e-3) / 1e12,
                 "bwd_tflops": achieved}
        launches = 4
    else:
        unit = "TFLOP/s"
        work = fwd_flops(x, w)
        value = global_flops / (ms * 1e-3) / 1e12
        achieved = work / (statistics.mean(per) * 1e-3) / 1e12
        if plan.cdt in (np.float16,):
            roof = {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"],
                    "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops"],
                    "traffic": traffic_for(args.workload), "peak_kind": pk_kind + " (burst)",
                    "kernel": "fwd_tc"}
        else:
            # fp32 on CUDA cores (FFMA, no TF32): no measured fp32 peak exists.
            roof = {"bound": "fp32 ffma", "achieved": achieved, "peak": FP32_FFMA_PEAK_TFLOPS,
                    "unit": "TFLOP/s", "frac": achieved / FP32_FFMA_PEAK_TFLOPS,
                    "traffic": traffic_for(args.workload),
                    "peak_kind": "theoretical (148 SMs x 128 FFMA lanes x 2 x 1965 MHz)",
                    "kernel": "sdpa_exact_rt"}
        # a boolean mask adds the tile-classification pre-pass
        launches = 2 if (mask is not None and mask.dtype == np.bool_) else 1

    # End to end through the public call on page-locked NumPy inputs.
    host = {key: pa_b200.pinned_empty(x[key].shape, x[key].dtype)
            for key in ("q", "k", "v") + (("dout",) if backward else ())}
    for key, arr in host.items():
        arr[...] = x[key]
    kw = {"is_causal": w.is_causal, "enable_gqa": w.enable_gqa}
    if mask is not None:
        kw["attn_mask"] = mask

    def public_call():
        if backward:
            return pa_b200.sdpa_backward(host["q"], host["k"], host["v"], host["dout"], **kw)
        return (pa_b200.scaled_dot_product_attention(host["q"], host["k"], host["v"], **kw),)

    # Warm up exactly like the timed loop (the previous result stays alive while
    # the next call runs), so the pinned-output pool reaches its steady state.
    res = None
    for _ in range(3):
        res = public_call()
    e2e_steps = max(1, min(args.steps, 10))
    barrier(pg)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        res = public_call()
    e2e_ms_local = (time.perf_counter() - t0) * 1e3 / e2e_steps
    barrier(pg)
    e2e_ms = max_over_ranks(pg, e2e_ms_local, local)
    global_work = global_bytes if decode else (3.5 * global_flops if backward else global_flops)
    e2e_val = global_work / (e2e_ms * 1e-3) / (1e9 if decode else 1e12)
    h2d = sum_over_ranks(pg, sum(a.nbytes for a in host.values()) + (mask.nbytes if mask is not None else 0), local)
    d2h = sum_over_ranks(pg, sum(r.nbytes for r in res), local)

    # The same public call on ordinary (pageable) NumPy arrays, as most callers hold them.
    del res
    plain = {key: np.ascontiguousarray(x[key]) for key in host}

    def pageable_call():
        if backward:
            return pa_b200.sdpa_backward(plain["q"], plain["k"], plain["v"], plain["dout"], **kw)
        return (pa_b200.scaled_dot_product_attention(plain["q"], plain["k"], plain["v"], **kw),)

    res = pageable_call()
    pg_steps = max(1, min(args.steps, 5))
    barrier(pg)
    t0 = time.perf_counter()
    for _ in range(pg_steps):
        res = pageable_call()
    pg_ms = max_over_ranks(pg, (time.perf_counter() - t0) * 1e3 / pg_steps, local)
    del res

    subs = None
    if args.workload == "fp16_causal_gqa" and not args.no_workloads and args.batch is None and args.heads is None:
        try:
            subs = workload_subrecords(rank, local, world, pg)
        except Exception as exc:  # noqa: BLE001 -- keep the main line; every rank fails alike
            subs = {"error": f"{type(exc).__name__}: {exc}"}

    ring = None
    if world > 1 and not args.no_ring and not backward and not decode:
        try:
            ring = ring_subrecord(rank, local, world, pg, clock_path=clock_log(args, rank, "_ring"))
        except Exception as exc:  # noqa: BLE001 -- keep the main line; every rank fails alike
            ring = {"error": f"{type(exc).__name__}: {exc}"}

    if rank != 0:
        if pg is not None:
            pg.destroy_process_group()
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16" if plan.cdt == np.float16 else str(plan.cdt).replace("float", "f"),
        "data": "synthetic", "config": workload_config(args.workload, world, x_global),
        "roofline": roof,
        "e2e": {"value": e2e_val, "unit": unit, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms,
                "timing": "host wall clock around the synchronous public call, page-locked inputs",
                "pageable": {"value": global_work / (pg_ms * 1e-3) / (1e9 if decode else 1e12),
                             "ms_per_step": pg_ms,
                             "timing": "the same call on ordinary pageable NumPy arrays"}},
        "gpu_launches": args.steps * launches * world,
        "clocks": clocks.summary(),
        **extra,
    }
    if subs is not None:
        line["workloads"] = subs
    if ring is not None:
        line["ring"] = ring
    if world == 1 and not args.no_cpu:
        rate, threads, desc_s, kind = cpu_sample(args.workload, x=x if w.backward else None)
        line["cpu_baseline"] = {"value": rate, "unit": unit, "cores": threads, "kind": kind,
                                "sample": desc_s,
                                "thread_settings": cpu_thread_settings(
                                    args.workload, x=x if w.backward else None)}
    print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


FP32_FFMA_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12   # theoretical; no measured fp32 peak exists


def _timed(step, steps, warmup, stream, pg, local):
    """Max-over-ranks mean CUDA-event time of ``step`` (ms), after warm-up."""
    import pa_b200
    from pa_b200.device import Event

    for _ in range(warmup):
        step()
    stream.synchronize()
    pa_b200.sync_device_status()
    ev = [Event() for _ in range(steps + 1)]
    barrier(pg)
    ev[0].record(stream)
    for i in range(steps):
        step()
        ev[i + 1].record(stream)
    stream.synchronize()
    pa_b200.sync_device_status()
    return max_over_ranks(pg, ev[0].elapsed_ms(ev[-1]) / steps, local)


def workload_subrecords(rank, local, world, pg):
    """Device-timed lines for the other benchmark configurations, in the same run.

    N = 1: the fp32 exact forward (4, 8, 512, 64), the masked cross-attention
    forward (16, 16, 1024 x 2048, 64), the split-KV decode (64 x 32 heads,
    32768 keys) and the long-context causal forward + backward (1, 32,
    131072, 128). N > 1: the decode with its batch split over the ranks (one
    global problem, no collective). The two small workloads use their seeded
    NumPy inputs; the decode and long-context tensors (8 GiB / 4 GiB) are
    drawn on the device (``torch.randn``, N(0, 1) scaled as the workload
    says) because only their timing is used.
    """
    import ctypes

    import torch

    import pa_b200
    from pa_b200 import workloads
    from pa_b200._lib import check, lib
    from pa_b200.backend import sdpa_device
    from pa_b200.device import Event, Stream

    pk, pk_kind = peaks()
    dev = torch.device("cuda", local)
    stream = Stream()
    out = {}

    def to_dev(arr):
        return torch.from_numpy(np.ascontiguousarray(arr)).to(dev)

    if world == 1:
        for name in ("fp32_unmasked", "fp16_masked_cross"):
            w = workloads.WORKLOADS[name]
            x = workloads.make(name)
            t = {key: to_dev(x[key]) for key in ("q", "k", "v")}
            m = to_dev(x["mask"].view(np.uint8)) if "mask" in x else None
            o = torch.empty(w.q_shape[:3] + (w.kv_shape[3],), device=dev, dtype=t["q"].dtype)
            plan = pa_b200.plan_call(w.q_shape, w.kv_shape, w.kv_shape, x["q"].dtype, x["k"].dtype,
                                     x["v"].dtype, None if m is None else x["mask"].shape,
                                     None if m is None else np.bool_, w.is_causal, None, 1)
            torch.cuda.synchronize(dev)

            def step():
                sdpa_device(plan, t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(),
                            o.data_ptr(), mask_ptr=None if m is None else m.data_ptr(),
                            stream=stream, decode=False)

            ms = _timed(step, 50, 5, stream, pg, local)
            tf = w.flops_fwd / (ms * 1e-3) / 1e12
            if name == "fp32_unmasked":
                out[name] = {"value": tf, "unit": "TFLOP/s", "ms_per_step": ms, "kernel": "sdpa_exact_rt (fp32 FFMA)",
                             "traffic": traffic_for(name),
                             "frac_of_fp32_ffma_theoretical": tf / FP32_FFMA_PEAK_TFLOPS,
                             "peak_note": "148 SMs x 128 FFMA lanes x 2 x 1965 MHz; no measured fp32 peak"}
            else:
                out[name] = {"value": tf, "unit": "TFLOP/s", "ms_per_step": ms,
                             "kernel": "mask_classify + fwd_tc<64, bool mask>", "traffic": traffic_for(name),
                             "frac": tf / pk["bf16_tflops"], "peak": pk["bf16_tflops"],
                             "peak_kind": pk_kind + " (burst)",
                             "note": "algorithmic FLOPs of the whole 1024 x 2048 problem; masked-out key tiles are skipped"}
            del t, m, o

    # Split-KV decode; at N > 1 each rank holds 64 / N batch rows.
    w = workloads.WORKLOADS["fp16_decode_gqa"]
    B, Hq, _, D = w.q_shape
    Hkv, S = w.kv_shape[1], w.kv_shape[2]
    rows = np.array_split(np.arange(B), world)[rank]
    b = len(rows)
    gen = torch.Generator(device=dev).manual_seed(3 + rank)
    q = (torch.randn((b, Hq, 1, D), generator=gen, device=dev) * 0.5).half()
    k = (torch.randn((b, Hkv, S, D), generator=gen, device=dev, dtype=torch.float16) * 0.5)
    v = (torch.randn((b, Hkv, S, D), generator=gen, device=dev, dtype=torch.float16) * 0.5)
    o = torch.empty_like(q)
    plan = pa_b200.plan_call(q.shape, k.shape, v.shape, np.float16, np.float16, np.float16, group=Hq // Hkv)
    nb = ctypes.c_size_t(0)
    check(lib().pa_decode_workspace_size(ctypes.byref(plan.desc), ctypes.byref(nb)))
    ws_bytes = int(nb.value)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    torch.cuda.synchronize(dev)

    def dstep():
        sdpa_device(plan, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), stream=stream,
                    decode=True, workspace=(ws.data_ptr(), ws_bytes))

    ms = _timed(dstep, 30, 5, stream, pg, local)
    gbytes = 2.0 * B * Hkv * S * D * 2 + 2.0 * B * Hq * D * 2
    gbs = gbytes / (ms * 1e-3) / 1e9
    out["fp16_decode_gqa"] = {"value": gbs, "unit": "GB/s", "ms_per_step": ms,
                              "kernel": "decode_partial + decode_combine",
                              "traffic": traffic_for("fp16_decode_gqa") if world == 1 else None,
                              "frac": gbs / world / pk["hbm_gbs"], "peak": pk["hbm_gbs"],
                              "peak_kind": pk_kind + " (per GPU)",
                              "parallelism": f"batch-shard x{world}" if world > 1 else "single",
                              "scaling": "strong"}
    del q, k, v, o, ws

    if world == 1:
        # Long-context causal forward + backward on one GPU.
        w = workloads.WORKLOADS["fp16_long_causal"]
        gen = torch.Generator(device=dev).manual_seed(4)
        t = {key: torch.randn(w.q_shape, generator=gen, device=dev, dtype=torch.float16)
             for key in ("q", "k", "v", "dout")}
        for key in ("out", "dq", "dk", "dv"):
            t[key] = torch.empty(w.q_shape, device=dev, dtype=torch.float16)
        lse = torch.empty(w.q_shape[:3], device=dev, dtype=torch.float32)
        plan = pa_b200.plan_call(w.q_shape, w.kv_shape, w.kv_shape, np.float16, np.float16, np.float16,
                                 is_causal=True)
        desc = ctypes.byref(plan.desc)
        mid = [None]
        torch.cuda.synchronize(dev)

        def lstep():
            check(lib().pa_sdpa_fwd(desc, t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), None,
                                    t["out"].data_ptr(), lse.data_ptr(), stream.handle))
            if mid[0] is not None:
                mid[0].record(stream)
            check(lib().pa_sdpa_bwd(desc, t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(),
                                    t["out"].data_ptr(), t["dout"].data_ptr(), lse.data_ptr(),
                                    t["dq"].data_ptr(), t["dk"].data_ptr(), t["dv"].data_ptr(),
                                    stream.handle))

        ms = _timed(lstep, 3, 2, stream, pg, local)
        e0, mid[0], e1 = Event(), Event(), Event()
        e0.record(stream)
        lstep()
        e1.record(stream)
        stream.synchronize()
        fwd_ms, bwd_ms = e0.elapsed_ms(mid[0]), mid[0].elapsed_ms(e1)
        peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
        bwd_tf = w.flops_bwd / (bwd_ms * 1e-3) / 1e12
        out["fp16_long_causal"] = {
            "value": (w.flops_fwd + w.flops_bwd) / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": ms, "fwd_tflops": w.flops_fwd / (fwd_ms * 1e-3) / 1e12,
            "bwd_tflops": bwd_tf, "bwd_frac": bwd_tf / peak, "peak": peak,
            "peak_kind": pk_kind + " (sustained: seconds-long step)",
            "kernel": "fwd_tc + bwd_prep + bwd_dkdv + bwd_dq"}
        del t, lse
    torch.cuda.synchronize(dev)
    return out


def ring_subrecord(rank, local, world, pg, steps=3, warmup=2, clock_path=None):
    """The long-context causal fwd+bwd as a ring over the same ranks (one global problem).

    q, k, v, dO (1, 32, 131072, 128) fp16, N(0, 1) like the long-context
    workload but drawn on each device (``torch.randn``, seed 4 + rank) since
    only the timing is used; each rank holds its zig-zag shard. Returns the
    whole-job TFLOP/s (max-over-ranks step time), the forward / backward
    split, and the per-phase split of one extra profiled step (CUDA events at
    the phase boundaries inside ``pa_ring_fwd`` / ``pa_ring_bwd``): repacking
    copies, attention kernels, fp32 accumulation, compute-stream stalls on
    NCCL, and NCCL transfer time on the side stream.
    """
    import torch

    import pa_b200
    from pa_b200 import workloads
    from pa_b200.device import Event, Stream
    from pa_b200.ring import RingComm

    w = workloads.WORKLOADS["fp16_long_causal"]
    _, H, L, D = w.q_shape
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(4 + rank)
    shape = (1, H, L // world, D)
    t = {key: torch.randn(shape, generator=gen, device=dev, dtype=torch.float16)
         for key in ("q", "k", "v", "dout")}
    for key in ("out", "dq", "dk", "dv"):
        t[key] = torch.empty(shape, device=dev, dtype=torch.float16)
    lse = torch.empty(shape[:-1], device=dev, dtype=torch.float32)
    torch.cuda.synchronize(dev)
    plan = pa_b200.plan_call(shape, shape, shape, np.float16, np.float16, np.float16, is_causal=True)
    comm = RingComm.from_process_group()
    stream = Stream()
    p = {key: val.data_ptr() for key, val in t.items()}

    def step(mid=None):
        comm.forward(plan, p["q"], p["k"], p["v"], p["out"], lse.data_ptr(), stream)
        if mid is not None:
            mid.record(stream)
        comm.backward(plan, p["q"], p["k"], p["v"], p["out"], p["dout"], lse.data_ptr(), p["dq"],
                      p["dk"], p["dv"], stream)

    try:
        for _ in range(warmup):
            step()
        comm.wait(stream, timeout_ms=300000)
        ev = [Event() for _ in range(steps + 1)]
        mids = [Event() for _ in range(steps)]
        clocks = ClockSampler(local, clock_path).start() if clock_path is not None else None
        barrier(pg)
        if clocks:
            clocks.mark(0)
        ev[0].record(stream)
        for i in range(steps):
            step(mids[i])
            ev[i + 1].record(stream)
        comm.wait(stream, timeout_ms=300000)
        if clocks:
            clocks.mark(1)
            clocks.stop()
        ms = max_over_ranks(pg, ev[0].elapsed_ms(ev[-1]) / steps, local)
        fwd_ms = max_over_ranks(pg, statistics.mean(ev[i].elapsed_ms(mids[i]) for i in range(steps)), local)
        bwd_ms = max_over_ranks(pg, statistics.mean(mids[i].elapsed_ms(ev[i + 1]) for i in range(steps)), local)
        barrier(pg)
        comm.profile_start()
        step()
        comm.wait(stream, timeout_ms=300000)
        phases = comm.profile_read()
        phases_max = {key: max_over_ranks(pg, val, local) for key, val in phases.items()}
    finally:
        comm.close()
    work = w.flops_fwd + w.flops_bwd
    return {"workload": "fp16_long_causal fwd+bwd: q,k,v,dO (1, 32, 131072, 128) causal, "
                        "zig-zag sequence shards, inputs drawn on the device",
            "value": work / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "steps": steps, "warmup": warmup,
            "phase_ms_rank0": phases, "phase_ms_max_over_ranks": phases_max,
            "phase_note": "one extra profiled step; attention + accumulate + repack + wait_nccl "
                          "is the compute stream's busy time, nccl_transfer overlaps it",
            "clocks_rank0": clocks.summary() if clocks else None}


def run_ring(args, rank, local, world, pg):
    """Long-context causal fwd+bwd, sequence-sharded over ``world`` GPUs (ring attention).

    Every rank keeps its zig-zag shard of the one global problem (strong
    scaling: total work is fixed); K/V move between GPUs with NCCL inside
    ``pa_ring_fwd`` / ``pa_ring_bwd``. ``value`` = the global problem's fwd+bwd
    FLOPs over the max-over-ranks step time.
    """
    import ctypes

    import pa_b200
    from pa_b200 import workloads
    from pa_b200._lib import check, lib
    from pa_b200.device import DeviceBuffer, Event, Stream
    from pa_b200.ring import RingComm, shard

    w = workloads.WORKLOADS[args.workload]
    x = workloads.make(args.workload)
    sh = {key: np.ascontiguousarray(shard(x[key], world, rank)) for key in ("q", "k", "v", "dout")}
    del x
    plan = pa_b200.plan_call(sh["q"].shape, sh["k"].shape, sh["v"].shape, sh["q"].dtype, sh["k"].dtype,
                             sh["v"].dtype, is_causal=True)
    comm = RingComm.from_process_group()
    stream = Stream()
    bufs = {key: DeviceBuffer(arr.nbytes) for key, arr in sh.items()}
    for key, arr in sh.items():
        check(lib().pa_memcpy_h2d(bufs[key].ptr, arr.ctypes.data, arr.nbytes, stream.handle))
    for key in ("out", "dq", "dk", "dv"):
        bufs[key] = DeviceBuffer(sh["q"].nbytes)
    bufs["lse"] = DeviceBuffer(int(np.prod(sh["q"].shape[:-1])) * 4)
    stream.synchronize()

    def step(mark=None):
        comm.forward(plan, bufs["q"].ptr, bufs["k"].ptr, bufs["v"].ptr, bufs["out"].ptr,
                     bufs["lse"].ptr, stream)
        if mark is not None:
            mark.record(stream)
        comm.backward(plan, bufs["q"].ptr, bufs["k"].ptr, bufs["v"].ptr, bufs["out"].ptr,
                      bufs["dout"].ptr, bufs["lse"].ptr, bufs["dq"].ptr, bufs["dk"].ptr,
                      bufs["dv"].ptr, stream)

    clocks = ClockSampler(local, clock_log(args, rank)).start()
    for _ in range(args.warmup):
        step()
    comm.wait(stream, timeout_ms=300000)
    pa_b200.sync_device_status()
    events = [Event() for _ in range(args.steps + 1)]
    mids = [Event() for _ in range(args.steps)]
    barrier(pg)
    clocks.mark(0)
    events[0].record(stream)
    for i in range(args.steps):
        step(mids[i])
        events[i + 1].record(stream)
    comm.wait(stream, timeout_ms=300000)
    clocks.mark(1)
    clocks.stop()
    barrier(pg)
    ms = max_over_ranks(pg, events[0].elapsed_ms(events[-1]) / args.steps, local)
    fwd_ms = max_over_ranks(pg, statistics.mean(events[i].elapsed_ms(mids[i]) for i in range(args.steps)), local)
    bwd_ms = max_over_ranks(pg, statistics.mean(mids[i].elapsed_ms(events[i + 1]) for i in range(args.steps)), local)
    barrier(pg)
    comm.profile_start()
    step()
    comm.wait(stream, timeout_ms=300000)
    phases = comm.profile_read()
    phases_max = {key: max_over_ranks(pg, val, local) for key, val in phases.items()}
    work = w.flops_fwd + w.flops_bwd
    value = work / (ms * 1e-3) / 1e12
    pk, pk_kind = peaks()
    peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    per_gpu = value / world
    roof = {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
            "frac": per_gpu / peak, "traffic": None, "peak_kind": pk_kind + " (sustained)",
            "kernel": "ring step (fwd_tc + bwd kernels per chunk pair, NCCL send/recv overlapped)"}

    # End to end: pinned host shards in, gradients out, around the public ring calls.
    host = {key: pa_b200.pinned_empty(arr.shape, arr.dtype) for key, arr in sh.items()}
    for key in host:
        host[key][...] = sh[key]
    res = {key: pa_b200.pinned_empty(sh["q"].shape, sh["q"].dtype) for key in ("dq", "dk", "dv")}
    barrier(pg)
    t0 = time.perf_counter()
    e2e_steps = max(1, min(args.steps, 3))
    for _ in range(e2e_steps):
        for key, arr in host.items():
            check(lib().pa_memcpy_h2d(bufs[key].ptr, arr.ctypes.data, arr.nbytes, stream.handle))
        step()
        for key, arr in res.items():
            check(lib().pa_memcpy_d2h(arr.ctypes.data, bufs[key].ptr, arr.nbytes, stream.handle))
        comm.wait(stream, timeout_ms=300000)
    e2e_ms = max_over_ranks(pg, (time.perf_counter() - t0) * 1e3 / e2e_steps, local)
    h2d = sum(a.nbytes for a in host.values())
    d2h = sum(a.nbytes for a in res.values())
    summary = clocks.summary()
    comm.close()
    if rank == 0:
        cfg = workload_config(args.workload, world)
        cfg["global_batch"] = w.q_shape[0]
        cfg["parallelism"] = f"ring (zig-zag sequence shards) x{world}"
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic", "config": cfg, "roofline": roof,
            "e2e": {"value": work / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": int(h2d) * world, "d2h_bytes_per_step": int(d2h) * world,
                    "ms_per_step": e2e_ms, "timing": "host wall clock, pinned shards, max over ranks"},
            # per rank per step: fwd 2 per chunk pair + 6 fills/stores, bwd 6 per pair + 8
            "gpu_launches": args.steps * (8 * (2 * world + 1) + 14), "clocks": summary,
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
            "phase_ms_rank0": phases, "phase_ms_max_over_ranks": phases_max,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


KV_WORKLOADS = {
    "kv_fp8_decode_gqa": {"kv_format": "e4m3", "page_size": None},
    "kv_paged_decode_gqa": {"kv_format": None, "page_size": 16},
    "kv_paged_fp8_decode_gqa": {"kv_format": "e4m3", "page_size": 16},
}


_KV_SAMPLE: dict = {}


def kv_cpu_sample(name, budget_s=12.0):
    """The oracle's KV-cache decode (float64 restatement of the reference math on
    the gathered, dequantised keys) on whole sequences of the workload's shape,
    one thread per host core. Rate in GB/s of cache bytes in the storage type."""
    from oracle.kvcache import decode_kv_reference, float_to_e4m3
    from pa_b200 import workloads

    spec = KV_WORKLOADS[name]
    w = workloads.WORKLOADS["fp16_decode_gqa"]
    _, hq, _, d = w.q_shape
    _, hkv, s, _ = w.kv_shape
    key = (name, hq, hkv, s, d)
    if key not in _KV_SAMPLE:
        gen = np.random.default_rng(3)
        q = (gen.standard_normal((1, hq, d)) * 0.5).astype(np.float16)
        k = (gen.standard_normal((1, hkv, s, d)) * 0.5).astype(np.float16)
        v = (gen.standard_normal((1, hkv, s, d)) * 0.5).astype(np.float16)
        if spec["kv_format"] == "e4m3":
            k, v = float_to_e4m3(k), float_to_e4m3(v)
        _KV_SAMPLE[key] = (q, k, v)
    q, k, v = _KV_SAMPLE[key]
    kw = {"kv_format": "e4m3"} if spec["kv_format"] == "e4m3" else {}
    per_seq = 2 * k.nbytes
    threads = os.cpu_count() or 1
    done = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        while True:
            list(ex.map(lambda _: decode_kv_reference(q, k, v, **kw), range(threads)))
            done += threads
            if time.perf_counter() - t0 > budget_s:
                break
    dt = time.perf_counter() - t0
    return (done * per_seq / dt / 1e9, threads,
            f"{done} sequences of q (1,{hq},{d}) vs a {hkv}x{s}x{d} cache, float64 oracle, {dt:.1f}s wall")


def run_kvcache(args):
    """Decode from an fp8 and/or paged KV cache (pa_decode_kv_fwd) on the decode shapes."""
    rank, local, world, pg = dist_setup(args.gpus)
    import torch

    import pa_b200
    from pa_b200 import workloads
    from pa_b200._lib import check, lib
    from pa_b200.device import DeviceBuffer, Event, Stream
    from pa_b200.kvcache import kv_workspace_size

    spec = KV_WORKLOADS[args.workload]
    pa_b200.set_device(local)
    dev = torch.device("cuda", local)
    x = workloads.make("fp16_decode_gqa")
    rows = slice(0, args.batch) if args.batch else slice(None)   # --batch: the first sequences only
    q = torch.from_numpy(np.ascontiguousarray(x["q"][rows, :, 0])).to(dev)
    k = torch.from_numpy(np.ascontiguousarray(x["k"][rows])).to(dev)
    v = torch.from_numpy(np.ascontiguousarray(x["v"][rows])).to(dev)
    del x
    B, Hq, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    if spec["kv_format"] == "e4m3":
        k = k.to(torch.float8_e4m3fn).view(torch.uint8)
        v = v.to(torch.float8_e4m3fn).view(torch.uint8)
    table = None
    ps = spec["page_size"]
    if ps:
        n_pages = B * S // ps
        gen = torch.Generator(device=dev).manual_seed(7)
        perm = torch.randperm(n_pages, device=dev, generator=gen)

        def to_pages(t):
            tp = t.view(B, Hkv, S // ps, ps, D).permute(0, 2, 1, 3, 4).reshape(n_pages, Hkv, ps, D)
            out = torch.empty_like(tp)
            out[perm] = tp
            return out

        k, v = to_pages(k), to_pages(v)
        table = perm.view(B, S // ps).to(torch.int32).contiguous()
    torch.cuda.synchronize(dev)
    desc = pa_b200.kv_cache_desc(B, Hq, D, tuple(k.shape), kv_format=spec["kv_format"],
                                 paged=table is not None,
                                 max_pages_per_seq=table.shape[1] if table is not None else 0,
                                 max_seq_len=S)
    ws_bytes = kv_workspace_size(desc, table is not None)
    ws = DeviceBuffer(ws_bytes)
    out = torch.empty_like(q)
    stream = Stream()

    def step():
        pa_b200.decode_kv_device(desc, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                 block_table_ptr=None if table is None else table.data_ptr(),
                                 stream=stream, workspace=(ws.ptr, ws_bytes))

    clocks = ClockSampler(local, clock_log(args, rank)).start()
    for _ in range(args.warmup):
        step()
    stream.synchronize()
    pa_b200.sync_device_status()
    events = [Event() for _ in range(args.steps + 1)]
    barrier(pg)
    stream.synchronize()
    clocks.mark(0)
    events[0].record(stream)
    for i in range(args.steps):
        step()
        events[i + 1].record(stream)
    stream.synchronize()
    clocks.mark(1)
    clocks.stop()
    barrier(pg)
    pa_b200.sync_device_status()
    per = [events[i].elapsed_ms(events[i + 1]) for i in range(args.steps)]
    ms = max_over_ranks(pg, events[0].elapsed_ms(events[-1]) / args.steps, local)
    work = float(2 * k.numel() * k.element_size() + 2 * q.numel() * q.element_size()
                 + (table.numel() * 4 if table is not None else 0))
    value = world * work / (ms * 1e-3) / 1e9
    pk, pk_kind = peaks()
    achieved = work / (statistics.mean(per) * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"], "traffic": traffic_for(args.workload),
            "peak_kind": pk_kind, "kernel": "decode_partial + decode_combine"}

    # Serving step end to end: the query in from page-locked memory, decode on the
    # resident cache, the output back (synchronous per step).
    hq_in = pa_b200.pinned_empty((B, Hq, D), np.float16)
    hq_in[...] = q.cpu().numpy()
    h_out = pa_b200.pinned_empty((B, Hq, D), np.float16)
    for _ in range(3):
        check(lib().pa_memcpy_h2d(q.data_ptr(), hq_in.ctypes.data, hq_in.nbytes, stream.handle))
        step()
        check(lib().pa_memcpy_d2h(h_out.ctypes.data, out.data_ptr(), h_out.nbytes, stream.handle))
        stream.synchronize()
    e2e_steps = max(1, min(args.steps, 20))
    barrier(pg)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        check(lib().pa_memcpy_h2d(q.data_ptr(), hq_in.ctypes.data, hq_in.nbytes, stream.handle))
        step()
        check(lib().pa_memcpy_d2h(h_out.ctypes.data, out.data_ptr(), h_out.nbytes, stream.handle))
        stream.synchronize()
    e2e_ms = max_over_ranks(pg, (time.perf_counter() - t0) * 1e3 / e2e_steps, local)
    pa_b200.sync_device_status()
    if rank != 0:
        if pg is not None:
            pg.destroy_process_group()
        return 0
    cache = f"{'fp8 e4m3' if spec['kv_format'] else 'fp16'} {'paged (16-key pages, random order)' if ps else 'contiguous'}"
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 cache, f16 q/out" if spec["kv_format"] else "f16",
        "data": "synthetic",
        "config": {"workload": f"{args.workload}: q ({B}, {Hq}, 1, {D}) vs a {cache} cache of "
                               f"{B} sequences x {Hkv} kv heads x {S} keys x {D}",
                   "global_batch": B * world, "seq_len": S,
                   "parallelism": f"batch-shard x{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (no flush)"},
        "roofline": roof,
        "e2e": {"value": world * work / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": int(hq_in.nbytes) * world,
                "d2h_bytes_per_step": int(h_out.nbytes) * world, "ms_per_step": e2e_ms,
                "timing": "host wall clock; cache resident on the device, query in and output out per step"},
        "gpu_launches": args.steps * 2,
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu:
        rate, threads, desc_s = kv_cpu_sample(args.workload)
        line["cpu_baseline"] = {"value": rate, "unit": "GB/s", "cores": threads, "kind": "port",
                                "sample": desc_s}
    print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


def traffic_for(name):
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get(name)
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="fp16_causal_gqa")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-workloads", action="store_true",
                    help="skip the device-timed lines of the other workloads")
    ap.add_argument("--no-ring", action="store_true",
                    help="N > 1: skip the ring-attention sub-record of the long-context workload")
    ap.add_argument("--clock-dir", default=None,
                    help="folder for the per-rank nvidia-smi clock samples (default: a temp folder)")
    ap.add_argument("--batch", type=int, default=None,
                    help="keep only the first BATCH batch rows of the workload (profiling)")
    ap.add_argument("--heads", type=int, default=None,
                    help="keep only the first HEADS query heads (and their KV heads)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload in KV_WORKLOADS:
        return run_kvcache(args)
    return run_gpu(args)


if __name__ == "__main__":
    raise SystemExit(main())
