"""Host logic of ``bench.py`` (CPU only): how one global problem is cut over N ranks.

``bench.py --gpus N`` splits the one global workload into N contiguous parts
(batch rows, or whole grouped-query KV-head groups when there are fewer batch
rows than ranks) with no data-path collective; the parts must tile the global
inputs exactly, or the whole-job rate would count work twice or not at all.
The two-rank ``gloo`` test exchanges each rank's part and reassembles it.
"""

from __future__ import annotations

import importlib.util
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("pa_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _small(w):
    """Small stand-ins with the workload's batch / head structure (values index their position)."""
    b, hq, _, d = w.q_shape
    hkv = w.kv_shape[1]
    q = np.arange(b * hq * 3 * 2, dtype=np.float32).reshape(b, hq, 3, 2)
    k = np.arange(b * hkv * 4 * 2, dtype=np.float32).reshape(b, hkv, 4, 2)
    x = {"q": q, "k": k, "v": -k}
    if w.masked:
        x["mask"] = np.arange(b * 3 * 4).reshape(b, 1, 3, 4) % 3 > 0
        x["keep"] = np.arange(b)
    if w.backward:
        x["dout"] = -q
    return x


@pytest.mark.parametrize("n", [1, 2, 4, 8])
@pytest.mark.parametrize("name", ["fp32_unmasked", "fp16_causal_gqa", "fp16_masked_cross",
                                  "fp16_decode_gqa"])
def test_rank_parts_tile_the_global_problem(name, n):
    bench = _bench()
    from pa_b200 import workloads

    w = workloads.WORKLOADS[name]
    x = _small(w)
    parts = [bench.rank_part(x, w, n, r) for r in range(n)]
    axis = 0 if bench.split_axis(w, n) == "batch" else 1
    for key in ("q", "k", "v"):
        np.testing.assert_array_equal(np.concatenate([p[key] for p in parts], axis=axis), x[key])
    group = w.q_shape[1] // w.kv_shape[1]
    for p in parts:
        assert p["q"].shape[1] == p["k"].shape[1] * group     # whole grouped-query groups
        assert p["q"].shape[0] == p["k"].shape[0]
    if w.masked:
        np.testing.assert_array_equal(np.concatenate([p["mask"] for p in parts], axis=0)
                                      if axis == 0 else parts[0]["mask"], x["mask"])
    cfg = bench.workload_config(name, n)
    assert cfg["global_batch"] == w.q_shape[0]
    assert ("shard x%d" % n in cfg["parallelism"]) == (n > 1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT / "portable-attention_b200"))
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        bench = _bench()
        from pa_b200 import workloads

        w = workloads.WORKLOADS["fp16_causal_gqa"]
        x = _small(w)
        mine = bench.rank_part(x, w, world, rank)
        got = [None] * world
        dist.all_gather_object(got, {k: mine[k] for k in ("q", "k", "v")})
        if rank == 0:
            ok = all(np.array_equal(np.concatenate([g[k] for g in got], axis=0), x[k])
                     for k in ("q", "k", "v"))
            out.put(ok)
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_parts_reassemble():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) is True
