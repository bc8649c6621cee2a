"""One rank of the multi-GPU ring attention check (run under torchrun).

Every rank draws the same seeded causal problem, keeps its zig-zag shard,
runs ``pa_ring_fwd`` and ``pa_ring_bwd`` over an NCCL communicator of the
native library, and rank 0 compares the gathered output, lse and gradients
with the float64 oracle (output 2e-3 abs/rel, lse 1e-3, gradients 2e-2
relative Frobenius). Exit status 0 means every rank passed.
"""

from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "portable-attention_b200")]


def main():
    import torch.distributed as dist

    import pa_b200
    from oracle.sdpa import reference_lse, reference_sdpa
    from oracle.vjp import reference_vjp
    from pa_b200._lib import check, lib
    from pa_b200.device import DeviceBuffer, Stream
    from pa_b200.ring import RingComm, shard, unshard

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    pa_b200.set_device(local)
    comm = RingComm.from_process_group()
    B, H, L, D = 1, 4, 4096, 128
    rng = np.random.default_rng(77)
    q, k, v, do = (rng.standard_normal((B, H, L, D)).astype(np.float16) for _ in range(4))
    sq, sk, sv, sdo = (np.ascontiguousarray(shard(x, world, rank)) for x in (q, k, v, do))
    plan = pa_b200.plan_call(sq.shape, sk.shape, sv.shape, sq.dtype, sk.dtype, sv.dtype,
                             is_causal=True, scale=None)
    st = Stream()
    bufs = {}
    for name, arr in (("q", sq), ("k", sk), ("v", sv), ("do", sdo)):
        bufs[name] = DeviceBuffer(arr.nbytes)
        check(lib().pa_memcpy_h2d(bufs[name].ptr, arr.ctypes.data, arr.nbytes, st.handle))
    for name in ("o", "dq", "dk", "dv"):
        bufs[name] = DeviceBuffer(sq.nbytes)
    bufs["lse"] = DeviceBuffer(B * H * sq.shape[2] * 4)
    # Two calls in a row, the second with phase profiling on: the accumulators
    # and buffers must start clean in every call, and profiling must not change
    # the results.
    for it in range(2):
        if it == 1:
            comm.profile_start()
        comm.forward(plan, bufs["q"].ptr, bufs["k"].ptr, bufs["v"].ptr, bufs["o"].ptr, bufs["lse"].ptr, st)
        comm.backward(plan, bufs["q"].ptr, bufs["k"].ptr, bufs["v"].ptr, bufs["o"].ptr, bufs["do"].ptr,
                      bufs["lse"].ptr, bufs["dq"].ptr, bufs["dk"].ptr, bufs["dv"].ptr, st)
        comm.wait(st, timeout_ms=120000)
    phases = comm.profile_read()
    assert phases["attention"] > 0 and all(v >= 0 for v in phases.values()), phases
    if world > 1:
        assert phases["nccl_transfer"] > 0, phases
    res = {}
    for name in ("o", "dq", "dk", "dv"):
        res[name] = np.empty_like(sq)
        check(lib().pa_memcpy_d2h(res[name].ctypes.data, bufs[name].ptr, sq.nbytes, st.handle))
    res["lse"] = np.empty((B, H, sq.shape[2]), np.float32)
    check(lib().pa_memcpy_d2h(res["lse"].ctypes.data, bufs["lse"].ptr, res["lse"].nbytes, st.handle))
    st.synchronize()
    pa_b200.sync_device_status()
    gathered = [None] * world
    dist.all_gather_object(gathered, res)
    ok = True
    if rank == 0:
        try:
            full = {name: unshard([g[name] for g in gathered], axis=-1 if name == "lse" else -2)
                    for name in res}
            want_o = reference_sdpa(q, k, v, is_causal=True)
            err_o = float(np.max(np.abs(full["o"].astype(np.float64) - want_o)))
            err_l = float(np.max(np.abs(full["lse"] - reference_lse(q, k, is_causal=True))))
            wq, wk, wv = reference_vjp(q, k, v, do, is_causal=True)
            rel = {n: float(np.linalg.norm(full[n].astype(np.float64) - w) / np.linalg.norm(w))
                   for n, w in (("dq", wq), ("dk", wk), ("dv", wv))}
            print(f"ring n={world}: out max abs {err_o:.2e}, lse max abs {err_l:.2e}, grad rel {rel}")
            ok = err_o <= 2e-3 and err_l <= 1e-3 and all(r <= 2e-2 for r in rel.values())
        except Exception as exc:  # noqa: BLE001 -- report, then let every rank exit cleanly
            print(f"ring check failed: {type(exc).__name__}: {exc}")
            ok = False
    flag = [ok]
    dist.broadcast_object_list(flag, src=0)
    comm.close()
    dist.destroy_process_group()
    return 0 if flag[0] else 1


if __name__ == "__main__":
    raise SystemExit(main())
