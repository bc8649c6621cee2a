"""Ring attention host logic on CPU: shards, schedule, merge, and a 2-rank gloo run.

The GPU ring (``pa_ring_fwd`` / ``pa_ring_bwd``) follows the schedule of
``pa_b200.ring.ring_pairs``. Here that schedule is checked for coverage, the
float64 simulation of the whole ring (``oracle/ring.py``) is checked against
the oracle forward and VJP on the gathered sequence for 1-4 ranks, and a
world-size-2 ``gloo`` job runs the same algorithm with real point-to-point
messages between processes (the forward, and the backward in the native
schedule's message order, accumulators travelling with their key/value block
and coming home after the last step) and the NCCL-id exchange of ``RingComm``
against a fake native library.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from oracle.ring import block_attention, block_grads, simulate_ring
from oracle.sdpa import reference_sdpa
from oracle.vjp import reference_vjp
from pa_b200.ring import owned_chunks, ring_pairs, shard, unshard


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_shard_roundtrip_and_balance(n):
    x = np.arange(2 * n * 3 * 5).reshape(2 * n * 3, 5)[None]
    parts = [shard(x, n, r) for r in range(n)]
    np.testing.assert_array_equal(unshard(parts), x)
    assert sorted(c for r in range(n) for c in owned_chunks(n, r)) == list(range(2 * n))


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_schedule_covers_every_causal_pair_once(n):
    for r in range(n):
        seen = []
        for t in range(n):
            src = (r - t) % n
            for qs, ks, causal in ring_pairs(n, r, t):
                qid, kid = owned_chunks(n, r)[qs], owned_chunks(n, src)[ks]
                assert kid <= qid and causal == (kid == qid)
                seen.append((qid, kid))
        want = sorted((qid, kid) for qid in owned_chunks(n, r) for kid in range(2 * n) if kid <= qid)
        assert sorted(seen) == want
    # Zig-zag balance: every rank computes the same number of full-chunk-equivalents.
    work = [sum((0.5 if c else 1.0) for t in range(n) for _, _, c in ring_pairs(n, r, t)) for r in range(n)]
    assert max(work) == min(work)


@pytest.mark.parametrize("n", [1, 2, 3, 4])
def test_simulated_ring_matches_oracle(n):
    rng = np.random.default_rng(n)
    B, H, C, D = 1, 2, 3, 8
    L = 2 * n * C
    q, k, v, do = (rng.standard_normal((B, H, L, D)) for _ in range(4))
    sh = lambda x: [shard(x, n, r) for r in range(n)]  # noqa: E731
    outs, lses, grads = simulate_ring(sh(q), sh(k), sh(v), n, ring_pairs, do=sh(do))
    np.testing.assert_allclose(unshard(outs), reference_sdpa(q, k, v, is_causal=True), rtol=1e-12, atol=1e-12)
    wq, wk, wv = reference_vjp(q, k, v, do, is_causal=True)
    for i, want in enumerate((wq, wk, wv)):
        np.testing.assert_allclose(unshard([g[i] for g in grads]), want, rtol=1e-10, atol=1e-12)


# ------------------------------------------------------------- gloo, 2 ranks

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _FakeLib:
    """Stands in for libpa_b200 so the id exchange runs without a GPU."""

    def __init__(self):
        self.init_args = None

    def pa_comm_unique_id(self, buf):
        buf[:] = bytes(range(128))[::-1]
        return 0

    def pa_comm_init(self, handle_ref, uid, nranks, rank):
        self.init_args = (bytes(uid), nranks, rank)
        return 0


def _worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    import pa_b200.ring as ring_mod

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        # NCCL id exchange through RingComm against a fake native library.
        fake = _FakeLib()
        ring_mod.lib = lambda: fake
        comm = ring_mod.RingComm.from_process_group()
        got = [None] * world
        dist.all_gather_object(got, fake.init_args)
        assert comm.nranks == world and comm.rank == rank
        assert all(g[0] == bytes(range(128))[::-1] and g[1] == world for g in got)
        assert sorted(g[2] for g in got) == list(range(world))

        # The ring itself, with real messages: K/V shards travel r -> r+1.
        rng = np.random.default_rng(123)
        B, H, C, D = 1, 2, 4, 8
        n = world
        q, k, v = (rng.standard_normal((B, H, 2 * n * C, D)) for _ in range(3))
        scale = 1 / np.sqrt(D)
        qs, ks, vs = shard(q, n, rank), shard(k, n, rank), shard(v, n, rank)
        held = torch.from_numpy(np.concatenate([ks, vs], axis=-1).copy())
        acc_o = np.zeros(qs.shape)
        acc_l = np.full(qs.shape[:-1], -np.inf)
        for t in range(n):
            kv = held.numpy()
            hk, hv = kv[..., :D], kv[..., D:]
            if t + 1 < n:
                nxt = torch.empty_like(held)
                reqs = [dist.isend(held, (rank + 1) % n), dist.irecv(nxt, (rank - 1) % n)]
            for qsl, ksl, causal in ring_pairs(n, rank, t):
                qq = qs[..., qsl * C:(qsl + 1) * C, :]
                w, tot, lse = block_attention(qq, hk[..., ksl * C:(ksl + 1) * C, :], causal, scale)
                part = w @ hv[..., ksl * C:(ksl + 1) * C, :] / tot
                rows = slice(qsl * C, (qsl + 1) * C)
                la = acc_l[..., rows]
                m = np.maximum(la, lse)
                wa = np.where(np.isfinite(la), np.exp(la - m), 0.0)
                wb = np.exp(lse - m)
                acc_o[..., rows, :] = (acc_o[..., rows, :] * wa[..., None] + part * wb[..., None]) / (wa + wb)[..., None]
                acc_l[..., rows] = m + np.log(wa + wb)
            if t + 1 < n:
                for rq in reqs:
                    rq.wait()
                held = nxt
        outs = [None] * world
        dist.all_gather_object(outs, acc_o)
        if rank == 0:
            np.testing.assert_allclose(unshard(outs), reference_sdpa(q, k, v, is_causal=True),
                                       rtol=1e-12, atol=1e-12)

        # Backward with the native message schedule (csrc/ring.cu pa_ring_bwd): per step
        # the K/V group for the next step, this step's pairs, then one group that sends the
        # held block's dK/dV accumulators on to r+1 and receives, from r-1, those of the
        # block held next (after the last step: this rank's own block, home).
        do = rng.standard_normal(q.shape)
        dos = shard(do, n, rank)
        held = torch.from_numpy(np.concatenate([ks, vs], axis=-1).copy())
        acc = torch.zeros_like(held)          # dK | dV of the held block
        dq = np.zeros(qs.shape)
        for t in range(n):
            if t + 1 < n:
                nxt = torch.empty_like(held)
                kv_reqs = [dist.isend(held, (rank + 1) % n), dist.irecv(nxt, (rank - 1) % n)]
            kv = held.numpy()
            hk, hv = kv[..., :D], kv[..., D:]
            a = acc.numpy()
            for qsl, ksl, causal in ring_pairs(n, rank, t):
                rows = slice(qsl * C, (qsl + 1) * C)
                cols = slice(ksl * C, (ksl + 1) * C)
                gq, gk, gv = block_grads(qs[..., rows, :], hk[..., cols, :], hv[..., cols, :],
                                         dos[..., rows, :], acc_o[..., rows, :], acc_l[..., rows],
                                         causal, scale)
                dq[..., rows, :] += gq
                a[..., cols, :D] += gk
                a[..., cols, D:] += gv
            if n > 1:
                nacc = torch.empty_like(acc)
                acc_reqs = [dist.isend(acc, (rank + 1) % n), dist.irecv(nacc, (rank - 1) % n)]
                for rq in acc_reqs:
                    rq.wait()
                acc = nacc
            if t + 1 < n:
                for rq in kv_reqs:
                    rq.wait()
                held = nxt
        grads = [None] * world
        dist.all_gather_object(grads, (dq, acc.numpy()[..., :D].copy(), acc.numpy()[..., D:].copy()))
        if rank == 0:
            wq, wk, wv = reference_vjp(q, k, v, do, is_causal=True)
            for i, want in enumerate((wq, wk, wv)):
                np.testing.assert_allclose(unshard([g[i] for g in grads]), want, rtol=1e-10, atol=1e-12)
            with open(result_path, "w") as f:
                f.write("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ring(tmp_path, world):
    import torch.multiprocessing as mp

    result = tmp_path / "result.txt"
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.start_processes(_worker, args=(world, _free_port(), str(result)), nprocs=world, join=True,
                       start_method="spawn")
    assert result.read_text() == "ok"


def test_ring_profile_phases_map_to_names(monkeypatch):
    """RingComm.profile_read returns the five phase times in include/pa_b200.h's
    PA_RING_PHASE_* order (checked against a fake native library)."""
    import ctypes

    import pa_b200.ring as ring_mod

    calls = []

    class Fake:
        def pa_comm_init(self, handle_ref, uid, nranks, rank):
            return 0

        def pa_comm_profile_start(self, handle):
            calls.append("start")
            return 0

        def pa_comm_profile_read(self, handle, ms):
            arr = ctypes.cast(ms, ctypes.POINTER(ctypes.c_float * 5)).contents
            for i, v in enumerate((1.5, 100.0, 2.0, 3.0, 40.0)):
                arr[i] = v
            calls.append("read")
            return 0

    monkeypatch.setattr(ring_mod, "lib", lambda: Fake())
    comm = ring_mod.RingComm(bytes(128), 2, 0)
    comm.handle = 1
    comm.profile_start()
    got = comm.profile_read()
    assert calls == ["start", "read"]
    assert got == {"repack": 1.5, "attention": 100.0, "accumulate": 2.0, "wait_nccl": 3.0,
                   "nccl_transfer": 40.0}
    comm.handle = None
