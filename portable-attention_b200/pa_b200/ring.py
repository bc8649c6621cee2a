"""Ring (context-parallel) causal attention across GPUs: host-side logic.

The reference has no distributed code; this is the long-sequence path of the
backend. A sequence of ``2 n C`` rows is cut into ``2 n`` chunks and rank
``r`` of ``n`` owns chunks ``r`` and ``2n-1-r`` (zig-zag), so every rank gets
the same amount of causal work. Its shard is those two chunks back to back:
``(B, H, 2C, D)``.

In step ``t`` rank ``r`` holds the key/value shard of rank ``(r - t) mod n``
and computes every (query chunk, key chunk) pair with key chunk <= query
chunk (:func:`ring_pairs`); partial outputs merge by log-sum-exp. The native
entry points ``pa_ring_fwd`` / ``pa_ring_bwd`` run that schedule with
NCCL send/recv overlapped with the tensor-core kernels; this module gives the
schedule, the shard layout and the communicator set-up.
"""

from __future__ import annotations

import ctypes

import numpy as np

from ._lib import check, lib

__all__ = ["RingComm", "owned_chunks", "ring_pairs", "shard", "unshard"]


def owned_chunks(n: int, r: int) -> tuple[int, int]:
    """Chunk ids (of ``2n``) that rank ``r`` owns, in shard order."""
    return (r, 2 * n - 1 - r)


def ring_pairs(n: int, r: int, t: int):
    """(query slot, key slot, causal) pairs rank ``r`` computes in step ``t``.

    Slots index the two chunks of a shard (0 = first, 1 = second). The held
    key/value shard at step ``t`` belongs to rank ``(r - t) mod n``.
    """
    src = (r - t) % n
    out = []
    for qs, qid in enumerate(owned_chunks(n, r)):
        for ks, kid in enumerate(owned_chunks(n, src)):
            if kid <= qid:
                out.append((qs, ks, kid == qid))
    return out


def shard(x, n: int, r: int, axis: int = -2):
    """Rank ``r``'s zig-zag shard of ``x`` along the sequence ``axis``."""
    L = x.shape[axis]
    if L % (2 * n):
        raise ValueError(f"sequence length {L} is not a multiple of 2 * {n}")
    c = L // (2 * n)
    a, b = owned_chunks(n, r)
    xa = np.take(x, np.arange(a * c, (a + 1) * c), axis=axis)
    xb = np.take(x, np.arange(b * c, (b + 1) * c), axis=axis)
    return np.concatenate([xa, xb], axis=axis)


def unshard(shards, axis: int = -2):
    """Inverse of :func:`shard` given every rank's shard in rank order."""
    n = len(shards)
    c = shards[0].shape[axis] // 2
    chunks = [None] * (2 * n)
    for r, s in enumerate(shards):
        a, b = owned_chunks(n, r)
        chunks[a] = np.take(s, np.arange(0, c), axis=axis)
        chunks[b] = np.take(s, np.arange(c, 2 * c), axis=axis)
    return np.concatenate(chunks, axis=axis)


class RingComm:
    """An NCCL communicator of the native library, one rank per process/GPU.

    ``from_process_group`` makes the 128-byte NCCL unique id on rank 0 and
    shares it with ``torch.distributed.broadcast_object_list`` (any backend,
    gloo included), then every rank calls ``pa_comm_init``.
    """

    def __init__(self, uid: bytes, nranks: int, rank: int):
        if len(uid) != 128:
            raise ValueError("NCCL unique id must be 128 bytes")
        h = ctypes.c_void_p()
        check(lib().pa_comm_init(ctypes.byref(h), uid, int(nranks), int(rank)))
        self.handle = h.value
        self.nranks, self.rank = int(nranks), int(rank)

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(lib().pa_comm_unique_id(buf))
        return buf.raw

    @classmethod
    def from_process_group(cls, group=None) -> "RingComm":
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        box = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0, group=group)
        return cls(box[0], world, rank)

    def wait(self, stream=None, timeout_ms: int = 60000) -> None:
        """Bounded wait for this rank's ring work; aborts the communicator on failure."""
        check(lib().pa_comm_wait(self.handle, stream.handle if stream is not None else None,
                                 int(timeout_ms)))

    def forward(self, plan, q_ptr, k_ptr, v_ptr, out_ptr, lse_ptr, stream=None) -> None:
        """Enqueue the ring forward on device shards described by ``plan``."""
        check(lib().pa_ring_fwd(self.handle, ctypes.byref(plan.desc), q_ptr, k_ptr, v_ptr, out_ptr,
                                lse_ptr, stream.handle if stream is not None else None))

    def backward(self, plan, q_ptr, k_ptr, v_ptr, out_ptr, dout_ptr, lse_ptr, dq_ptr, dk_ptr, dv_ptr,
                 stream=None) -> None:
        """Enqueue the ring backward (dQ, dK, dV of this rank's shard)."""
        check(lib().pa_ring_bwd(self.handle, ctypes.byref(plan.desc), q_ptr, k_ptr, v_ptr, out_ptr,
                                dout_ptr, lse_ptr, dq_ptr, dk_ptr, dv_ptr,
                                stream.handle if stream is not None else None))

    PHASES = ("repack", "attention", "accumulate", "wait_nccl", "nccl_transfer")

    def profile_start(self) -> None:
        """Start timing the phases of the next ring calls (CUDA events at phase boundaries)."""
        check(lib().pa_comm_profile_start(self.handle))

    def profile_read(self) -> dict:
        """Milliseconds per phase since :meth:`profile_start` (waits for the recorded events).

        ``repack``: chunk copies, fills and output stores on the compute stream;
        ``attention``: the tensor-core kernels of every chunk pair;
        ``accumulate``: fp32 merge / gradient accumulation kernels;
        ``wait_nccl``: time the compute stream stalled waiting for a transfer;
        ``nccl_transfer``: time the side stream spent in NCCL send/recv.
        """
        ms = (ctypes.c_float * len(self.PHASES))()
        check(lib().pa_comm_profile_read(self.handle, ms))
        return dict(zip(self.PHASES, (float(x) for x in ms)))

    def close(self) -> None:
        if self.handle:
            check(lib().pa_comm_destroy(self.handle))
            self.handle = None
