"""B200 entry for the reference's tile planner, and the tcgen05 tile plan.

The reference sizes blocked-attention tiles from three device numbers
(``DeviceLimits``, ``src/portable_attention/tiling.py:68-102``) and returns a
``TilePlan`` (``tiling.py:125-166``) for a thread-per-score kernel that keeps
Q, K, V and the score tile in shared memory. This module gives

* :data:`B200_LIMITS` -- the B200's numbers in that vocabulary: 232,448 bytes
  of shared memory per CTA (227 KB opt-in), 1,024 threads per CTA, 32-wide
  warps. It is the reference's own ``DeviceLimits`` when ``portable_attention``
  is importable, otherwise a field-for-field mirror with the same checks.
* :func:`plan_tcgen05_tiles` -- the tile shape the tensor-core forward of this
  package actually compiles (two 128-row query tiles per CTA, 128-key K/V
  tiles streamed by TMA, accumulators in TMEM), read from the native library
  (``pa_fwd_tile_plan``) so the plan cannot drift from the kernel. The
  reference's thread-per-score layout does not describe it: scores live in
  tensor memory, not shared memory, and one thread owns a query row.

Nothing in the reference consumes a plan for this backend; these exist so a
caller of ``plan_tiles`` can reason about the B200 in the same terms.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

__all__ = ["B200_LIMITS", "DeviceLimitsMirror", "Tcgen05TilePlan", "TileSizingError",
           "plan_tcgen05_tiles"]


class TileSizingError(ValueError):
    """Raised when the tensor-core forward has no tile plan for a shape (``tiling.py:48``)."""


def _require_positive_int(name: str, value: object) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
        raise ValueError(f"{name} must be a positive integer, got {value!r}")
    return value


@dataclass(frozen=True)
class DeviceLimitsMirror:
    """Same fields and checks as the reference's ``DeviceLimits`` (``tiling.py:68-102``)."""

    shared_memory_bytes: int
    max_threads_per_group: int
    simd_width: int
    name: str = ""

    def __post_init__(self) -> None:
        for field, value in (("shared_memory_bytes", self.shared_memory_bytes),
                             ("max_threads_per_group", self.max_threads_per_group),
                             ("simd_width", self.simd_width)):
            _require_positive_int(field, value)
        if self.simd_width & (self.simd_width - 1):
            raise ValueError(f"simd_width must be a power of two, got {self.simd_width}")
        if self.max_threads_per_group < self.simd_width:
            raise ValueError("max_threads_per_group must be at least simd_width "
                             f"({self.max_threads_per_group} < {self.simd_width})")


_B200 = dict(shared_memory_bytes=232448, max_threads_per_group=1024, simd_width=32,
             name="NVIDIA B200 (sm_100a)")


def _limits():
    try:
        from portable_attention.tiling import DeviceLimits  # the reference, when installed
    except ImportError:
        return DeviceLimitsMirror(**_B200)
    return DeviceLimits(**_B200)


B200_LIMITS = _limits()


class _PlanC(ctypes.Structure):
    """Mirror of ``pa_tile_plan`` (include/pa_b200.h)."""

    _fields_ = [(n, ctypes.c_int32) for n in ("block_q", "block_k", "query_tiles", "threads",
                                               "shared_memory_bytes", "tmem_columns", "k_stages",
                                               "v_stages")]


@dataclass(frozen=True)
class Tcgen05TilePlan:
    """The reference's ``TilePlan`` fields (``tiling.py:125-145``) plus what tcgen05 adds.

    ``threads_per_group`` and ``shared_memory_bytes`` are per CTA; a CTA holds
    ``query_tiles`` query tiles of ``block_q`` rows and streams ``block_k``-key
    K/V tiles through ``k_stages`` / ``v_stages`` shared-memory stages.
    """

    block_q: int
    block_k: int
    threads_per_group: int
    shared_memory_bytes: int
    head_dim: int
    dtype_bytes: int
    limits: object
    query_tiles: int
    tmem_columns: int
    k_stages: int
    v_stages: int

    @property
    def shared_memory_utilization(self) -> float:
        """Fraction of the device's shared memory the CTA occupies (``tiling.py:147-150``)."""
        return self.shared_memory_bytes / self.limits.shared_memory_bytes

    @property
    def subgroups_per_group(self) -> float:
        """CTA size in warps (``tiling.py:152-159``)."""
        return self.threads_per_group / self.limits.simd_width

    def q_tiles(self, seq_len_q: int) -> int:
        """Query tiles needed to cover ``seq_len_q`` rows (``tiling.py:161-163``)."""
        _require_positive_int("seq_len_q", seq_len_q)
        return -(-seq_len_q // self.block_q)

    def k_tiles(self, seq_len_k: int) -> int:
        """Streaming steps needed to cover ``seq_len_k`` keys (``tiling.py:165-167``)."""
        _require_positive_int("seq_len_k", seq_len_k)
        return -(-seq_len_k // self.block_k)


def plan_tcgen05_tiles(head_dim: int, dtype_bytes: int, limits=B200_LIMITS) -> Tcgen05TilePlan:
    """The tile plan of the tensor-core forward for ``head_dim`` and ``dtype_bytes``.

    Raises :class:`TileSizingError` when the kernel does not take the shape
    (those calls run on the exact CUDA-core kernel) or when the plan does not
    fit ``limits``.
    """
    from ._lib import lib

    _require_positive_int("head_dim", head_dim)
    _require_positive_int("dtype_bytes", dtype_bytes)
    p = _PlanC()
    if lib().pa_fwd_tile_plan(head_dim, dtype_bytes, ctypes.byref(p)) != 0:
        raise TileSizingError(
            f"the tensor-core forward has no tile plan for head_dim={head_dim}, "
            f"dtype_bytes={dtype_bytes}: {(lib().pa_last_error() or b'').decode()}")
    plan = Tcgen05TilePlan(block_q=p.block_q, block_k=p.block_k, threads_per_group=p.threads,
                           shared_memory_bytes=p.shared_memory_bytes, head_dim=head_dim,
                           dtype_bytes=dtype_bytes, limits=limits, query_tiles=p.query_tiles,
                           tmem_columns=p.tmem_columns, k_stages=p.k_stages, v_stages=p.v_stages)
    if plan.shared_memory_bytes > limits.shared_memory_bytes or plan.threads_per_group > limits.max_threads_per_group:
        raise TileSizingError(f"the tcgen05 plan ({plan.shared_memory_bytes} B, {plan.threads_per_group} "
                              f"threads) does not fit {limits.name or 'the device'}")
    return plan
