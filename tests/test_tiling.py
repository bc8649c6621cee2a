"""The B200 entry for the reference's tile planner (no GPU needed)."""

from __future__ import annotations

import pytest


def test_b200_limits_in_the_reference_vocabulary():
    from pa_b200.tiling import B200_LIMITS

    assert (B200_LIMITS.shared_memory_bytes, B200_LIMITS.max_threads_per_group, B200_LIMITS.simd_width) == (
        232448, 1024, 32)
    assert "B200" in B200_LIMITS.name


def test_mirror_rejects_what_the_reference_rejects():
    from pa_b200.tiling import DeviceLimitsMirror

    with pytest.raises(ValueError, match="power of two"):
        DeviceLimitsMirror(1024, 256, 24)
    with pytest.raises(ValueError, match="positive integer"):
        DeviceLimitsMirror(1024.0, 256, 32)
    with pytest.raises(ValueError, match="at least simd_width"):
        DeviceLimitsMirror(1024, 16, 32)


@pytest.mark.parametrize("d,k_stages,v_stages", [(128, 2, 3), (64, 3, 4)])
def test_tcgen05_plan_matches_the_kernel(d, k_stages, v_stages):
    from pa_b200.tiling import plan_tcgen05_tiles

    p = plan_tcgen05_tiles(d, 2)
    assert (p.block_q, p.block_k, p.query_tiles, p.tmem_columns) == (128, 128, 2, 512)
    assert (p.k_stages, p.v_stages) == (k_stages, v_stages)
    # Q tiles + K/V stages + barriers: the layout fits the B200's 227 KB per CTA.
    assert p.shared_memory_bytes >= (2 * 128 + (k_stages + v_stages) * 128) * d * 2
    assert 0.5 < p.shared_memory_utilization <= 1.0
    assert p.subgroups_per_group == p.threads_per_group / 32
    assert p.q_tiles(4096) == 32 and p.k_tiles(4097) == 33


@pytest.mark.parametrize("d,b", [(96, 2), (128, 4), (64, 1)])
def test_shapes_without_a_tensor_core_plan(d, b):
    from pa_b200.tiling import TileSizingError, plan_tcgen05_tiles

    with pytest.raises(TileSizingError):
        plan_tcgen05_tiles(d, b)
