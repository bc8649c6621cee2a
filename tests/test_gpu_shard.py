"""pa_shard_fwd: one call spread over several GPUs (or several streams of one GPU).

Shards run the same kernels on rows of the first leading dimension, so every
forward row must be bit-identical to the single-GPU call. A device index may
repeat (two host threads driving one GPU), which exercises the sharding logic
-- boundaries, grouped-query heads on the first axis, masks broadcast over or
indexed by the batch -- on a one-GPU box; the last test uses two GPUs when
present.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle.sdpa import reference_sdpa

pytestmark = pytest.mark.gpu


def _inputs(rng, qs, ks, dtype=np.float16):
    return (rng.standard_normal(qs).astype(dtype), rng.standard_normal(ks).astype(dtype),
            rng.standard_normal(ks).astype(dtype))


@pytest.mark.parametrize("devices", [[0], [0, 0], [0, 0, 0]])
def test_causal_gqa_shards_are_bit_identical(devices):
    import pa_b200

    q, k, v = _inputs(np.random.default_rng(1), (5, 8, 300, 128), (5, 2, 300, 128))
    want = pa_b200.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
    got = pa_b200.sdpa_sharded(q, k, v, is_causal=True, enable_gqa=True, devices=devices)
    np.testing.assert_array_equal(got, want)


def test_grouped_heads_on_the_first_axis_stay_together():
    import pa_b200

    q, k, v = _inputs(np.random.default_rng(2), (8, 200, 64), (2, 200, 64))
    want = pa_b200.scaled_dot_product_attention(q, k, v, enable_gqa=True)
    got = pa_b200.sdpa_sharded(q, k, v, enable_gqa=True, devices=[0, 0, 0])
    np.testing.assert_array_equal(got, want)
    np.testing.assert_allclose(got.astype(np.float64), reference_sdpa(q, k, v, enable_gqa=True),
                               rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("mask_shape", [(1, 1, 160, 224), (4, 1, 160, 224), (4, 3, 160, 224)])
def test_masks_broadcast_or_indexed_by_batch(mask_shape):
    import pa_b200

    rng = np.random.default_rng(3)
    q, k, v = _inputs(rng, (4, 3, 160, 64), (4, 3, 224, 64))
    m = rng.random(mask_shape) < 0.7
    want = pa_b200.scaled_dot_product_attention(q, k, v, attn_mask=m)
    got = pa_b200.sdpa_sharded(q, k, v, attn_mask=m, devices=[0, 0])
    np.testing.assert_array_equal(got, want)


def test_float32_exact_kernel_and_decode_through_shards():
    import pa_b200

    rng = np.random.default_rng(4)
    q, k, v = _inputs(rng, (3, 4, 50, 24), (3, 4, 70, 24), np.float32)
    got = pa_b200.sdpa_sharded(q, k, v, devices=[0, 0])
    np.testing.assert_allclose(got, reference_sdpa(q, k, v), rtol=1e-4, atol=1e-5)
    q, k, v = _inputs(rng, (6, 16, 1, 128), (6, 4, 3000, 128))
    got = pa_b200.sdpa_sharded(q, k, v, enable_gqa=True, devices=[0, 0, 0])
    np.testing.assert_allclose(got.astype(np.float64), reference_sdpa(q, k, v, enable_gqa=True),
                               rtol=2e-3, atol=2e-3)


def test_two_gpus():
    import pa_b200

    if pa_b200.device_count() < 2:
        pytest.skip("needs two GPUs")
    q, k, v = _inputs(np.random.default_rng(5), (4, 8, 512, 128), (4, 2, 512, 128))
    want = pa_b200.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
    got = pa_b200.sdpa_sharded(q, k, v, is_causal=True, enable_gqa=True, devices=[0, 1])
    np.testing.assert_array_equal(got, want)
