"""The device-side failure path, made to run out on purpose (needs a GPU).

Every pipelined kernel of the library waits on mbarriers through one bounded
routine: after a time limit it records a code in the device status word,
raises the CTA's abort flag so the other warps stop, and returns, so a lost
tile or a stuck producer ends in an error instead of a hang. Here
``pa_selftest_wait_timeout`` runs that routine on a barrier nothing arrives
on, with a 1 ms limit: the launch must finish by itself, the status word must
carry the time-out code (0x105), the Python layer must raise, and the context
must stay usable for the next call. Nothing faults, traps or hangs: the wait
is bounded and the kernel returns normally.

The reference's analogue is its bounded fence wait
(``src/portable_attention/vkcompute.py:1031-1042``).
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports():
    import pa_b200
    from pa_b200._lib import PA_ERR_TIMEOUT, PaError, check, lib
    from pa_b200.device import Stream

    pa_b200.set_device(0)
    pa_b200.sync_device_status()          # start from a clear status word
    st = Stream()
    t0 = time.perf_counter()
    check(lib().pa_selftest_wait_timeout(1000, st.handle))
    st.synchronize()
    elapsed = time.perf_counter() - t0
    # Warp 0 gives up after 1 ms; warp 1 (2 s bound) must leave through the
    # abort flag right after, so the launch ends far below the 2 s bound.
    assert elapsed < 1.0, f"self-test took {elapsed:.3f} s"

    code = ctypes.c_int32(0)
    rc = lib().pa_device_status(ctypes.byref(code))
    assert rc == PA_ERR_TIMEOUT and code.value == 0x105
    assert b"gave up" in lib().pa_last_error()
    # The status word is read-and-clear: a second read is clean.
    assert lib().pa_device_status(ctypes.byref(code)) == 0 and code.value == 0

    # Through the Python layer: the same give-up surfaces as an exception.
    check(lib().pa_selftest_wait_timeout(1000, st.handle))
    st.synchronize()
    with pytest.raises(PaError) as err:
        pa_b200.sync_device_status()
    assert err.value.status == PA_ERR_TIMEOUT

    # The context is still usable: a normal call right after gives correct output.
    from oracle.sdpa import reference_sdpa

    rng = np.random.default_rng(9)
    q = rng.standard_normal((1, 2, 130, 64)).astype(np.float16)
    k = rng.standard_normal((1, 2, 200, 64)).astype(np.float16)
    v = rng.standard_normal((1, 2, 200, 64)).astype(np.float16)
    got = pa_b200.scaled_dot_product_attention(q, k, v, is_causal=True)
    want = reference_sdpa(q, k, v, is_causal=True)
    np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=2e-3, atol=2e-3)
