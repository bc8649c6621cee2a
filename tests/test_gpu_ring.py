"""Multi-GPU ring attention, run as a 2-rank torchrun job (needs >= 2 GPUs).

The job (``tests/ring_worker.py``) checks the gathered ring forward output,
lse and the ring backward gradients against the float64 oracle. On a
single-GPU host this test is skipped; the host-side schedule is covered by
``tests/test_ring_host.py`` on CPU.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_ring_two_gpus():
    import pa_b200

    if pa_b200.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", "29533", str(ROOT / "tests" / "ring_worker.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    print(res.stdout[-3000:], res.stderr[-3000:])
    assert res.returncode == 0
