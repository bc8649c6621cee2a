"""Multi-GPU ring attention, run as a 2- and a 4-rank torchrun job (needs that many GPUs).

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


@pytest.mark.parametrize("ranks", [2, 4])
def test_ring_multi_gpu(ranks):
    import pa_b200

    if pa_b200.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={ranks}", "--master-addr", "127.0.0.1",
           "--master-port", str(29533 + ranks), str(ROOT / "tests" / "ring_worker.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    print(res.stdout[-3000:], res.stderr[-3000:])
    assert res.returncode == 0
