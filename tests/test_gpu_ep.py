"""GPU, 2+ devices: expert-parallel forward (peer-memory and collective
transports) against the CPU oracle over all 256 experts (tests/ep_gpu_check.py
under torchrun, NVLS off). Skipped when the machine has fewer than two GPUs."""
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_matches_single_gpu():
    world = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", "--master-port=29531", str(ROOT / "tests" / "ep_gpu_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    lines = [l for l in r.stdout.splitlines() if l.startswith("EP_CHECK")]
    print("\n".join(lines))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert len(lines) == world and all("ok=True" in l for l in lines)
