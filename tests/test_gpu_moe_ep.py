"""Expert-parallel MoE on 2 GPUs (NCCL all-to-all over NVLink) against the
single-GPU model: data-parallel blocks (batch 2: one sequence per rank) and
half-sequence blocks (batch 1: the second rank all-gathers K/V and runs the
causal block mask). Skipped on hosts with fewer than 2 GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("batch", [2, 1])
def test_expert_parallel_matches_single_gpu(batch):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(29600 + batch),
           str(ROOT / "tests" / "ep_check.py"), str(batch)]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    print(res.stdout[-3000:], res.stderr[-3000:])
    assert res.returncode == 0
