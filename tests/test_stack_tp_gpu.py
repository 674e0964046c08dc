"""Tensor-parallel stack on two GPUs, with the all-gathers done by the library's peer-store
kernel, by the O and down projections' own epilogues (fused) and by NCCL: the plan graph
equals eager steps and the residual stream equals the single-GPU stack's, bit for bit (skipped
with fewer than two GPUs)."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("exchange,port", [("fused", 29519), ("peer", 29517), ("nccl", 29518)])
def test_two_gpu_stack_matches_single_gpu(cuda, exchange, port):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, PYTHONPATH=os.path.join(REPO, "specdec-quant-triton_b200"), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "specq.stack_tp",
           "--layers", "2", "--steps", "20", "--b-max", "8", "--check", "--exchange", exchange]
    out = subprocess.run(cmd, env=env, cwd=REPO, capture_output=True, text=True, timeout=700)
    assert out.returncode == 0, out.stderr[-3000:]
    res = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith("{")][-1])
    assert res["plan_vs_eager_max_abs_diff"] == 0.0
    assert res["tp_vs_single_gpu_max_abs_diff"] == 0.0
