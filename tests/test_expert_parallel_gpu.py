"""Expert parallelism over NCCL on 2+ GPUs (skipped with fewer): the partitioned routed experts are
bitwise equal to the single-GPU path, for 1, 5 and 32 tokens per rank."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_expert_parallel_two_gpus():
    n = 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", "29631", os.path.join(HERE, "ep_gpu_worker.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert res.returncode == 0 and "EP_OK" in res.stdout, res.stdout[-3000:] + res.stderr[-3000:]
