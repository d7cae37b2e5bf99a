"""Expert parallelism over NCCL on 2, 4 and 8 GPUs (each case skipped with fewer): the partitioned
routed experts are bitwise equal to the single-GPU path, for 1, 5 and 32 tokens per rank."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("n", [2, 4, 8])
def test_expert_parallel(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", str(29631 + n), os.path.join(HERE, "ep_gpu_worker.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert res.returncode == 0 and "EP_OK" in res.stdout, res.stdout[-3000:] + res.stderr[-3000:]
