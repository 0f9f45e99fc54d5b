"""GPU (2+ devices): sequence parallelism over NCCL, one process per GPU, against
the single-GPU full-sequence call (bf16 tolerance 2e-2). Skipped with one GPU."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_seq_parallel_two_ranks(native_lib):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29577", os.path.join(ROOT, "tests", "seqpar_worker.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert "SEQPAR_OK" in out.stdout, out.stdout[-2000:] + out.stderr[-3000:]
