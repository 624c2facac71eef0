"""2-GPU equivalence of the fused sharded path (skipped with fewer than 2 GPUs)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_matches_single_gpu_on_global_batch():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", "-m", "flare_b200.testing.dist_dlrm_check"]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    if res.returncode != 0 or "DIST_OK" not in res.stdout:
        lines = [ln for ln in (res.stdout + res.stderr).splitlines() if "[rank" in ln or "Error" in ln or "diff" in ln]
        raise AssertionError("\n".join(lines[-80:]))
