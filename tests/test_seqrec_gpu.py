"""Sequential model fused path vs PyTorch: 1 GPU in-process, 2 GPUs (FSDP over both) under torchrun."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_seqrec_single_gpu_matches_torch(cuda):
    from flare_b200.testing.seqrec_check import run

    assert run() == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_seqrec_two_gpus_matches_torch():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", "-m", "flare_b200.testing.seqrec_check"]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    if res.returncode != 0 or "SEQREC_OK" not in res.stdout:
        raise AssertionError((res.stdout + res.stderr)[-6000:])
