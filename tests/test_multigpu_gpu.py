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


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["marker", "silent"])
def test_rank_loss_between_steps_is_detected_on_the_host(mode):
    """A rank leaves between steps of the fused 2-GPU run (no kernel of its in flight); the survivor
    finds it with the heartbeat watchdog before its next launch and exits cleanly.  NVLS is off and
    the fused kernels use plain peer loads, so no memory is bound to a multicast object."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT, RANK_LOSS_MODE=mode, LEAVE_AFTER="3")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           "-m", "flare_b200.testing.rank_loss_check"]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    out = res.stdout + res.stderr
    assert "[rank0] RANK_LOSS_DETECTED ranks=[1] after step 3" in out, out[-4000:]
    assert "[rank1] leaving after step 3" in out, out[-4000:]
    assert "NO_DETECTION" not in out, out[-4000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_accumulation_windows_and_staleness_two_on_two_gpus():
    import os
    import socket
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=root)
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           "-m", "flare_b200.testing.dlrm_policy_dist_check"]
    res = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=450)
    assert res.returncode == 0 and "POLICY_DIST_OK" in res.stdout, (res.stdout + res.stderr)[-5000:]
