"""A save that dies mid-way leaves the last complete step in charge; a rerun finishes the job."""
import subprocess
import sys
from pathlib import Path

from flare_b200.checkpoint.store import CheckpointManager, latest_step, list_steps
from flare_b200.testing.ckpt_crash import CpuModel

ROOT = Path(__file__).resolve().parents[1]


def _run(root, phase):
    return subprocess.run([sys.executable, "-m", "flare_b200.testing.ckpt_crash", str(root), phase], cwd=ROOT,
                          capture_output=True, text=True, timeout=300)


def test_crash_inside_a_save_keeps_the_last_complete_step(tmp_path):
    assert _run(tmp_path, "first").returncode == 0
    assert latest_step(tmp_path) == 10

    r = _run(tmp_path, "crash")
    assert r.returncode == 86, r.stderr
    assert list_steps(tmp_path) == [10]  # the half-written step is not a step
    assert (tmp_path / "steps" / "20.partial" / "model").is_dir()

    after_crash = CpuModel()
    assert CheckpointManager(str(tmp_path)).restore(after_crash) == 10
    expect10 = CpuModel()
    expect10.run(1, 10)
    assert after_crash.digest() == expect10.digest()

    r = _run(tmp_path, "resume")
    assert r.returncode == 0, r.stderr
    assert list_steps(tmp_path) == [10, 20] and not (tmp_path / "steps" / "20.partial").exists()
    restored = CpuModel()
    assert CheckpointManager(str(tmp_path)).restore(restored) == 20
    expect20 = CpuModel()
    expect20.run(1, 20)
    got, want = restored.digest(), expect20.digest()
    assert all(abs(a - b) <= 1e-5 * max(1.0, abs(b)) for a, b in zip(got, want)), (got, want)
