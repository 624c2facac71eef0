"""Job bundles (CPU): tracked sources + one built extension, digest manifest, tamper detection,
safe extraction and the one-node launch line."""
import json
import subprocess
import zipfile

import pytest

from flare_b200.runtime.bundle import build_bundle, bundle_paths, extract_bundle, launch_command, verify_bundle


def _repo(tmp_path):
    r = tmp_path / "repo"
    (r / "flare_b200").mkdir(parents=True)
    (r / "flare_b200" / "__init__.py").write_text("x = 1\n")
    (r / "flare_b200" / "untracked.py").write_text("y = 2\n")
    (r / "bench.py").write_text("print('bench')\n")
    git = lambda *a: subprocess.run(["git", *a], cwd=r, check=True, capture_output=True)  # noqa: E731
    git("init", "-q")
    git("add", "flare_b200/__init__.py", "bench.py")
    git("-c", "user.name=t", "-c", "user.email=t@t", "commit", "-qm", "init")
    return r


def test_bundle_round_trip_and_tamper_detection(tmp_path):
    r = _repo(tmp_path)
    with pytest.raises(RuntimeError, match="native extension"):
        bundle_paths(r, ("flare_b200", "bench.py"))
    import importlib.machinery

    so = r / "flare_b200" / ("_C" + importlib.machinery.EXTENSION_SUFFIXES[0])
    so.write_bytes(b"\x7fELF fake")
    files = bundle_paths(r, ("flare_b200", "bench.py"))
    assert "flare_b200/untracked.py" not in files and so.relative_to(r).as_posix() in files
    z = build_bundle(r, tmp_path / "out", paths=("flare_b200", "bench.py"))
    man = verify_bundle(z)
    assert man["clean"] and set(man["members"]) == set(files)
    root = extract_bundle(z, tmp_path / "x")
    assert (root / "bench.py").read_text() == "print('bench')\n"
    cmd = launch_command(root, "bench.py", nproc_per_node=8, args=["--gpus", "8"])
    assert "--master-addr=127.0.0.1" in cmd and cmd[-3:] == [str(root / "bench.py"), "--gpus", "8"]
    assert launch_command(root, "-m flare_b200.cli", nproc_per_node=2)[-2:] == ["-m", "flare_b200.cli"]
    # a modified member fails verification
    bad = tmp_path / "bad.zip"
    with zipfile.ZipFile(z) as src, zipfile.ZipFile(bad, "w") as dst:
        for n in src.namelist():
            data = src.read(n)
            dst.writestr(n, b"print('evil')\n" if n == "bench.py" else data)
    with pytest.raises(ValueError, match="digest"):
        verify_bundle(bad)
    json.loads(zipfile.ZipFile(z).read("BUNDLE.json"))


def test_symlinks_are_refused(tmp_path):
    r = _repo(tmp_path)
    import importlib.machinery

    (r / "flare_b200" / ("_C" + importlib.machinery.EXTENSION_SUFFIXES[0])).write_bytes(b"so")
    (r / "flare_b200" / "link.py").symlink_to(r / "bench.py")
    subprocess.run(["git", "add", "flare_b200/link.py"], cwd=r, check=True)
    with pytest.raises(ValueError, match="symbolic link"):
        bundle_paths(r, ("flare_b200",))
