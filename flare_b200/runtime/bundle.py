"""Job bundles: the tracked sources and the built native extension in one verifiable archive.

``build_bundle(repo, out_dir)`` packs the git-tracked files under the
selected paths plus exactly one built ``flare_b200/_C`` extension into a
zip whose ``BUNDLE.json`` lists every member with its SHA-256, the git
commit and whether the tree was clean; symbolic links are refused.
``verify_bundle`` re-hashes an archive against its manifest and
``extract_bundle`` unpacks a verified archive.  ``launch_command`` gives
the ``torch.distributed.run`` command that starts a job from an extracted
bundle on one node (one process per GPU, rendezvous on 127.0.0.1).

Reference behaviour: recipes/recsys/data/submit_job.py (git-tracked sources
plus the two native modules, zipped for a Ray job); here the launcher is
``torch.distributed.run``.
"""
from __future__ import annotations

import hashlib
import importlib.machinery
import json
import subprocess
import sys
import zipfile
from collections.abc import Sequence
from pathlib import Path

MANIFEST = "BUNDLE.json"
DEFAULT_PATHS = ("flare_b200", "bench.py", "setup.py", "__graft_entry__.py")
NATIVE_MODULES = ("flare_b200/_C",)


def _git(repo: Path, *args: str) -> str:
    return subprocess.run(["git", *args], cwd=repo, check=True, capture_output=True, text=True).stdout


def _sha256(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def bundle_paths(repo: str | Path, paths: Sequence[str] = DEFAULT_PATHS,
                 native_modules: Sequence[str] = NATIVE_MODULES) -> list[str]:
    """Tracked files under ``paths`` plus one built extension per native module (sorted, repo-relative)."""
    repo = Path(repo)
    out = {p for p in _git(repo, "ls-files", "-z", "--", *paths).split("\0") if p}
    for mod in native_modules:
        m = Path(mod)
        found = [str(m.parent / (m.name + suf)) for suf in importlib.machinery.EXTENSION_SUFFIXES
                 if (repo / m.parent / (m.name + suf)).is_file()]
        if len(found) != 1:
            raise RuntimeError(f"build exactly one native extension before bundling: {mod} (found {found})")
        out.add(found[0])
    selected = []
    for p in sorted(out):
        f = repo / p
        if f.is_symlink():
            raise ValueError(f"a bundle must not follow a symbolic link: {p}")
        if f.is_file():
            selected.append(p)
    return selected


def build_bundle(repo: str | Path, out_dir: str | Path, *, name: str = "job",
                 paths: Sequence[str] = DEFAULT_PATHS, native_modules: Sequence[str] = NATIVE_MODULES) -> Path:
    repo, out_dir = Path(repo), Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    files = bundle_paths(repo, paths, native_modules)
    commit = _git(repo, "rev-parse", "HEAD").strip()
    clean = _git(repo, "status", "--porcelain", "--untracked-files=no", "--", *paths).strip() == ""
    members = {}
    target = out_dir / f"{name}-{commit[:12]}.zip"
    tmp = target.with_suffix(".zip.tmp")
    with zipfile.ZipFile(tmp, "w", compression=zipfile.ZIP_DEFLATED) as z:
        for p in files:
            data = (repo / p).read_bytes()
            members[p] = {"sha256": _sha256(data), "bytes": len(data)}
            z.writestr(p, data)
        z.writestr(MANIFEST, json.dumps({"commit": commit, "clean": clean, "python": sys.version.split()[0],
                                         "members": members}, indent=2, sort_keys=True))
    tmp.replace(target)
    return target


def verify_bundle(path: str | Path) -> dict:
    """The manifest of an archive whose every member matches its recorded digest (else raises)."""
    with zipfile.ZipFile(path) as z:
        man = json.loads(z.read(MANIFEST))
        names = set(z.namelist()) - {MANIFEST}
        if names != set(man["members"]):
            raise ValueError(f"bundle members differ from its manifest: {sorted(names ^ set(man['members']))[:5]}")
        for p, meta in man["members"].items():
            if _sha256(z.read(p)) != meta["sha256"]:
                raise ValueError(f"bundle member {p} does not match its digest")
    return man


def extract_bundle(path: str | Path, dest: str | Path) -> Path:
    verify_bundle(path)
    dest = Path(dest)
    with zipfile.ZipFile(path) as z:
        for p in z.namelist():
            if Path(p).is_absolute() or ".." in Path(p).parts:
                raise ValueError(f"unsafe bundle member path {p}")
        z.extractall(dest)
    return dest


def launch_command(bundle_root: str | Path, script: str, *, nproc_per_node: int, master_port: int = 29500,
                   args: Sequence[str] = ()) -> list[str]:
    """One-node launch of ``script`` (a module with ``-m`` or a file path) from an extracted bundle."""
    root = Path(bundle_root)
    target = ["-m", script[3:]] if script.startswith("-m ") else [str(root / script)]
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={int(nproc_per_node)}",
            "--master-addr=127.0.0.1", f"--master-port={int(master_port)}", *target, *args]


__all__ = ["bundle_paths", "build_bundle", "extract_bundle", "launch_command", "verify_bundle"]
