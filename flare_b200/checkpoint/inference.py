"""Published inference weights: immutable ``steps/<step>`` assets.

Contract of the reference's inference weights
(src/flare/inference/weights/source.py:72-444): an asset directory has
exactly two children, ``model/`` and ``sparse/``; the caller binds the asset
once, which records POSIX evidence (relative path, size, mtime, inode of every
file, folded into a tree signature); every later load re-checks the evidence
and refuses a mutated asset.  ``load_model`` restores dense weights only (no
optimizer state), ``load_sparse`` restores table values into a collection with
the consumer's own topology (column/table re-planning happens on load).
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from .store import FORMAT_DENSE, load_sparse, step_dir

REQUIRED_CHILDREN = frozenset({"model", "sparse"})


@dataclass(frozen=True)
class PublishedAssetEvidence:
    path: str
    files: int
    total_bytes: int
    tree_signature: str

    @classmethod
    def capture(cls, path: str | os.PathLike) -> "PublishedAssetEvidence":
        root = Path(path)
        h = hashlib.sha256()
        nfiles = total = 0
        for p in sorted(root.rglob("*")):
            if p.is_file():
                st = p.stat()
                rel = p.relative_to(root).as_posix()
                h.update(f"{rel}|{st.st_size}|{st.st_mtime_ns}|{st.st_ino}\n".encode())
                nfiles += 1
                total += st.st_size
        return cls(str(root.resolve()), nfiles, total, h.hexdigest())


def _validate_asset_path(path: Path) -> None:
    if not path.is_dir():
        raise FileNotFoundError(f"inference asset {path} does not exist")
    children = {p.name for p in path.iterdir()}
    if children != REQUIRED_CHILDREN:
        raise ValueError(f"inference asset {path} must contain exactly {sorted(REQUIRED_CHILDREN)}, "
                         f"found {sorted(children)}")
    if not (path / "model" / "manifest.json").is_file():
        raise ValueError(f"inference asset {path} has no model manifest")


@dataclass
class InferenceWeights:
    root: str
    step: int
    evidence: PublishedAssetEvidence

    @classmethod
    def bind(cls, root: str | os.PathLike, step: int) -> "InferenceWeights":
        path = step_dir(root, step)
        _validate_asset_path(path)
        return cls(str(root), int(step), PublishedAssetEvidence.capture(path))

    @property
    def path(self) -> Path:
        return step_dir(self.root, self.step)

    def verify(self) -> None:
        now = PublishedAssetEvidence.capture(self.path)
        if now != self.evidence:
            raise RuntimeError(f"inference asset {self.path} changed after it was bound")

    def load_model(self, dense) -> dict:
        """Dense weights only (compute copy and fp32 master), no optimizer state."""
        self.verify()
        d = self.path / "model"
        manifest = json.loads((d / "manifest.json").read_text())
        if manifest.get("format") != FORMAT_DENSE:
            raise ValueError("not a dense model asset")
        master = torch.zeros(dense.n, dtype=torch.float32)
        for name, e in dense.params.entries.items():
            if name not in manifest["entries"]:
                raise ValueError(f"model asset lacks parameter {name}")
            master[e.offset:e.offset + e.numel] = torch.from_numpy(np.load(d / f"{name}.master.npy")).reshape(-1)
        dense.master.copy_(master.to(dense.device)[dense.lo:dense.hi])
        dense.compute.copy_(master.to(dense.device).to(dense.compute.dtype))
        return manifest

    def load_sparse(self, coll, group: str = "tables") -> dict:
        self.verify()
        return load_sparse(self.root, self.step, group, coll)


def bind_inference_weights(root: str | os.PathLike, step: int) -> InferenceWeights:
    return InferenceWeights.bind(root, step)


__all__ = ["InferenceWeights", "PublishedAssetEvidence", "bind_inference_weights"]
