"""Checkpoint audits: read a committed step back through the checkpoint format and check it.

    python -m flare_b200.checkpoint.audit --root ckpt [--step S] [--group tables]

``audit_dense`` checks the dense manifest against the files (every entry has
master / m / v arrays of the recorded shape, all finite) and fingerprints
them; ``audit_sparse`` follows the FULL + INCREMENTAL chain of a sparse
group, checks that the pieces of every table cover each column and each row
residue exactly once, that every array has the table's row count and width,
that values and optimizer state are finite (and row-wise / Adagrad state
non-negative), and fingerprints the assembled tables; ``audit_step`` does
both and adds a file inventory.  Two audits of the same logical state have
the same digests whatever the sharding they were saved from.  Reference
behaviour: tools/validation/audit_dense_checkpoint.py,
audit_sparse_checkpoint.py (BLAKE2b fingerprints, file inventory).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

from .store import FORMAT_DENSE, _FIELDS, _piece_name, _sparse_chain, latest_step, step_dir


def _digest(arrs: dict[str, np.ndarray]) -> dict:
    leaves, comb = {}, hashlib.blake2b(digest_size=32)
    for name in sorted(arrs):
        a = np.ascontiguousarray(arrs[name])
        h = hashlib.blake2b(digest_size=32)
        h.update(f"{name}|{a.shape}|{a.dtype}|".encode())
        h.update(a.tobytes())
        leaves[name] = h.hexdigest()
        comb.update(leaves[name].encode())
    return {"digest": comb.hexdigest(), "leaves": leaves}


def file_inventory(root: Path) -> dict[str, list[int]]:
    """Relative path -> [size bytes, 0] for every file under ``root`` (sorted)."""
    return {str(p.relative_to(root)): [p.stat().st_size, 0] for p in sorted(root.rglob("*")) if p.is_file()}


def audit_dense(dirpath: Path) -> dict:
    man = json.loads((dirpath / "manifest.json").read_text())
    if man.get("format") != FORMAT_DENSE:
        raise ValueError(f"{dirpath}: not a dense checkpoint")
    arrs, problems = {}, []
    for name, e in man["entries"].items():
        for field in ("master", "m", "v"):
            f = dirpath / f"{name}.{field}.npy"
            if not f.exists():
                problems.append(f"missing {f.name}")
                continue
            a = np.load(f)
            if list(a.shape) != list(e["shape"]):
                problems.append(f"{f.name}: shape {list(a.shape)} != {e['shape']}")
            if not np.isfinite(a).all():
                problems.append(f"{f.name}: non-finite values")
            if field == "v" and (a < 0).any():
                problems.append(f"{f.name}: negative second moment")
            arrs[f"{name}.{field}"] = a
    return {"step": man["step"], "optimizer_step": man["optimizer_step"], "entries": len(man["entries"]),
            "problems": problems, **_digest(arrs)}


def audit_sparse(root: Path, step: int, group: str = "tables") -> dict:
    chain = _sparse_chain(lambda s: step_dir(root, s) / "sparse" / group, step)
    last = chain[-1][1]
    problems = []
    tables = {t["name"]: t for t in last["tables"]}
    full: dict[str, dict[str, np.ndarray]] = {}
    for name, t in tables.items():
        rows, dim = int(t["rows"]), int(t["dim"])
        # coverage: every column is covered by pieces with one row split R and residues exactly 0..R-1
        by_col: dict[int, list[tuple[int, int]]] = {}
        for p in chain[0][1]["pieces"]:
            if p["table"] != name:
                continue
            for c in range(p["col_begin"], p["col_begin"] + p["ncols"]):
                by_col.setdefault(c, []).append((int(p.get("row_shards", 1)), int(p.get("row_index", 0))))
        bad = set(by_col) != set(range(dim)) or any(
            len({R for R, _ in v}) != 1 or sorted(r for _, r in v) != list(range(v[0][0])) for v in by_col.values())
        if bad:
            problems.append(f"table {name}: pieces do not cover its columns / rows exactly once")
        entry: dict[str, np.ndarray] = {}
        for _, man, d in chain:
            for p in man["pieces"]:
                if p["table"] != name:
                    continue
                R, r = int(p.get("row_shards", 1)), int(p.get("row_index", 0))
                prefix = d / _piece_name(name, p["col_begin"], r, R)
                local = np.load(f"{prefix}.rows.npy") if man["mode"] == "incremental" else None
                for field in _FIELDS:
                    f = Path(f"{prefix}.{field}.npy")
                    if not f.exists():
                        continue
                    a = np.load(f)
                    nloc = (rows - r + R - 1) // R
                    if local is None and a.shape[0] != nloc:
                        problems.append(f"{f.name}: {a.shape[0]} rows, expected {nloc}")
                        continue
                    if not np.isfinite(a).all():
                        problems.append(f"{f.name}: non-finite values")
                    if field in ("state_row", "state_v") and (a < 0).any():
                        problems.append(f"{f.name}: negative optimizer state")
                    if field not in entry:
                        entry[field] = np.zeros((rows, dim) if a.ndim == 2 else (rows,), dtype=np.float32)
                    idx = (np.arange(a.shape[0]) if local is None else local) * R + r
                    if a.ndim == 2:
                        entry[field][idx, p["col_begin"]:p["col_begin"] + a.shape[1]] = a
                    else:
                        entry[field][idx] = a
        full[name] = entry
    arrs = {f"{t}.{f}": a for t, e in full.items() for f, a in e.items()}
    return {"step": step, "chain": [s for s, _, _ in chain], "optimizer": last["optimizer"],
            "optimizer_step": last["optimizer_step"], "tables": len(tables), "problems": problems, **_digest(arrs)}


def audit_step(root: str | Path, step: int | None = None, group: str = "tables") -> dict:
    root = Path(root)
    step = latest_step(root) if step is None else step
    if step is None:
        raise FileNotFoundError(f"no checkpoint under {root}")
    d = step_dir(root, step)
    dense = audit_dense(d / "model")
    sparse = audit_sparse(root, step, group)
    return {"step": step, "dense": dense, "sparse": sparse, "files": file_inventory(d),
            "ok": not dense["problems"] and not sparse["problems"]}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--root", required=True)
    ap.add_argument("--step", type=int, default=None)
    ap.add_argument("--group", default="tables")
    a = ap.parse_args(argv)
    rep = audit_step(a.root, a.step, a.group)
    print(json.dumps({k: v for k, v in rep.items() if k != "files"} | {"files": len(rep["files"])}, indent=1))
    return 0 if rep["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())


__all__ = ["audit_dense", "audit_sparse", "audit_step", "file_inventory"]
