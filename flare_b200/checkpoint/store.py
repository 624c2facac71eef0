"""Checkpoints in the ``steps/<step>/{model,sparse/<group>}`` layout.

Layout (kept from the reference, src/flare/runtime/fluxway/workers/
dynamic_embedding.py:793-812 and src/flare/inference/weights/source.py:168-217):

    <root>/steps/<step>/model/manifest.json      dense schema, step, optimizer kind
    <root>/steps/<step>/model/*.npy              fp32 master / moments (logical shapes)
    <root>/steps/<step>/sparse/<group>/manifest.json
    <root>/steps/<step>/sparse/<group>/<table>.c<col>.<field>.npy

The file format is this framework's own: one ``.npy`` file per array and a
JSON manifest.  A step directory is written under ``<step>.partial`` and
renamed into place by rank 0 after every rank finished, so a visible step is
always complete.  Dense state is captured only at an optimizer-window
boundary and stored unpadded.  Sparse saves are ``full`` or ``incremental``:
an incremental save stores only rows updated since the previous save (the
fused backward marks them) and names the step it builds on; restore applies
the chain FULL -> increments.  Restore re-plans tables for the current world
size, so a checkpoint written on N GPUs restores on M.
"""
from __future__ import annotations

import json
import os
import shutil
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

FORMAT_DENSE = "flare_b200.dense/1"
FORMAT_SPARSE = "flare_b200.sparse/1"


def _rank_world() -> tuple[int, int]:
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def _barrier() -> None:
    if dist.is_initialized() and dist.get_world_size() > 1:
        from ..parallel.dist import barrier

        barrier()


READ_ATTEMPTS = 3


def _read_array(path) -> np.ndarray:
    """``np.load`` with up to ``READ_ATTEMPTS`` tries on transient I/O errors (network file systems);
    a missing file fails at once.  The reference retries transient read errors of its sparse
    checkpoints three times (src/flare/runtime/fluxway/checkpoint/sparse.py:20-47)."""
    for attempt in range(READ_ATTEMPTS):
        try:
            return np.load(path)
        except FileNotFoundError:
            raise
        except OSError:
            if attempt == READ_ATTEMPTS - 1:
                raise
            time.sleep(0.05 * (attempt + 1))
    raise AssertionError("unreachable")


def step_dir(root: str | os.PathLike, step: int) -> Path:
    return Path(root) / "steps" / str(int(step))


def list_steps(root: str | os.PathLike) -> list[int]:
    d = Path(root) / "steps"
    if not d.is_dir():
        return []
    return sorted(int(p.name) for p in d.iterdir() if p.is_dir() and p.name.isdigit())


def latest_step(root: str | os.PathLike) -> int | None:
    s = list_steps(root)
    return s[-1] if s else None


# ---------------------------------------------------------------- dense
def save_dense(dirpath: Path, dense, step: int) -> None:
    """Write the dense flat state (gathered over ranks) with per-parameter logical shapes."""
    state = dense.state_dict()  # collective when sharded
    rank, _ = _rank_world()
    if rank != 0:
        return
    dirpath.mkdir(parents=True, exist_ok=True)
    entries = {}
    for name, e in dense.params.entries.items():
        for field in ("master", "m", "v"):
            arr = state[field][e.offset:e.offset + e.numel].reshape(e.shape).numpy()
            np.save(dirpath / f"{name}.{field}.npy", arr)
        entries[name] = {"shape": list(e.shape), "dtype": "float32"}
    manifest = {"format": FORMAT_DENSE, "step": int(step), "optimizer_step": int(state["step"]),
                "optimizer": dense.opt.kind, "entries": entries}
    (dirpath / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))


def load_dense(dirpath: Path, dense) -> dict:
    manifest = json.loads((dirpath / "manifest.json").read_text())
    if manifest.get("format") != FORMAT_DENSE:
        raise ValueError(f"{dirpath}: not a dense checkpoint")
    if set(manifest["entries"]) != set(dense.params.entries):
        raise ValueError("dense checkpoint parameters do not match the model")
    full = {f: torch.zeros(dense.n, dtype=torch.float32) for f in ("master", "m", "v")}
    for name, e in dense.params.entries.items():
        if tuple(manifest["entries"][name]["shape"]) != tuple(e.shape):
            raise ValueError(f"parameter {name}: checkpoint shape differs from the model")
        for field in ("master", "m", "v"):
            full[field][e.offset:e.offset + e.numel] = torch.from_numpy(
                _read_array(dirpath / f"{name}.{field}.npy")).reshape(-1)
    dense.load_state_dict({"step": manifest["optimizer_step"], **full})
    return manifest


# --------------------------------------------------------------- sparse
_FIELDS = ("weight", "state_row", "state_m", "state_v", "score")


def _piece_name(table: str, col_begin: int, row_index: int = 0, row_shards: int = 1) -> str:
    """File prefix of one piece: columns from ``col_begin``; a row-wise piece adds its residue."""
    name = f"{table}.c{col_begin}"
    return name if row_shards == 1 else f"{name}.r{row_index}of{row_shards}"


def save_sparse(dirpath: Path, coll, step: int, *, mode: str = "full", base_step: int | None = None) -> None:
    """Each rank writes its shards; rank 0 writes the manifest."""
    if mode not in ("full", "incremental"):
        raise ValueError("mode must be full or incremental")
    if mode == "incremental" and base_step is None:
        raise ValueError("an incremental save needs the step it builds on")
    rank, world = _rank_world()
    if any(s.slot_map_off >= 0 for s in coll.shards):
        raise NotImplementedError("host-tier tables are checkpointed from their host copy (HostTier.export_state)")
    dirpath.mkdir(parents=True, exist_ok=True)
    for i, s in enumerate(coll.shards):
        fields = coll.shard_fields(i)
        prefix = dirpath / _piece_name(s.spec.name, s.col_begin, s.row_index, s.row_shards)
        rows = None
        if mode == "incremental":
            rows = coll.dirty_rows(s.row_base, s.storage_rows)
            np.save(f"{prefix}.rows.npy", rows.cpu().numpy().astype(np.int64))
        for field, t in fields.items():
            arr = t if rows is None else t.index_select(0, rows)
            np.save(f"{prefix}.{field}.npy", arr.float().cpu().numpy())
    coll.clear_dirty()
    pieces = [{"table": s.spec.name, "col_begin": s.col_begin, "ncols": s.ncols, "rank": rank,
               "row_index": s.row_index, "row_shards": s.row_shards} for s in coll.shards]
    gathered = [pieces]
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, pieces)
    if rank == 0:
        manifest = {
            "format": FORMAT_SPARSE, "step": int(step), "mode": mode, "base_step": base_step,
            "optimizer": coll.optimizer.kind, "optimizer_step": int(coll.step),
            "tables": [{"name": t.name, "rows": t.num_embeddings, "dim": t.embedding_dim,
                        "value_dtype": t.value_dtype, "pooling": t.pooling} for t in coll.tables],
            "pieces": [p for part in gathered for p in part], "world_size": world,
        }
        (dirpath / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))


def _sparse_chain(group_dir_of_step, step: int) -> list[tuple[int, dict, Path]]:
    chain = []
    s = step
    while True:
        d = group_dir_of_step(s)
        m = json.loads((d / "manifest.json").read_text())
        if m.get("format") != FORMAT_SPARSE:
            raise ValueError(f"{d}: not a sparse checkpoint")
        chain.append((s, m, d))
        if m["mode"] == "full":
            break
        s = int(m["base_step"])
    return list(reversed(chain))


def load_sparse(root: str | os.PathLike, step: int, group: str, coll) -> dict:
    """Restore the collection's local shards from the FULL + incremental chain ending at ``step``."""
    chain = _sparse_chain(lambda s: step_dir(root, s) / "sparse" / group, step)
    names = {t.name for t in coll.tables}
    last = chain[-1][1]
    if {t["name"] for t in last["tables"]} != names:
        raise ValueError("sparse checkpoint tables do not match the collection")
    state = {}
    for s in coll.shards:
        entry = {}
        for _, man, d in chain:
            pieces = [p for p in man["pieces"] if p["table"] == s.spec.name]
            for p in pieces:
                lo, hi = max(p["col_begin"], s.col_begin), min(p["col_begin"] + p["ncols"], s.col_begin + s.ncols)
                if lo >= hi:
                    continue
                R, r = int(p.get("row_shards", 1)), int(p.get("row_index", 0))
                prefix = d / _piece_name(s.spec.name, p["col_begin"], r, R)
                local = _read_array(f"{prefix}.rows.npy") if man["mode"] == "incremental" else None
                for field in _FIELDS:
                    f = Path(f"{prefix}.{field}.npy")
                    if not f.exists():
                        continue
                    arr = _read_array(f)
                    if field not in entry:
                        shape = (s.spec.num_embeddings, s.ncols) if arr.ndim == 2 else (s.spec.num_embeddings,)
                        entry[field] = np.zeros(shape, dtype=np.float32)
                    tgt = entry[field]
                    # table rows of the saved rows: local row l of a row-wise piece is row l * R + r
                    rows = (np.arange(arr.shape[0]) if local is None else local) * R + r
                    if arr.ndim == 2:
                        tgt[rows, lo - s.col_begin:hi - s.col_begin] = arr[:, lo - p["col_begin"]:hi - p["col_begin"]]
                    else:
                        tgt[rows] = arr
        state[(s.spec.name, s.col_begin, s.row_index)] = {k: torch.from_numpy(np.ascontiguousarray(v[s.row_slice]))
                                             for k, v in entry.items()}
    coll.load_local_state(state)
    coll.step = int(last["optimizer_step"])
    coll.step_dev.fill_(coll.step)
    coll.clear_dirty()
    return last


# --------------------------------------------------------------- manager
@dataclass
class CheckpointManager:
    """Save / restore a fused model (dense flat state + sparse collections)."""

    root: str

    def save(self, step: int, model, *, group: str = "tables", incremental: bool | None = None,
             reader=None) -> Path:
        """Write ``steps/<step>`` for every rank's part of ``model``.  A sparse update the model still
        holds back (pipelined policy) is applied first, so the saved tables include every step.  With
        ``reader`` (this rank's ``data.reader.BatchReader``) its cut position goes into
        ``reader/rank<k>.json`` of the same step, committed together with the model."""
        flush = getattr(model, "flush_pending_updates", None)
        if flush is not None:
            flush()
        rank, _ = _rank_world()
        final = step_dir(self.root, step)
        tmp = final.with_name(f"{final.name}.partial")
        if rank == 0:
            if tmp.exists():
                shutil.rmtree(tmp)
            tmp.mkdir(parents=True)
        _barrier()
        prev = latest_step(self.root)
        mode = "incremental" if (incremental and prev is not None) else "full"
        save_dense(tmp / "model", model.dense, step)
        save_sparse(tmp / "sparse" / group, model.emb, step, mode=mode, base_step=prev if mode == "incremental" else None)
        if reader is not None:
            from .source_cut import save_reader_cut

            save_reader_cut(tmp, step, reader.capture_state())
        _barrier()
        if rank == 0:
            if final.exists():
                shutil.rmtree(final)
            os.replace(tmp, final)
        _barrier()
        return final

    def restore(self, model, step: int | None = None, *, group: str = "tables", reader=None) -> int:
        step = latest_step(self.root) if step is None else step
        if step is None:
            raise FileNotFoundError(f"no checkpoint under {self.root}")
        flush = getattr(model, "flush_pending_updates", None)
        if flush is not None:
            flush()  # a pending update belongs to the state being replaced
        load_dense(step_dir(self.root, step) / "model", model.dense)
        load_sparse(self.root, step, group, model.emb)
        if reader is not None:  # every saved rank's cut; the remaining items are dealt to this run's ranks
            from .source_cut import load_reader_cut

            states = load_reader_cut(step_dir(self.root, step))
            if not states:
                raise ValueError(f"step {step} has no reader cut to restore")
            reader.restore_state(states)
        return step


__all__ = ["CheckpointManager", "latest_step", "list_steps", "load_dense", "load_sparse", "save_dense", "save_sparse",
           "step_dir"]
