"""Checkpoints of the CPU configuration (generic engine + CPU embedding collection).

Same directory contract as the fused models' checkpoints: ``steps/<step>/model``
(the engine's boundary state: unpadded parameters, optimizer moments, buffers,
step) and ``steps/<step>/sparse/<group>`` (the collection's tables, optimizer
state, dynamic key maps and row-init RNG).  A step is written under
``steps/<step>.partial`` and renamed into place, so a crash mid-save leaves
the previous step as the latest (``list_steps`` ignores ``*.partial``).
Files are ``torch.save`` archives with a small JSON manifest beside them.
Reference behaviour: the ``steps/<step>/{model,sparse/<group>}`` asset of
src/flare/inference/weights/source.py:168-217 and the boundary-only dense
capture of src/flare/jax/training/engines/distributed.py:1182-1244.
"""
from __future__ import annotations

import json
import os
import shutil
from pathlib import Path

import torch

from .store import latest_step, step_dir

FORMAT = "flare_b200.cpu.v1"


def save_cpu(root: str | os.PathLike, step: int, engine, emb, *, group: str = "tables", reader=None) -> Path:
    """Write step ``step``: ``engine.capture_checkpoint_state()`` and ``emb.state_dict()``, and with
    ``reader`` (a ``data.reader.BatchReader``) its cut position, committed by the same rename."""
    final = step_dir(root, step)
    tmp = final.with_name(f"{final.name}.partial")
    if tmp.exists():
        shutil.rmtree(tmp)
    (tmp / "model").mkdir(parents=True)
    (tmp / "sparse" / group).mkdir(parents=True)
    dense = engine.capture_checkpoint_state()
    torch.save(dense, tmp / "model" / "state.pt")
    (tmp / "model" / "manifest.json").write_text(json.dumps(
        {"format": FORMAT, "step": int(step), "optimizer_step": int(dense["step"]),
         "schema_digest": dense["schema_digest"]}, indent=1))
    sparse = emb.state_dict()
    torch.save(sparse, tmp / "sparse" / group / "state.pt")
    (tmp / "sparse" / group / "manifest.json").write_text(json.dumps(
        {"format": FORMAT, "step": int(step), "optimizer_step": int(sparse["step"]),
         "tables": sorted(sparse["tables"]), "dynamic": sorted(sparse["dynamic"])}, indent=1))
    if reader is not None:
        from .source_cut import save_reader_cut

        save_reader_cut(tmp, step, reader.capture_state())
    if final.exists():
        shutil.rmtree(final)
    os.replace(tmp, final)
    return final


def restore_cpu(root: str | os.PathLike, engine, emb, step: int | None = None, *, group: str = "tables",
                reader=None) -> int:
    """Load step ``step`` (default: the latest complete one) into ``engine`` and ``emb`` (and ``reader``'s
    cut position, when the step has one); returns it."""
    step = latest_step(root) if step is None else step
    if step is None:
        raise FileNotFoundError(f"no checkpoint under {root}")
    d = step_dir(root, step)
    for part in (d / "model", d / "sparse" / group):
        man = json.loads((part / "manifest.json").read_text())
        if man.get("format") != FORMAT:
            raise ValueError(f"{part}: not a CPU-configuration checkpoint")
    engine.restore_checkpoint_state(torch.load(d / "model" / "state.pt", weights_only=False))
    emb.load_state_dict(torch.load(d / "sparse" / group / "state.pt", weights_only=False))
    if reader is not None:
        from .source_cut import load_reader_cut

        states = load_reader_cut(d)
        if not states:
            raise ValueError(f"step {step} has no reader cut to restore")
        reader.restore_state(states)
    return step


__all__ = ["FORMAT", "restore_cpu", "save_cpu"]
