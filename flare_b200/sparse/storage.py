"""Sparse storage tier options: memory limit, disk spill, page geometry.

``SparseStorageOptions`` validates the storage keys of a sparse group's
configuration (the reference's names: ``sparse_storage_memory_limit_bytes``,
``sparse_storage_max_spill_bytes``, ``sparse_storage_spill_dir``,
``sparse_storage_max_pages``, ``sparse_storage_entries_per_page``; reference:
src/flare/runtime/sparse_storage.py:8-47) and builds one native
``PagedRowStore`` per table (``csrc/paged_store.cpp``): records of the
embedding row plus its optimizer state in pages of ``entries_per_page`` rows,
at most the memory limit resident, the rest in a spill file of at most
``max_spill_bytes``.  The group's memory limit is split over its tables in
proportion to their size.  Every store spills into its own fresh directory
under ``spill_directory`` (``worker-*``), so groups, ranks and restored
workers never share spill files.  The CPU collection
(``sparse/reference.py``) keeps its tables in these stores when given options.
"""
from __future__ import annotations

import tempfile
from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

from .._native import native

PAGE_SIZES = (0, 4096, 8192, 16384)
DEFAULT_ENTRIES_PER_PAGE = 4096


def _positive_or_none(name: str, v) -> None:
    if v is not None and (isinstance(v, bool) or not isinstance(v, int) or v <= 0):
        raise ValueError(f"sparse storage {name} must be a positive integer")


@dataclass(frozen=True)
class SparseStorageOptions:
    memory_limit_bytes: int | None = None   # resident bytes of the group (None: everything resident)
    max_spill_bytes: int | None = None      # spill file bytes of the group (None: no limit)
    spill_directory: str | None = None
    max_pages: int = 0                      # resident pages per table at most (0: no cap)
    entries_per_page: int = 0               # rows per page (0: the default, 4096)

    def __post_init__(self) -> None:
        _positive_or_none("memory limit", self.memory_limit_bytes)
        _positive_or_none("spill limit", self.max_spill_bytes)
        if isinstance(self.max_pages, bool) or not isinstance(self.max_pages, int) or self.max_pages < 0:
            raise ValueError("sparse storage max_pages must be a non-negative integer")
        if self.entries_per_page not in PAGE_SIZES:
            raise ValueError("sparse storage entries_per_page must be 0, 4096, 8192 or 16384")
        if self.max_spill_bytes is not None and self.spill_directory is None:
            raise ValueError("sparse storage spill limit requires a spill directory")
        if self.memory_limit_bytes is not None and self.spill_directory is None:
            raise ValueError("a sparse storage memory limit needs a spill directory for the rows that do not fit")

    @classmethod
    def from_spec(cls, spec: Mapping[str, Any]) -> "SparseStorageOptions":
        return cls(memory_limit_bytes=spec.get("sparse_storage_memory_limit_bytes"),
                   max_spill_bytes=spec.get("sparse_storage_max_spill_bytes"),
                   spill_directory=spec.get("sparse_storage_spill_dir"),
                   max_pages=spec.get("sparse_storage_max_pages", 0),
                   entries_per_page=spec.get("sparse_storage_entries_per_page", 0))

    @property
    def rows_per_page(self) -> int:
        return self.entries_per_page or DEFAULT_ENTRIES_PER_PAGE

    def build_stores(self, tables: list[tuple[str, int, int, int, float]], seed: int = 0) -> list["TableStore"]:
        """One store per table: (name, rows, record width, initialised columns, init scale)."""
        directory = None
        if self.spill_directory is not None:
            root = Path(self.spill_directory)
            root.mkdir(parents=True, exist_ok=True)
            directory = Path(tempfile.mkdtemp(prefix="worker-", dir=root))
        total = sum(rows * width * 4 for _, rows, width, _, _ in tables) or 1
        stores = []
        for k, (name, rows, width, init_cols, scale) in enumerate(tables):
            share = rows * width * 4 / total
            limit = 0 if self.memory_limit_bytes is None else max(1, int(self.memory_limit_bytes * share))
            rpp = min(self.rows_per_page, rows)
            if self.max_pages:
                cap = self.max_pages * rpp * width * 4
                limit = cap if limit == 0 else min(limit, cap)
            spill = 0 if self.max_spill_bytes is None else max(1, int(self.max_spill_bytes * share))
            path = str(directory / f"{k:03d}_{name}.spill") if directory is not None else ""
            stores.append(TableStore(native().PagedRowStore(rows, width, rpp, limit, path, spill, init_cols,
                                                            float(scale), int(seed) * 1_000_003 + k), width))
        return stores


class TableStore:
    """Torch-facing wrapper of one native paged store: gather / scatter whole records by row id."""

    def __init__(self, store, width: int):
        self.store, self.width = store, width

    def gather(self, ids: torch.Tensor) -> torch.Tensor:
        ids = ids.detach().to("cpu", torch.int64).contiguous()
        out = torch.empty(ids.numel(), self.width, dtype=torch.float32)
        self.store.gather(ids, out)
        return out

    def scatter(self, ids: torch.Tensor, records: torch.Tensor) -> None:
        self.store.scatter(ids.detach().to("cpu", torch.int64).contiguous(), records.detach().float().contiguous())

    def stats(self) -> dict:
        return dict(self.store.stats())


__all__ = ["PAGE_SIZES", "SparseStorageOptions", "TableStore"]
