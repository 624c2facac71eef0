"""Crash-window worker for the Iceberg publication tests: a publisher that dies around its commit.

    python -m flare_b200.testing.iceberg_crash TABLE WINDOW before   # data files and manifests written,
                                                                    # os._exit(85) before the metadata commit
    python -m flare_b200.testing.iceberg_crash TABLE WINDOW after    # os._exit(86) right after the commit,
                                                                    # before the publisher learns of it
    python -m flare_b200.testing.iceberg_crash TABLE WINDOW clean    # publish normally

Each run publishes window ``WINDOW`` (100 rows whose ids start at ``WINDOW * 100``) into the table at
``TABLE`` (created on first use) with the commit id ``window-<WINDOW>``, the way the feature
pipeline publishes an input: ``IcebergSink.append(..., commit_id=...)`` finds a commit that already
happened and otherwise writes and commits.  The crash is a process exit at the chosen point, as the
reference's crash-recovery workers do with ``os._exit`` around an Iceberg commit
(data/pipeline/production/publish/tests/crash_recovery_worker.py:65-69).
"""
from __future__ import annotations

import os
import sys

import pyarrow as pa

from ..data.iceberg import IcebergSink, IcebergTable

ROWS = 100


def window_rows(window: int) -> pa.Table:
    ids = list(range(window * ROWS, (window + 1) * ROWS))
    return pa.table({"id": pa.array(ids, type=pa.int64()), "v": pa.array([i * 0.5 for i in ids], type=pa.float64())})


def publish(table_path: str, window: int, mode: str) -> dict | None:
    data = window_rows(window)
    table = IcebergTable.create(table_path, data.schema, exist_ok=True)
    if mode in ("before", "after"):
        original = IcebergTable._commit_metadata

        def commit_then_maybe_die(self, meta):
            if mode == "before" and meta.get("snapshots"):
                os._exit(85)
            original(self, meta)
            if mode == "after" and meta.get("snapshots"):
                os._exit(86)

        IcebergTable._commit_metadata = commit_then_maybe_die
    return IcebergSink(table).append([data], commit_id=f"window-{window}")


def main(argv=None) -> int:
    args = list(sys.argv[1:] if argv is None else argv)
    if len(args) != 3 or args[2] not in ("before", "after", "clean"):
        raise SystemExit("usage: python -m flare_b200.testing.iceberg_crash TABLE WINDOW before|after|clean")
    snap = publish(args[0], int(args[1]), args[2])
    print(f"committed snapshot={snap['snapshot-id'] if snap else None}", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
