"""Offline audit of a feature-pipeline output directory (``data.pipeline.DataPipeline``).

``audit_publication(output)`` checks that what the publication manifest (``_publication.json``) claims
is what is on disk:

* window ids run 0, 1, 2, ... and every window directory holds exactly its ``parts`` Parquet files,
  whose footers add up to the window's ``rows``;
* every window's input is listed as done and no done input is listed twice;
* every data file has exactly the columns of the feature catalog (``feature_manifest.json``) when one
  is published;
* no temporary window of a crashed run (``.window-*``) is left behind, unless ``allow_temporary``
  (the next run removes them when it starts).

It returns a summary (windows, inputs, data files, rows, rows per input) and raises
``AssertionError`` naming the first inconsistency.

    python -m flare_b200.data.publication_audit OUTPUT_DIR [--allow-temporary]

Reference behaviour: the publication manifest and window checks of the reference's production
publication (src/flare/data/pipeline/production/publication/manifest.py and window.py), as an
offline tool.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import pyarrow.parquet as pq

from ..io.artifacts import read_json
from .pipeline import MANIFEST, TMP_PREFIX


def audit_publication(output: str | Path, *, allow_temporary: bool = False) -> dict:
    out = Path(output)
    if not (out / MANIFEST).is_file():
        raise AssertionError(f"{out} has no publication manifest ({MANIFEST})")
    man = read_json(out / MANIFEST)
    done = list(man.get("inputs_done", []))
    if len(set(done)) != len(done):
        raise AssertionError("an input is listed as done twice")
    columns = None
    from .feature_catalog import MANIFEST_NAME, FeatureCatalog

    if (out / MANIFEST_NAME).is_file():
        columns = set(FeatureCatalog.from_manifest_dir(out).columns)
    rows_per_input: dict[str, int] = {}
    files = 0
    for k, w in enumerate(man.get("windows", [])):
        if w.get("id") != k:
            raise AssertionError(f"window {k} has id {w.get('id')!r}")
        if w["input"] not in done:
            raise AssertionError(f"window {k} comes from {w['input']!r}, which is not listed as done")
        d = out / w["dir"]
        parts = sorted(p.name for p in d.glob("*.parquet")) if d.is_dir() else []
        want = [f"part-{i:05d}.parquet" for i in range(int(w["parts"]))]
        if parts != want:
            raise AssertionError(f"window {k} ({w['dir']}) holds {parts}, its manifest entry says {want}")
        rows = 0
        for name in want:
            f = pq.ParquetFile(d / name)
            rows += f.metadata.num_rows
            if columns is not None and set(f.schema_arrow.names) != columns:
                got = set(f.schema_arrow.names)
                raise AssertionError(f"{d / name}: columns differ from the feature catalog: missing "
                                     f"{sorted(columns - got)} unexpected {sorted(got - columns)}")
        if rows != int(w["rows"]):
            raise AssertionError(f"window {k} holds {rows} rows, its manifest entry says {w['rows']}")
        rows_per_input[w["input"]] = rows_per_input.get(w["input"], 0) + rows
        files += len(want)
    leftovers = sorted(p.name for p in out.glob(TMP_PREFIX + "*"))
    if leftovers and not allow_temporary:
        raise AssertionError(f"temporary windows of a crashed run are left: {leftovers}")
    return {"windows": len(man.get("windows", [])), "inputs_done": len(done), "data_files": files,
            "rows": sum(rows_per_input.values()), "rows_per_input": rows_per_input,
            "catalog_columns": sorted(columns) if columns is not None else None, "temporary": leftovers}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="audit a feature-pipeline output directory")
    ap.add_argument("output")
    ap.add_argument("--allow-temporary", action="store_true")
    a = ap.parse_args(argv)
    print(json.dumps(audit_publication(a.output, allow_temporary=a.allow_temporary), indent=2, sort_keys=True))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())


__all__ = ["audit_publication"]
