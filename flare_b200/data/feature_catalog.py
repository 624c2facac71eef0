"""Feature catalog: the published description of a feature pipeline's output columns.

``catalog_for(cfg)`` describes every column the feature pipeline (``data.pipeline``) writes for a
``PipelineConfig``: the label, each dense feature (``d<i>``: float32, its transform) and each sparse
feature (``s<i>``: a list of int32 ids, its encoder, source feature codes and bucket count), plus a
digest of the configuration that produced them.  ``DataPipeline.run`` writes it as
``feature_manifest.json`` beside the published windows and refuses to publish into an output whose
manifest has another digest (two feature configurations must not share one dataset).  Readers resolve
feature names to columns through it (``column_for``), and ``validation.iceberg`` checks published
data files against its columns (``--manifest-dir``).

Reference behaviour: src/flare/data/schema/feature_catalog.py (feature descriptors keyed by code,
configuration digest, column validation, manifest write / load with exact field checks).
"""
from __future__ import annotations

import hashlib
import json
import re
from dataclasses import asdict, dataclass, fields
from pathlib import Path

MANIFEST_NAME = "feature_manifest.json"
KINDS = ("label", "dense", "sparse")
_COLUMN = re.compile(r"^[A-Za-z_][A-Za-z0-9_]*$")
_DIGEST = re.compile(r"^[0-9a-f]{64}$")


@dataclass(frozen=True)
class FeatureDescriptor:
    column: str
    name: str
    kind: str                       # label | dense | sparse
    encoder: str                    # identity / log1p / bucketize / fixed_width, or a sparse encoder
    source_codes: tuple[int, ...]   # feature codes of the raw record it is computed from
    buckets: int = 0                # id space of a hashed sparse feature (0: not bucketed)

    def __post_init__(self) -> None:
        if not _COLUMN.match(self.column or ""):
            raise ValueError(f"column name {self.column!r} is not an identifier")
        if not self.name:
            raise ValueError("a feature needs a name")
        if self.kind not in KINDS:
            raise ValueError(f"feature kind must be one of {KINDS}, got {self.kind!r}")
        if not self.encoder:
            raise ValueError("a feature needs an encoder")
        codes = tuple(self.source_codes)
        if not codes or any(isinstance(c, bool) or not isinstance(c, int) or c < 0 for c in codes):
            raise ValueError(f"feature {self.column}: source codes must be non-negative integers")
        if len(set(codes)) != len(codes):
            raise ValueError(f"feature {self.column}: duplicate source codes")
        if isinstance(self.buckets, bool) or not isinstance(self.buckets, int) or self.buckets < 0:
            raise ValueError(f"feature {self.column}: buckets must be a non-negative integer")
        object.__setattr__(self, "source_codes", codes)

    def to_entry(self) -> dict:
        d = asdict(self)
        d["source_codes"] = list(self.source_codes)
        return d


_ENTRY_FIELDS = frozenset(f.name for f in fields(FeatureDescriptor))


class FeatureCatalog:
    def __init__(self, descriptors, *, config_digest: str):
        if not _DIGEST.match(config_digest or ""):
            raise ValueError("config_digest must be a lowercase SHA-256 hex digest")
        self.config_digest = config_digest
        self._by_column: dict[str, FeatureDescriptor] = {}
        names: dict[str, list[str]] = {}
        for d in descriptors:
            if not isinstance(d, FeatureDescriptor):
                raise TypeError("descriptors must be FeatureDescriptor values")
            if d.column in self._by_column:
                raise ValueError(f"duplicate column {d.column!r}")
            self._by_column[d.column] = d
            names.setdefault(d.name, []).append(d.column)
        if sum(d.kind == "label" for d in self._by_column.values()) > 1:
            raise ValueError("a catalog has at most one label column")
        self._by_name = names

    @property
    def descriptors(self) -> tuple[FeatureDescriptor, ...]:
        return tuple(self._by_column.values())

    @property
    def columns(self) -> tuple[str, ...]:
        return tuple(self._by_column)

    def require(self, column: str) -> FeatureDescriptor:
        try:
            return self._by_column[column]
        except KeyError:
            raise ValueError(f"column {column!r} is not in the catalog") from None

    def column_for(self, name: str) -> str:
        """The column of the feature named ``name`` (an error if none or several have that name)."""
        cols = self._by_name.get(name, [])
        if len(cols) != 1:
            raise ValueError(f"feature name {name!r} is " + ("not declared" if not cols else f"ambiguous: {cols}"))
        return cols[0]

    def table_specs(self, embedding_dim: int, *, columns=None, sizes=None, **spec_kwargs) -> list:
        """One ``sparse.config.SparseTableSpec`` per sparse column (all of them, or ``columns``), named and
        fed by the column, with the column's id space (``buckets``) as its rows; ``sizes`` gives the rows
        of columns whose ids are not bucketed (an error names any column left without a size).  Further
        keyword arguments go to every spec (pooling, optimizer, shards, ...)."""
        from ..sparse.config import SparseTableSpec

        sizes = dict(sizes or {})
        wanted = list(columns) if columns is not None else [d.column for d in self.descriptors if d.kind == "sparse"]
        specs = []
        for c in wanted:
            d = self.require(c)
            if d.kind != "sparse":
                raise ValueError(f"column {c!r} is a {d.kind} feature, not a sparse one")
            rows = int(sizes.get(c, d.buckets))
            if rows <= 0:
                raise ValueError(f"sparse column {c!r} has no bounded id space: give its rows in sizes")
            specs.append(SparseTableSpec(name=c, num_embeddings=rows, embedding_dim=embedding_dim, feature=c,
                                         **spec_kwargs))
        return specs

    def to_manifest(self) -> dict:
        return {"config_digest": self.config_digest, "features": [d.to_entry() for d in self.descriptors]}

    def write_manifest(self, directory: str | Path) -> Path:
        from ..io.artifacts import write_json

        path = Path(directory) / MANIFEST_NAME
        write_json(path, self.to_manifest())
        return path

    @classmethod
    def from_manifest(cls, payload: dict) -> "FeatureCatalog":
        if not isinstance(payload, dict) or set(payload) != {"config_digest", "features"}:
            raise ValueError("a feature manifest has exactly the fields config_digest and features")
        if not isinstance(payload["features"], list):
            raise TypeError("manifest features must be a list")
        descs = []
        for e in payload["features"]:
            if not isinstance(e, dict) or set(e) != _ENTRY_FIELDS:
                raise ValueError(f"feature entry fields must be {sorted(_ENTRY_FIELDS)}")
            descs.append(FeatureDescriptor(**{**e, "source_codes": tuple(e["source_codes"])}))
        return cls(descs, config_digest=payload["config_digest"])

    @classmethod
    def from_manifest_dir(cls, directory: str | Path) -> "FeatureCatalog":
        path = Path(directory) / MANIFEST_NAME
        if not path.is_file():
            raise FileNotFoundError(f"no feature manifest at {path}")
        return cls.from_manifest(json.loads(path.read_text(encoding="utf-8")))


def config_digest(cfg) -> str:
    """SHA-256 of the parts of a ``PipelineConfig`` that decide the output columns and their values."""
    doc = {"feature_column": cfg.feature_column, "label_code": cfg.label_code,
           "dense": [asdict(d) for d in cfg.dense],
           "sparse": [{**asdict(s), "vocab": sorted((str(k), v) for k, v in dict(s.vocab).items())}
                      for s in cfg.sparse]}
    return hashlib.sha256(json.dumps(doc, sort_keys=True, default=list).encode("utf-8")).hexdigest()


def catalog_for(cfg) -> FeatureCatalog:
    """The catalog of the columns ``data.pipeline.FeatureProcessor`` writes for ``cfg``."""
    descs = [FeatureDescriptor("label", "label", "label", "identity", (cfg.label_code,))]
    for i, d in enumerate(cfg.dense):
        descs.append(FeatureDescriptor(f"d{i}", f"dense_{d.code}", "dense", d.transform, (d.code,)))
    for i, s in enumerate(cfg.sparse):
        buckets = int(s.buckets)
        if s.kind == "category":  # vocabulary indices and the default index
            buckets = max([int(v) for v in dict(s.vocab).values()] + [int(s.default)]) + 1
        elif s.kind == "intersect":  # raw ids shared by two lists: no bounded id space
            buckets = 0
        descs.append(FeatureDescriptor(f"s{i}", f"{s.kind}_" + "_".join(str(c) for c in s.codes), "sparse", s.kind,
                                       tuple(s.codes), buckets))
    return FeatureCatalog(descs, config_digest=config_digest(cfg))


__all__ = ["FeatureCatalog", "FeatureDescriptor", "MANIFEST_NAME", "catalog_for", "config_digest"]
