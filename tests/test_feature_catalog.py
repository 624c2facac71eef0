"""Feature catalog of the feature pipeline: published beside the windows with the configuration digest,
matches the written columns, guards the output against another configuration, round-trips with strict
validation, and drives the published-table schema check (CPU)."""
import dataclasses

import pyarrow.parquet as pq
import pytest

from flare_b200.data.feature_catalog import MANIFEST_NAME, FeatureCatalog, FeatureDescriptor, catalog_for
from flare_b200.data.pipeline import DataPipeline


def _run(tmp_path, **kw):
    from test_pipeline import _cfg, _write_logs

    (tmp_path / "logs").mkdir(exist_ok=True)
    _write_logs(tmp_path / "logs" / "a.txt", 150, 1)
    cfg = _cfg(tmp_path, **kw)
    DataPipeline(cfg).run()
    return cfg


def test_pipeline_publishes_its_catalog_and_refuses_another_config(tmp_path):
    cfg = _run(tmp_path, iceberg_table=str(tmp_path / "ice"))
    cat = FeatureCatalog.from_manifest_dir(tmp_path / "out")
    assert cat.config_digest == catalog_for(cfg).config_digest
    files = DataPipeline(cfg).published_files()
    assert set(pq.read_schema(files[0]).names) == set(cat.columns) == {"label", "d0", "s0", "s1", "s2"}
    assert cat.column_for("cross_20_21") == "s1" and cat.require("s2").buckets == 777
    DataPipeline(cfg).run()  # the same configuration again: fine
    other = dataclasses.replace(cfg, label_code=2)
    with pytest.raises(ValueError, match="another configuration"):
        DataPipeline(other).run()

    from flare_b200.validation.iceberg import main

    assert main(["schema", str(tmp_path / "ice"), "--manifest-dir", str(tmp_path / "out")]) == 0


def test_manifest_round_trip_and_validation(tmp_path):
    cat = FeatureCatalog([FeatureDescriptor("label", "label", "label", "identity", (1,)),
                          FeatureDescriptor("s0", "hash_20", "sparse", "hash", (20,), 1000)],
                         config_digest="0" * 64)
    path = cat.write_manifest(tmp_path)
    assert path.name == MANIFEST_NAME
    back = FeatureCatalog.from_manifest_dir(tmp_path)
    assert back.descriptors == cat.descriptors and back.config_digest == cat.config_digest
    with pytest.raises(ValueError, match="SHA-256"):
        FeatureCatalog([], config_digest="abc")
    with pytest.raises(ValueError, match="duplicate column"):
        FeatureCatalog([FeatureDescriptor("a", "x", "dense", "identity", (1,))] * 2, config_digest="0" * 64)
    with pytest.raises(ValueError, match="identifier"):
        FeatureDescriptor("1bad", "x", "dense", "identity", (1,))
    with pytest.raises(ValueError, match="fields"):
        FeatureCatalog.from_manifest({"config_digest": "0" * 64, "features": [{"column": "a"}]})
    with pytest.raises(ValueError, match="not declared"):
        back.column_for("nope")


def test_table_specs_from_the_catalog(tmp_path):
    cfg = _run(tmp_path)
    cat = FeatureCatalog.from_manifest_dir(tmp_path / "out")
    specs = cat.table_specs(16, pooling="mean")
    assert [(t.name, t.num_embeddings, t.feature, t.pooling) for t in specs] == [
        ("s0", 1000, "s0", "mean"), ("s1", 500, "s1", "mean"), ("s2", 777, "s2", "mean")]
    assert cat.table_specs(8, columns=["s1"], sizes={"s1": 64})[0].num_embeddings == 64
    with pytest.raises(ValueError, match="not a sparse"):
        cat.table_specs(8, columns=["d0"])
    from test_pipeline import _cfg

    inter = catalog_for(_cfg(tmp_path, sparse=({"kind": "intersect", "codes": (30, 31)},
                                               {"kind": "category", "codes": (21,), "vocab": {"a": 0, "b": 4}})))
    with pytest.raises(ValueError, match="no bounded id space"):
        inter.table_specs(8)
    assert inter.table_specs(8, sizes={"s0": 100})[1].num_embeddings == 5
