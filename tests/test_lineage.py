"""Data lineage: coalescing, recency window, bounded pending facts, export failures keeping facts,
lazy exporter, single close with aggregated failures, and the feature pipeline's facts (CPU)."""
import json
import threading

import pytest

from flare_b200.data.lineage import (AssetRef, InputRead, JsonlLineageExporter, LineageContext, LineageRecorder,
                                     OutputPublished)


class Exporter:
    def __init__(self):
        self.batches, self.closes, self.fail, self.contexts = [], 0, False, []

    def export(self, events):
        if self.fail:
            raise ValueError("delivery failed")
        self.batches.append(events)

    def close(self):
        self.closes += 1


def _recorder(exporter, **kw):
    def factory(ctx):
        exporter.contexts.append(ctx)
        return exporter
    return LineageRecorder(factory, LineageContext("run", "op"), **kw)


def test_repeated_reads_are_one_fact_and_close_is_once():
    ex = Exporter()
    rec = _recorder(ex)
    a = AssetRef("catalog", "dataset", "snapshot")
    for _ in range(100):
        rec.inputs_read([a])
    assert ex.batches == [] and rec.pending_events == (InputRead(a),)
    rec.flush()
    rec.inputs_read([a])  # exported recently: still known
    assert rec.pending_events == ()
    rec.close()
    rec.close()
    assert ex.batches == [(InputRead(a),)] and ex.closes == 1 and ex.contexts == [LineageContext("run", "op")]
    with pytest.raises(RuntimeError, match="closed"):
        rec.inputs_read([a])


def test_recency_window_and_bounded_pending():
    rec = _recorder(Exporter(), coalesce_window=2)
    first, second, third = (AssetRef("c", str(i)) for i in range(3))
    for a in (first, second):
        rec.inputs_read([a])
        rec.flush()
    rec.inputs_read([first])  # refreshes first, so second is the oldest known fact
    rec.inputs_read([third])
    rec.flush()
    rec.inputs_read([first])
    assert rec.pending_events == ()
    rec.inputs_read([second])  # evicted from the window: recorded again
    assert rec.pending_events == (InputRead(second),)

    ex = Exporter()
    rec = _recorder(ex, max_pending_events=2)
    assets = [AssetRef("files", str(i)) for i in range(3)]
    rec.inputs_read(assets)
    assert ex.batches == [(InputRead(assets[0]), InputRead(assets[1]))]
    assert rec.pending_events == (InputRead(assets[2]),)
    ex.fail = True
    with pytest.raises(ValueError, match="delivery failed"):
        rec.flush()
    assert rec.pending_events == (InputRead(assets[2]),)  # kept for the next attempt
    ex.fail = False
    rec.close()
    assert ex.batches[-1] == (InputRead(assets[2]),)


def test_unused_recorder_opens_no_exporter_and_close_reports_every_failure():
    made = []
    rec = LineageRecorder(lambda ctx: made.append(ctx) or Exporter(), LineageContext("r", "o"))
    rec.close()
    assert made == []

    class Failing(Exporter):
        def export(self, events):
            raise ValueError("delivery failed")

        def close(self):
            self.closes += 1
            raise RuntimeError("release failed")

    ex = Failing()
    rec = _recorder(ex)
    rec.output_published([AssetRef("out", "t", "v1")], "pub-1")
    with pytest.raises(ExceptionGroup, match="lineage close failed") as e:
        rec.close()
    assert [type(x) for x in e.value.exceptions] == [ValueError, RuntimeError] and ex.closes == 1
    assert rec.pending_events == (OutputPublished(AssetRef("out", "t", "v1"), "pub-1"),)


def test_threads_share_a_recorder_and_values_are_validated():
    ex = Exporter()
    rec = _recorder(ex, max_pending_events=8)
    threads = [threading.Thread(target=lambda k=k: [rec.inputs_read([AssetRef("f", f"{k}-{i}")]) for i in range(50)])
               for k in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    rec.close()
    assert sum(len(b) for b in ex.batches) == 200 and all(len(b) <= 8 for b in ex.batches)
    with pytest.raises(ValueError):
        AssetRef("ns", " padded")
    with pytest.raises(ValueError):
        OutputPublished(AssetRef("ns", "x"), "")
    with pytest.raises(TypeError):
        InputRead("not an asset")


def test_feature_pipeline_records_inputs_and_publications(tmp_path):
    from test_pipeline import _cfg, _write_logs

    from flare_b200.data.pipeline import DataPipeline

    (tmp_path / "logs").mkdir()
    for i, n in enumerate([120, 80]):
        _write_logs(tmp_path / "logs" / f"f{i}.txt", n, 3 + i)
    cfg = _cfg(tmp_path, iceberg_table=str(tmp_path / "ice"))
    out = tmp_path / "lineage.jsonl"
    rec = LineageRecorder(lambda ctx: JsonlLineageExporter(out, ctx), LineageContext("run-1", "publish"))
    DataPipeline(cfg, lineage=rec).run()
    rec.close()
    facts = [json.loads(line) for line in out.read_text().splitlines()]
    kinds = [(f["kind"], f["asset"]["namespace"]) for f in facts]
    assert kinds.count(("input_read", "file")) == 2
    assert kinds.count(("output_published", "iceberg")) == 2 and ("output_published", "parquet") in kinds
    assert all(f["run_id"] == "run-1" and f["operation_id"] == "publish" for f in facts)
