"""Feature-production pipeline (CPU): parse + encode + windowed Parquet publication, resume, leases, reconcile."""
import json

import numpy as np
import pytest

pa = pytest.importorskip("pyarrow")
pq = pytest.importorskip("pyarrow.parquet")
try:
    from flare_b200._native import native

    native().etl
except Exception:  # pragma: no cover
    pytest.skip("native extension not built", allow_module_level=True)


from flare_b200.data.pipeline import DataPipeline, Lease, PipelineConfig  # noqa: E402
from flare_b200.data.run import main as run_main  # noqa: E402


def _write_logs(path, n, seed):
    rng = np.random.default_rng(seed)
    with open(path, "w") as f:
        for i in range(n):
            items = [f"1\x03{int(rng.random() < 0.3)}", f"10\x03{rng.exponential(5):.3f}",
                     f"20\x03{rng.integers(0, 10**9)}", f"21\x03{rng.integers(0, 50)}",
                     "30\x03" + ",".join(str(x) for x in rng.integers(0, 100, rng.integers(1, 5)))]
            if rng.random() < 0.2:
                items.pop(2)
            f.write(f"u{i}\tctx\t" + "\x02".join(items) + "\n")


def _cfg(tmp_path, **kw):
    base = dict(inputs=(str(tmp_path / "logs"),), output=str(tmp_path / "out"), feature_column=2, label_code=1,
                dense=({"code": 10, "transform": "log1p"},),
                sparse=({"kind": "hash", "codes": (20,), "buckets": 1000},
                        {"kind": "cross", "codes": (20, 21), "buckets": 500},
                        {"kind": "fnv_list", "codes": (30,), "buckets": 777}),
                rows_per_file=100, files_per_window=2)
    base.update(kw)
    from flare_b200.config.loader import build_dataclass

    return build_dataclass(PipelineConfig, base)


def test_publish_resume_and_training_layout(tmp_path):
    (tmp_path / "logs").mkdir()
    _write_logs(tmp_path / "logs" / "a.txt", 350, 0)
    pipe = DataPipeline(_cfg(tmp_path))
    (tmp_path / "out").mkdir()
    (tmp_path / "out" / ".window-crashed").mkdir()      # left by a crashed run
    man = pipe.run()
    assert not list((tmp_path / "out").glob(".window-*"))
    assert [w["rows"] for w in man["windows"]] == [200, 150]
    files = pipe.published_files()
    t = pq.read_table(files[0])
    assert set(t.column_names) == {"label", "d0", "s0", "s1", "s2"}
    s0 = t.column("s0").combine_chunks()
    assert np.asarray(s0.values).max() < 1000 and len(s0) == 100
    # hash column = value mod buckets of the parsed feature
    lines = open(tmp_path / "logs" / "a.txt").read().splitlines()[:100]
    want = []
    for ln in lines:
        kv = dict(item.split("\x03") for item in ln.split("\t")[2].split("\x02"))
        want.append([int(kv["20"]) % 1000] if "20" in kv else [])
    assert s0.to_pylist() == want
    # resume: a second run publishes only the new input
    _write_logs(tmp_path / "logs" / "b.txt", 120, 1)
    man2 = DataPipeline(_cfg(tmp_path)).run()
    assert len(man2["windows"]) == 3 and man2["windows"][-1]["rows"] == 120
    # the training source reads the published files
    from flare_b200.data.sources import ParquetSourceFactory, stream_batches

    batches = list(stream_batches(ParquetSourceFactory(DataPipeline(_cfg(tmp_path)).published_files()), 64,
                                  policy="drop"))
    assert sum(b.validity.valid_count for b in batches) == 64 * (470 // 64)


def test_lease_blocks_second_publisher(tmp_path):
    out = tmp_path / "o"
    out.mkdir()
    a, b = Lease(out, 60), Lease(out, 60)
    a.acquire()
    with pytest.raises(RuntimeError):
        b.acquire()
    a.release()
    b.acquire()
    b.release()


def test_stale_lease_takeover_has_one_winner_and_renewal_detects_loss(tmp_path):
    import threading

    out = tmp_path / "o"
    out.mkdir()
    old = Lease(out, -1.0)  # already expired: a crashed publisher's lease
    old.acquire()
    contenders = [Lease(out, 60) for _ in range(8)]
    won, barrier = [], threading.Barrier(len(contenders))

    def take(lease):
        barrier.wait()
        try:
            lease.acquire()
            won.append(lease)
        except RuntimeError:
            pass

    threads = [threading.Thread(target=take, args=(c,)) for c in contenders]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert len(won) == 1
    won[0].renew()  # still the owner
    with pytest.raises(RuntimeError, match="taken over"):
        old.renew()


def test_cli(tmp_path, capsys):
    (tmp_path / "logs").mkdir()
    _write_logs(tmp_path / "logs" / "a.txt", 50, 2)
    cfg = {"inputs": [str(tmp_path / "logs")], "output": str(tmp_path / "out"), "label_code": 1,
           "sparse": [{"kind": "hash", "codes": [20], "buckets": 10}]}
    (tmp_path / "p.json").write_text(json.dumps(cfg))
    assert run_main(["--config", str(tmp_path / "p.json")]) == 0
    assert json.loads(capsys.readouterr().out)["rows"] == 50



def test_parallel_workers_and_planning(tmp_path):
    from flare_b200.data.pipeline import load_category_values, plan_groups, plan_workers

    (tmp_path / "logs").mkdir()
    for i, n in enumerate([300, 50, 120, 80]):
        _write_logs(tmp_path / "logs" / f"f{i}.txt", n, 10 + i)
    files = sorted(str(p) for p in (tmp_path / "logs").iterdir())
    groups = plan_groups(files, 2)
    assert sorted(f for g in groups for f in g) == files and len(groups) == 2
    man = DataPipeline(_cfg(tmp_path)).run(workers=2, audit_path=tmp_path / "audit.json")
    assert sum(w["rows"] for w in man["windows"]) == 550 and len(man["inputs_done"]) == 4
    audit = json.loads((tmp_path / "audit.json").read_text())
    assert audit["total_rows"] == 550 and audit["groups"] == 2 and sorted(audit["source_rows"]) == files
    assert audit["data_files"] >= 4 and audit["max_worker_rss_bytes"] > 0 and len(audit["code_sha256"]) == 64
    assert plan_workers(cpus=64, memory_bytes=256 << 30, cpus_per_worker=4, memory_per_worker=8 << 30) == 15
    with pytest.raises(ValueError):
        plan_workers(cpus=4, memory_bytes=1 << 30, cpus_per_worker=8, memory_per_worker=1 << 20)
    (tmp_path / "colors.txt").write_text("red\ngreen\n\nblue\n")
    vals, auto = load_category_values({"c": "colors.txt", "d": "auto"}, tmp_path)
    assert vals["c"] == {"red": 0, "green": 1, "blue": 2} and auto == {"d"}


def test_zstd_inputs_encode_like_plain_ones(tmp_path):
    plain, packed = tmp_path / "p", tmp_path / "z"
    (plain / "logs").mkdir(parents=True)
    (packed / "logs").mkdir(parents=True)
    _write_logs(plain / "logs" / "a.txt", 230, 4)
    with pa.CompressedOutputStream(str(packed / "logs" / "a.txt.zst"), "zstd") as out:
        out.write((plain / "logs" / "a.txt").read_bytes())
    tabs = []
    for root in (plain, packed):
        DataPipeline(_cfg(root)).run()
        files = sorted((root / "out").rglob("*.parquet"))
        tabs.append(pa.concat_tables([pq.read_table(f) for f in files]))
    assert tabs[0].num_rows == tabs[1].num_rows == 230 and tabs[0].equals(tabs[1])


def test_encode_batch_tuning():
    from flare_b200.data.tuning import MIB, choose_encoded_batch, estimate_row_bytes

    narrow = pa.schema([("label", pa.float32()), ("d0", pa.float32()), ("s0", pa.list_(pa.int32()))])
    wide = pa.schema([(f"s{i}", pa.list_(pa.int64())) for i in range(600)])
    assert estimate_row_bytes(narrow) < estimate_row_bytes(wide)
    assert estimate_row_bytes(wide) >= 32 * 1024
    t = choose_encoded_batch(narrow, worker_memory_bytes=4 << 30)
    assert t.batch_bytes == 128 * MIB and t.rows_per_batch == 128 * MIB // t.row_bytes
    assert choose_encoded_batch(wide, worker_memory_bytes=4 << 30).batch_bytes == 256 * MIB
    # a smaller worker steps the automatic choice down; a supplied size is kept or refused
    assert choose_encoded_batch(wide, worker_memory_bytes=512 * MIB).batch_bytes == 64 * MIB
    assert choose_encoded_batch(narrow, worker_memory_bytes=4 << 30, supplied=32 * MIB).batch_bytes == 32 * MIB
    with pytest.raises(ValueError, match="fits"):
        choose_encoded_batch(narrow, worker_memory_bytes=64 * MIB)
