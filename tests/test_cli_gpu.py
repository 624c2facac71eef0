"""CLI train -> checkpoint -> resume -> eval on one GPU (small DLRM from a model-structure file)."""
import json

import pytest

from flare_b200 import cli

pytestmark = pytest.mark.gpu


def _model_file(tmp_path):
    spec = {"model": "dlrm", "num_dense": 13, "bottom": [128, 64], "top": [64, 32],
            "tables": [{"name": f"t{i}", "num_embeddings": v, "embedding_dim": 64, "shards": 2 if i == 1 else 1}
                       for i, v in enumerate([1000, 5000, 300])]}
    p = tmp_path / "model.json"
    p.write_text(json.dumps(spec))
    return str(p)


def test_train_resume_eval(tmp_path, capsys):
    m = _model_file(tmp_path)
    ck = str(tmp_path / "ckpt")
    base = ["train", "--model-config", m, "--batch-per-gpu", "512", "--max-bag", "8", "--checkpoint-dir", ck,
            "--metrics-every", "5", "--metrics-jsonl", str(tmp_path / "m.jsonl")]
    assert cli.main(base + ["--steps", "10", "--save-every", "5", "--incremental"]) == 0
    assert cli.main(base + ["--steps", "5", "--save-every", "5", "--resume"]) == 0
    out = capsys.readouterr().out.strip().splitlines()
    assert json.loads(out[-1])["last_step"] == 15
    lines = (tmp_path / "m.jsonl").read_text().strip().splitlines()
    assert len(lines) >= 3 and "train/auc_ctr" in lines[0]
    assert cli.main(["eval", "--model-config", m, "--checkpoint-dir", ck, "--batch", "512", "--batches", "4",
                     "--max-bag", "8", "--gauc-feature", "0"]) == 0
    out = capsys.readouterr().out.strip().splitlines()
    res = json.loads(out[-1])
    assert res["step"] == 15 and res["samples"] == 2048 and 0.0 <= res["auc"] <= 1.0
    assert out[-2].startswith("[MetricsAggregator] ") and isinstance(res["gauc"], float)
