"""Layered config loader, secrets/auth, JSON artifacts, HTTP session (CPU)."""
import json
import os

import pytest

from flare_b200.config.loader import LayeredConfigLoader, dict_to_cli_args, load_model_config
from flare_b200.config.secrets import ObjectStoreSettings, RestAuth, SecretValue
from flare_b200.io.artifacts import read_json, write_json
from flare_b200.io.http import get_process_http_session
from flare_b200.training.flat import DenseOptimizerConfig


def test_cli_args_roundtrip_and_layering(tmp_path, monkeypatch):
    assert dict_to_cli_args({"a": {"b_c": 1}, "flag": False, "xs": [1, 2]}) == \
        ["--a.b-c", "1", "--no-flag", "--xs", "1", "--xs", "2"]
    monkeypatch.setenv("FLARE_TEST_LR", "0.25")
    cfg = tmp_path / "opt.json"
    cfg.write_text(json.dumps({"kind": "adamw", "learning_rate": "${FLARE_TEST_LR}", "nesterov": True}))
    got = LayeredConfigLoader().load(DenseOptimizerConfig, ["--config", str(cfg), "--beta1", "0.8"])
    assert got == DenseOptimizerConfig(kind="adamw", learning_rate=0.25, beta1=0.8, nesterov=True)
    # command line wins over the file
    got = LayeredConfigLoader().load(DenseOptimizerConfig, ["--config", str(cfg), "--learning-rate", "3"])
    assert got.learning_rate == 3.0
    with pytest.raises(KeyError):
        LayeredConfigLoader().load(DenseOptimizerConfig, ["--nope", "1"])
    with pytest.raises(FileNotFoundError):
        LayeredConfigLoader().load(DenseOptimizerConfig, ["--config", str(tmp_path / "missing.json")])


def test_model_structure_file(tmp_path):
    spec = {"model": "dlrm", "bottom": [64, 32], "top": [64, 1], "num_dense": 4,
            "tables": [{"name": "a", "num_embeddings": 100, "embedding_dim": 32},
                       {"name": "b", "num_embeddings": 50, "embedding_dim": 32, "shards": 2}],
            "dense_optimizer": {"kind": "sgd", "learning_rate": 0.1}}
    p = tmp_path / "m.yaml"
    import yaml

    p.write_text(yaml.safe_dump(spec))
    name, cfg = load_model_config(p)
    assert name == "dlrm" and cfg.bottom == (64, 32) and cfg.tables[1].shards == 2
    assert cfg.dense_optimizer.kind == "sgd"
    with pytest.raises(ValueError):
        load_model_config({"model": "unknown"})


def test_secrets_and_auth(monkeypatch):
    s = SecretValue("hunter2")
    assert "hunter2" not in repr(s) and "hunter2" not in str(s) and s.value == "hunter2"
    monkeypatch.setenv("FLARE_TEST_TOKEN", "tok")
    assert RestAuth.bearer_from_environment("FLARE_TEST_TOKEN").headers() == {"Authorization": "Bearer tok"}
    assert RestAuth("basic", username="u", password=SecretValue("p")).headers()["Authorization"] == "Basic dTpw"
    assert RestAuth("oauth2", client_id="c", client_secret=SecretValue("s")).client_properties()["credential"] == "c:s"
    with pytest.raises(ValueError):
        RestAuth("bearer")
    monkeypatch.setenv("FLARE_TEST_SECRET", "sk")
    o = ObjectStoreSettings.from_options({"endpoint": "http://x", "secret_access_key": "${FLARE_TEST_SECRET}"})
    assert o.client_kwargs()["aws_secret_access_key"] == "sk" and "sk" not in repr(o)


def test_artifacts_atomic_and_exclusive(tmp_path):
    p = tmp_path / "sub" / "a.json"
    write_json(p, {"x": 1})
    assert read_json(p) == {"x": 1}
    write_json(p, {"x": 2})
    assert read_json(p) == {"x": 2}
    with pytest.raises(FileExistsError):
        write_json(p, {"x": 3}, exclusive=True)
    assert read_json(p) == {"x": 2} and not [f for f in os.listdir(p.parent) if f.endswith(".tmp")]


def test_http_session_per_process():
    s = get_process_http_session()
    assert s is get_process_http_session()
    assert s.get_adapter("https://example.invalid").max_retries.total == 5


def test_parse_group_counts():
    import pytest

    from flare_b200.config.loader import parse_group_counts

    g = ["users", "items", "ctx"]
    assert parse_group_counts("8", g) == {"users": 8, "items": 8, "ctx": 8}
    assert parse_group_counts("users:2,items:1", g, default=4) == {"users": 2, "items": 1, "ctx": 4}
    assert parse_group_counts("", g) == {}
    for bad, msg in [("0", "positive"), ("users:2,users:3", "twice"), ("nope:1", "unknown"), ("users:2:3", "name:count"),
                     ("users:x", "positive")]:
        with pytest.raises(ValueError, match=msg):
            parse_group_counts(bad, g)


def test_cli_group_ids_first_id_of_a_feature():
    import torch

    from flare_b200.cli import group_ids

    # 2 features x 3 samples: feature 1 bags = [7, 8], [], [9]
    offs = torch.tensor([0, 1, 2, 3, 5, 5, 6], dtype=torch.int32)
    vals = torch.tensor([1, 2, 3, 7, 8, 9], dtype=torch.int32)
    assert group_ids(offs, vals, 1, 3).tolist() == [7, -1, 9]
    assert group_ids(offs, vals, 0, 3).tolist() == [1, 2, 3]


def test_publish_bytes_create_mode_first_writer_wins(tmp_path):
    from flare_b200.io.artifacts import companion_file, publish_bytes

    p = tmp_path / "lease.json"
    publish_bytes(p, b"one", mode="create")
    try:
        publish_bytes(p, b"two", mode="create")
        raise AssertionError("a second create must fail")
    except FileExistsError:
        pass
    assert p.read_bytes() == b"one"
    publish_bytes(p, b"three")  # replace supersedes
    assert p.read_bytes() == b"three"
    assert not [q for q in tmp_path.iterdir() if q.name.endswith(".partial")]  # no scratch left behind
    assert companion_file(p, ".sha").name == "lease.json.sha"


def test_process_sessions_are_cached_per_settings():
    from flare_b200.io.http import HttpSettings, process_session

    a, b = process_session(), process_session()
    c = process_session(HttpSettings(retries=2))
    assert a is b and a is not c
    opts = HttpSettings().socket_options()
    import socket

    assert (socket.SOL_SOCKET, socket.SO_KEEPALIVE, 1) in opts
