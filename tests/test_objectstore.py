"""Object-store IO: S3 option sources and validation, renderings, URI resolution, retries (no network)."""
import io
import json

import pytest
from pyarrow import fs as pafs

from flare_b200.io.objectstore import ObjectStoreIO, S3Options


def test_s3_option_precedence_explicit_file_env(tmp_path):
    cfg = tmp_path / "s3.json"
    cfg.write_text(json.dumps({"endpoint": "http://minio:9000", "region": "eu-west-1"}))
    env = {"AWS_ENDPOINT_URL": "http://env:1", "AWS_REGION": "us-east-1", "AWS_ACCESS_KEY_ID": "AK",
           "AWS_SECRET_ACCESS_KEY": "SK"}
    o = S3Options.from_sources(config_file=cfg, environ=env, region="ap-south-1")
    assert o.region == "ap-south-1"          # explicit beats file and environment
    assert o.endpoint == "http://minio:9000"  # file beats environment
    assert (o.access_key, o.secret_key) == ("AK", "SK")
    assert S3Options.from_sources(environ={}).set_values() == {}


def test_s3_option_validation(tmp_path):
    with pytest.raises(ValueError, match="go together"):
        S3Options(access_key="a")
    with pytest.raises(ValueError, match="session_token"):
        S3Options(session_token="t")
    with pytest.raises(ValueError, match="profile"):
        S3Options(profile="p", access_key="a", secret_key="s")
    with pytest.raises(ValueError, match="unknown"):
        S3Options.from_sources(environ={}, bucket="x")
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps({"endpont": "x"}))
    with pytest.raises(ValueError, match="unknown"):
        S3Options.from_sources(config_file=bad, environ={})
    with pytest.raises(FileNotFoundError):
        S3Options.from_sources(config_file=tmp_path / "missing.json", environ={})
    # a profile from the environment yields to explicit keys instead of failing validation
    o = S3Options.from_sources(environ={"AWS_PROFILE": "dev"}, access_key="a", secret_key="s")
    assert o.profile is None and o.access_key == "a"
    with pytest.raises(ValueError, match="profile"):
        S3Options.from_sources(environ={}, profile="dev", access_key="a", secret_key="s")


def test_s3_option_renderings():
    o = S3Options(endpoint="http://minio:9000", access_key="a", secret_key="s", session_token="t", region="r")
    assert o.iceberg_properties() == {"s3.endpoint": "http://minio:9000", "s3.access-key-id": "a",
                                      "s3.secret-access-key": "s", "s3.session-token": "t", "s3.region": "r",
                                      "s3.path-style-access": "true"}
    assert o.object_store_options() == {"aws_endpoint": "http://minio:9000", "aws_access_key_id": "a",
                                        "aws_secret_access_key": "s", "aws_session_token": "t",
                                        "aws_region": "r", "aws_virtual_hosted_style_request": "false",
                                        "aws_allow_http": "true"}
    assert S3Options(profile="p").object_store_options() == {"aws_profile": "p"}
    with pytest.raises(ValueError, match="profile"):
        S3Options(profile="p").iceberg_properties()
    fs = o.pyarrow_filesystem()  # constructing the filesystem contacts nobody
    assert isinstance(fs, pafs.S3FileSystem) and fs.region == "r"


def test_local_paths_and_file_uris(tmp_path):
    store = ObjectStoreIO()
    store.write_json(tmp_path / "a" / "x.json", {"k": 1})
    assert store.read_json(f"file://{tmp_path}/a/x.json") == {"k": 1}
    store.write_bytes(str(tmp_path / "a" / "b" / "y.bin"), b"\x00\x01")
    assert store.exists(tmp_path / "a" / "b" / "y.bin") and not store.exists(tmp_path / "nope")
    assert store.list(tmp_path / "a") == [str(tmp_path / "a" / "x.json")]
    assert len(store.list(tmp_path / "a", recursive=True)) == 2
    assert store.list(tmp_path / "empty") == []
    store.delete(tmp_path / "a" / "x.json")
    assert not store.exists(tmp_path / "a" / "x.json")
    with pytest.raises(FileNotFoundError):
        store.read_bytes(tmp_path / "a" / "x.json")
    with pytest.raises(ValueError, match="scheme"):
        store.resolve("ftp://host/x")


def test_object_store_scheme_on_a_mock_filesystem():
    from datetime import datetime

    mock = pafs._MockFileSystem(datetime(2024, 1, 1))
    store = ObjectStoreIO(filesystems={"s3": mock})
    fs, path, scheme = store.resolve("s3://bucket/run/ckpt/meta.json")
    assert fs is mock and path == "bucket/run/ckpt/meta.json" and scheme == "s3"
    mock.create_dir("bucket/run/ckpt")
    store.write_json("s3://bucket/run/ckpt/meta.json", {"step": 7})
    assert store.read_json("s3://bucket/run/ckpt/meta.json") == {"step": 7}
    assert store.list("s3://bucket/run/ckpt") == ["bucket/run/ckpt/meta.json"]
    store.delete("s3://bucket/run/ckpt/meta.json")
    assert not store.exists("s3://bucket/run/ckpt/meta.json")


class _Flaky:
    """Duck-typed filesystem whose first reads time out."""

    def __init__(self, failures: int, message: str = "Connection timed out"):
        self.failures, self.message, self.calls = failures, message, 0

    def open_input_stream(self, path):
        self.calls += 1
        if self.calls <= self.failures:
            raise OSError(self.message)
        return io.BytesIO(b"payload")


def test_transient_errors_are_retried_and_others_are_not():
    flaky = _Flaky(2)
    assert ObjectStoreIO(filesystems={"s3": flaky}, backoff_s=0.0).read_bytes("s3://b/k") == b"payload"
    assert flaky.calls == 3
    gone = _Flaky(5)
    with pytest.raises(OSError, match="timed out"):
        ObjectStoreIO(filesystems={"s3": gone}, attempts=3, backoff_s=0.0).read_bytes("s3://b/k")
    assert gone.calls == 3
    denied = _Flaky(5, "Access Denied")
    with pytest.raises(OSError, match="Denied"):
        ObjectStoreIO(filesystems={"s3": denied}, backoff_s=0.0).read_bytes("s3://b/k")
    assert denied.calls == 1


def test_s3_credentials_come_from_one_layer():
    from flare_b200.io.objectstore import S3Options

    env = {"AWS_ACCESS_KEY_ID": "ENVKEY", "AWS_SECRET_ACCESS_KEY": "ENVSECRET", "AWS_SESSION_TOKEN": "ENVTOKEN"}
    o = S3Options.from_sources(environ=env, access_key="a", secret_key="s")
    assert (o.access_key, o.secret_key, o.session_token) == ("a", "s", None)
    o = S3Options.from_sources(environ=env)
    assert (o.access_key, o.secret_key, o.session_token) == ("ENVKEY", "ENVSECRET", "ENVTOKEN")
