"""Object-store and local file IO behind one URI interface (S3 / GCS / HDFS / local) on ``pyarrow.fs``.

``S3Options`` collects S3 connection settings from, in order of precedence,
explicit arguments, an optional JSON file, and the standard ``AWS_*``
environment variables, and validates them: an access key needs its secret
(and a session token needs both), and a named profile excludes explicit
keys.  It renders them for ``pyarrow.fs.S3FileSystem`` (path-style
addressing when an endpoint is set, as self-hosted stores expect), for
Iceberg catalogs (``s3.*`` properties) and for object_store-style clients
(``aws_*`` options).

``ObjectStoreIO`` resolves ``s3://``, ``s3a://``, ``s3n://``, ``gs://``,
``hdfs://``, ``file://`` and plain paths to a filesystem once per scheme and
offers whole-object reads and writes, existence checks, listing and
deletion, retrying transient failures with exponential back-off.  Local
writes are atomic (``io.artifacts.publish_bytes``); an object-store PUT is
atomic by itself.

Reference behaviour: src/flare/io/aws.py:12-160 (S3Config, option
normalisation, the s3 file IO used by Iceberg, the pyarrow S3 filesystem).
"""
from __future__ import annotations

import json
import os
import time
from collections.abc import Mapping
from dataclasses import dataclass, fields
from pathlib import Path
from typing import Any

from pyarrow import fs as pafs

from .artifacts import publish_bytes

# the AWS SDK's standard environment variables
_ENV = {"endpoint": "AWS_ENDPOINT_URL", "access_key": "AWS_ACCESS_KEY_ID", "secret_key": "AWS_SECRET_ACCESS_KEY",
        "session_token": "AWS_SESSION_TOKEN", "region": "AWS_REGION", "profile": "AWS_PROFILE"}


@dataclass(frozen=True)
class S3Options:
    endpoint: str | None = None
    access_key: str | None = None
    secret_key: str | None = None
    session_token: str | None = None
    region: str | None = None
    profile: str | None = None

    def __post_init__(self) -> None:
        has_key, has_secret = bool(self.access_key), bool(self.secret_key)
        if has_key != has_secret:
            raise ValueError("S3 access_key and secret_key go together")
        if self.session_token and not has_key:
            raise ValueError("an S3 session_token needs access_key and secret_key")
        if self.profile and (has_key or self.session_token):
            raise ValueError("an S3 profile cannot be combined with explicit keys")

    @classmethod
    def from_sources(cls, *, config_file: str | os.PathLike | None = None, environ: Mapping[str, str] | None = None,
                     **explicit: str | None) -> "S3Options":
        """Explicit values first, then the JSON file's keys, then ``AWS_*`` variables; empty values count as
        unset.  Unknown keys (in ``explicit`` or the file) are an error.  The access key, secret and session
        token are one credential: all three come from the first layer that sets any of them, so a session
        token from the environment is never attached to keys given explicitly or in the file."""
        names = {f.name for f in fields(cls)}
        cred = ("access_key", "secret_key", "session_token")
        merged: dict[str, Any] = {}
        cred_layer = None
        layers: list[Mapping[str, Any]] = [{k: v for k, v in explicit.items()}]
        if config_file is not None:
            p = Path(config_file)
            if not p.is_file():
                raise FileNotFoundError(str(p))
            layers.append(json.loads(p.read_text(encoding="utf-8")))
        env = os.environ if environ is None else environ
        layers.append({k: env.get(v) for k, v in _ENV.items()})
        for layer in layers:
            unknown = sorted(set(layer) - names)
            if unknown:
                raise ValueError(f"unknown S3 option keys: {unknown}")
            if cred_layer is None and any(layer.get(k) not in (None, "") for k in cred):
                cred_layer = layer
            for k, v in layer.items():
                if k in cred and layer is not cred_layer:
                    continue
                if k not in merged and v not in (None, ""):
                    merged[k] = v
        # a profile from the environment yields to keys given explicitly or in the file
        if "profile" in merged and "access_key" in merged and "profile" not in explicit:
            merged.pop("profile")
        return cls(**merged)

    def set_values(self) -> dict[str, str]:
        return {f.name: getattr(self, f.name) for f in fields(self) if getattr(self, f.name)}

    def pyarrow_filesystem(self) -> pafs.S3FileSystem:
        """An S3 filesystem with these settings.  A profile has no constructor argument: the AWS SDK's own
        credential chain resolves it (``AWS_PROFILE`` / the shared config files)."""
        kw: dict[str, Any] = {}
        if self.endpoint:
            kw["endpoint_override"] = self.endpoint
            kw["force_virtual_addressing"] = False
            if self.endpoint.startswith("http://"):
                kw["scheme"] = "http"
        for ours, theirs in (("access_key", "access_key"), ("secret_key", "secret_key"),
                             ("session_token", "session_token"), ("region", "region")):
            if getattr(self, ours):
                kw[theirs] = getattr(self, ours)
        return pafs.S3FileSystem(**kw)

    def iceberg_properties(self) -> dict[str, str]:
        """``s3.*`` catalog / file-IO properties (profiles are not expressible there)."""
        if self.profile:
            raise ValueError("Iceberg S3 properties cannot name a profile; use explicit keys")
        keys = {"endpoint": "s3.endpoint", "access_key": "s3.access-key-id", "secret_key": "s3.secret-access-key",
                "session_token": "s3.session-token", "region": "s3.region"}
        out = {keys[k]: v for k, v in self.set_values().items() if k in keys}
        if self.endpoint:
            out["s3.path-style-access"] = "true"
        return out

    def object_store_options(self) -> dict[str, str]:
        """``aws_*`` options of object_store-style clients (Vortex, Lance, ...)."""
        keys = {"endpoint": "aws_endpoint", "access_key": "aws_access_key_id",
                "secret_key": "aws_secret_access_key", "session_token": "aws_session_token",
                "region": "aws_region", "profile": "aws_profile"}
        out = {keys[k]: v for k, v in self.set_values().items()}
        if self.endpoint:
            out["aws_virtual_hosted_style_request"] = "false"
            if self.endpoint.startswith("http://"):
                out["aws_allow_http"] = "true"
        return out


_TRANSIENT = ("timed out", "timeout", "temporarily", "throttl", "slow down", "503", "500", "connection reset",
              "connection refused", "try again")


def _transient(exc: BaseException) -> bool:
    if isinstance(exc, (FileNotFoundError, IsADirectoryError, NotADirectoryError, PermissionError)):
        return False
    msg = str(exc).lower()
    return isinstance(exc, (OSError, TimeoutError)) and any(t in msg for t in _TRANSIENT)


class ObjectStoreIO:
    """Whole-object IO on URIs; one filesystem per scheme, transient failures retried."""

    def __init__(self, s3: S3Options | None = None, *, attempts: int = 4, backoff_s: float = 0.5,
                 filesystems: Mapping[str, pafs.FileSystem] | None = None):
        self.s3 = s3
        self.attempts, self.backoff_s = max(1, int(attempts)), float(backoff_s)
        self._fs: dict[str, pafs.FileSystem] = dict(filesystems or {})

    # ------------------------------------------------------------ resolution
    def resolve(self, uri: str | os.PathLike) -> tuple[pafs.FileSystem, str, str]:
        """(filesystem, path inside it, scheme) of ``uri``."""
        uri = str(uri)
        scheme, sep, rest = uri.partition("://")
        if not sep:
            scheme, rest = "file", uri
        scheme = scheme.lower()
        if scheme not in self._fs:
            if scheme == "file":
                self._fs[scheme] = pafs.LocalFileSystem()
            elif scheme in ("s3", "s3a", "s3n"):
                self._fs[scheme] = (self.s3 or S3Options.from_sources()).pyarrow_filesystem()
            elif scheme in ("gs", "gcs"):
                self._fs[scheme] = pafs.GcsFileSystem()
            elif scheme == "hdfs":
                host, _, _ = rest.partition("/")
                self._fs[scheme] = pafs.HadoopFileSystem.from_uri(f"hdfs://{host}")
            else:
                raise ValueError(f"unsupported URI scheme {scheme!r}")
        path = rest
        if scheme == "hdfs":
            path = "/" + rest.partition("/")[2]
        elif scheme == "file":
            path = str(Path(rest).absolute())
        return self._fs[scheme], path, scheme

    def _retry(self, what: str, fn):
        delay = self.backoff_s
        for attempt in range(self.attempts):
            try:
                return fn()
            except Exception as exc:  # noqa: BLE001 - classified below
                if attempt + 1 == self.attempts or not _transient(exc):
                    raise
                time.sleep(delay)
                delay *= 2
        raise AssertionError(what)  # unreachable

    # ------------------------------------------------------------------- IO
    def read_bytes(self, uri) -> bytes:
        fs, path, _ = self.resolve(uri)

        def read():
            with fs.open_input_stream(path) as f:
                return f.read()
        return self._retry("read", read)

    def write_bytes(self, uri, data: bytes) -> None:
        fs, path, scheme = self.resolve(uri)
        if scheme == "file" and isinstance(fs, pafs.LocalFileSystem):
            publish_bytes(path, data)  # rename into place: readers never see a partial file
            return

        def write():
            with fs.open_output_stream(path) as f:
                f.write(data)
        self._retry("write", write)

    def read_json(self, uri) -> Any:
        return json.loads(self.read_bytes(uri).decode("utf-8"))

    def write_json(self, uri, value: Any) -> None:
        self.write_bytes(uri, (json.dumps(value, indent=2, sort_keys=True) + "\n").encode("utf-8"))

    def exists(self, uri) -> bool:
        fs, path, _ = self.resolve(uri)
        info = self._retry("stat", lambda: fs.get_file_info(path))
        return info.type != pafs.FileType.NotFound

    def list(self, uri, *, recursive: bool = False) -> list[str]:
        """Files under a directory / prefix, as paths inside the filesystem, sorted."""
        fs, path, _ = self.resolve(uri)
        sel = pafs.FileSelector(path, allow_not_found=True, recursive=recursive)
        infos = self._retry("list", lambda: fs.get_file_info(sel))
        return sorted(i.path for i in infos if i.type == pafs.FileType.File)

    def delete(self, uri) -> None:
        fs, path, _ = self.resolve(uri)
        self._retry("delete", lambda: fs.delete_file(path))


__all__ = ["ObjectStoreIO", "S3Options"]
