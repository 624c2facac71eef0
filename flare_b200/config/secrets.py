"""Secrets and REST authentication for catalog / object-store clients.

``SecretValue`` never prints its value; ``RestAuth`` (noop / bearer / basic /
oauth2 client credentials) renders request headers or client properties;
``ObjectStoreSettings`` holds endpoint + credentials read from options with
``${ENV}`` indirection.  Reference behaviour: src/flare/config/iceberg.py:
20-160 (the Iceberg catalog itself is a connector this build does not ship).
"""
from __future__ import annotations

import base64
import dataclasses
import os
from collections.abc import Mapping
from typing import Any, Literal

from .loader import resolve_environment

AuthType = Literal["noop", "bearer", "basic", "oauth2"]


@dataclasses.dataclass(frozen=True)
class SecretValue:
    _value: str = dataclasses.field(repr=False)

    def __post_init__(self) -> None:
        if not self._value:
            raise ValueError("secret value must not be empty")

    @classmethod
    def from_environment(cls, name: str) -> "SecretValue":
        v = os.environ.get(name)
        if not v:
            raise ValueError(f"missing secret environment variable: {name}")
        return cls(v)

    @property
    def value(self) -> str:
        return self._value

    def __repr__(self) -> str:
        return "SecretValue(<redacted>)"

    __str__ = __repr__


@dataclasses.dataclass(frozen=True)
class RestAuth:
    kind: AuthType = "noop"
    token: SecretValue | None = None
    username: str | None = None
    password: SecretValue | None = None
    client_id: str | None = None
    client_secret: SecretValue | None = None
    token_url: str | None = None
    scope: str | None = None

    def __post_init__(self) -> None:
        need = {"noop": (), "bearer": ("token",), "basic": ("username", "password"),
                "oauth2": ("client_id", "client_secret")}
        if self.kind not in need:
            raise ValueError(f"unsupported auth type {self.kind!r}")
        missing = [f for f in need[self.kind] if getattr(self, f) is None]
        if missing:
            raise ValueError(f"{self.kind} auth needs {missing}")

    @classmethod
    def noop(cls) -> "RestAuth":
        return cls("noop")

    @classmethod
    def bearer_from_environment(cls, name: str) -> "RestAuth":
        return cls("bearer", token=SecretValue.from_environment(name))

    def headers(self) -> dict[str, str]:
        if self.kind == "bearer":
            return {"Authorization": f"Bearer {self.token.value}"}
        if self.kind == "basic":
            raw = f"{self.username}:{self.password.value}".encode()
            return {"Authorization": "Basic " + base64.b64encode(raw).decode()}
        return {}

    def client_properties(self) -> dict[str, Any]:
        """Properties for an OAuth2-capable client (credential = id:secret, optional token URL / scope)."""
        if self.kind != "oauth2":
            return {"token": self.token.value} if self.kind == "bearer" else {}
        out = {"credential": f"{self.client_id}:{self.client_secret.value}"}
        if self.token_url:
            out["oauth2-server-uri"] = self.token_url
        if self.scope:
            out["scope"] = self.scope
        return out


@dataclasses.dataclass(frozen=True)
class ObjectStoreSettings:
    endpoint: str | None = None
    region: str | None = None
    access_key_id: str | None = None
    secret_access_key: SecretValue | None = None

    @classmethod
    def from_options(cls, options: Mapping[str, Any]) -> "ObjectStoreSettings":
        o = resolve_environment(dict(options))
        unknown = set(o) - {"endpoint", "region", "access_key_id", "secret_access_key"}
        if unknown:
            raise ValueError(f"unknown object-store options {sorted(unknown)}")
        secret = o.get("secret_access_key")
        return cls(o.get("endpoint"), o.get("region"), o.get("access_key_id"),
                   SecretValue(secret) if secret else None)

    def client_kwargs(self) -> dict[str, Any]:
        out = {}
        if self.endpoint:
            out["endpoint_url"] = self.endpoint
        if self.region:
            out["region_name"] = self.region
        if self.access_key_id:
            out["aws_access_key_id"] = self.access_key_id
        if self.secret_access_key:
            out["aws_secret_access_key"] = self.secret_access_key.value
        return out


__all__ = ["ObjectStoreSettings", "RestAuth", "SecretValue"]
