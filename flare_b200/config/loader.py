"""Layered configuration: dataclass defaults <- config file (JSON / YAML) <- command-line overrides.

``LayeredConfigLoader.load(ConfigType, argv)`` finds ``--config PATH`` (or
``--user-config`` / ``--config-file``) in ``argv``, reads the file, turns it
into dotted overrides (``dict_to_cli_args``), appends the remaining command
line (later wins) and builds the nested dataclass, converting every value to
its field's type.  ``${NAME}`` strings are replaced by environment variables.
``load_model_config`` reads a model-structure file (``{"model": "dlrm",
...}``) into the matching config dataclass.  Reference behaviour:
src/flare/config/loader.py:14-120 (tyro based; this one parses dataclasses
directly).
"""
from __future__ import annotations

import dataclasses
import json
import os
import re
import types
import typing
from collections.abc import Callable, Mapping, Sequence
from pathlib import Path
from typing import Any, TypeVar

T = TypeVar("T")
_ENV = re.compile(r"^\$\{([A-Za-z_][A-Za-z0-9_]*)\}$")


def resolve_environment(value: Any) -> Any:
    """Replace ``"${NAME}"`` strings (recursively) by the environment variable; a missing one raises."""
    if isinstance(value, str):
        m = _ENV.match(value)
        if m:
            if m.group(1) not in os.environ:
                raise KeyError(f"missing environment variable {m.group(1)}")
            return os.environ[m.group(1)]
        return value
    if isinstance(value, Mapping):
        return {k: resolve_environment(v) for k, v in value.items()}
    if isinstance(value, list):
        return [resolve_environment(v) for v in value]
    return value


def _flatten(config: Mapping[str, Any], prefix: str = "") -> list[tuple[str, Any]]:
    """Leaves of a nested mapping as (dotted path, value), in the mapping's order; None leaves dropped."""
    out: list[tuple[str, Any]] = []
    pending: list[tuple[str, Any]] = [(prefix, config)]
    while pending:
        path, node = pending.pop()
        if isinstance(node, Mapping):
            # pushed in reverse so the mapping's own order comes out first
            pending.extend((f"{path}{k}." if isinstance(v, Mapping) else f"{path}{k}", v)
                           for k, v in reversed(list(node.items())))
        elif node is not None:
            out.append((path, node))
    return out


def _cli_tokens(flag: str, value: Any) -> list[str]:
    """One leaf in the command-line grammar of the configs."""
    if isinstance(value, bool):
        return [f"--{flag}" if value else f"--no-{flag}"]
    if isinstance(value, (list, tuple)):
        tokens: list[str] = []
        for item in value:  # the flag repeats once per item; structured items travel as JSON
            tokens += [f"--{flag}", json.dumps(item) if isinstance(item, (Mapping, list)) else str(item)]
        return tokens
    return [f"--{flag}", str(value)]


def dict_to_cli_args(config: Mapping[str, Any], prefix: str = "") -> list[str]:
    """Nested mapping -> ``--a.b-c value`` arguments (bools: ``--x`` / ``--no-x``; lists repeat the flag).

    The grammar is the configs' command-line interface: dotted paths for nesting, ``-`` for ``_``
    in names, ``None`` values left out."""
    args: list[str] = []
    for path, value in _flatten(config, prefix):
        args += _cli_tokens(path.replace("_", "-"), value)
    return args


def _read_file(path: Path) -> dict:
    text = path.read_text(encoding="utf-8")
    if path.suffix in (".yaml", ".yml"):
        import yaml

        data = yaml.safe_load(text)
    else:
        data = json.loads(text)
    if not isinstance(data, dict):
        raise TypeError(f"configuration file must hold a mapping, got {type(data).__name__}")
    return resolve_environment(data)


def _field_types(cls) -> dict[str, Any]:
    hints = typing.get_type_hints(cls)
    return {f.name: hints[f.name] for f in dataclasses.fields(cls)}


def _convert(tp, raw):
    origin = typing.get_origin(tp)
    args = typing.get_args(tp)
    if origin is typing.Union or origin is types.UnionType:
        non_none = [a for a in args if a is not type(None)]
        if raw in ("None", "none", "null", None):
            return None
        return _convert(non_none[0], raw)
    if origin in (list, tuple, Sequence):
        items = list(raw) if isinstance(raw, (list, tuple)) else [raw]
        inner = args[0] if args else str
        vals = [_convert(inner, x) for x in items]
        return tuple(vals) if origin is tuple else vals
    if tp is bool:
        if isinstance(raw, bool):
            return raw
        if str(raw).lower() in ("1", "true", "yes"):
            return True
        if str(raw).lower() in ("0", "false", "no"):
            return False
        raise ValueError(f"not a boolean: {raw!r}")
    if tp in (int, float, str):
        return tp(raw)
    if dataclasses.is_dataclass(tp):
        if isinstance(raw, str):
            raw = json.loads(raw)
        if isinstance(raw, Mapping):
            return build_dataclass(tp, raw)
    return raw


def build_dataclass(cls: type[T], values: Mapping[str, Any]) -> T:
    """Nested dataclass from a nested mapping of raw values (unknown keys raise)."""
    types = _field_types(cls)
    kw = {}
    for k, v in values.items():
        key = k.replace("-", "_")
        if key not in types:
            raise KeyError(f"{cls.__name__} has no field {k!r}")
        tp = types[key]
        if dataclasses.is_dataclass(tp) and isinstance(v, Mapping):
            kw[key] = build_dataclass(tp, v)
        else:
            kw[key] = _convert(tp, v)
    return cls(**kw)


def _args_to_tree(cls, argv: Sequence[str]) -> dict:
    tree: dict = {}
    i = 0
    while i < len(argv):
        a = argv[i]
        if not a.startswith("--"):
            raise ValueError(f"unexpected argument {a!r}")
        name = a[2:]
        value: Any
        if i + 1 < len(argv) and not argv[i + 1].startswith("--"):
            value, i = argv[i + 1], i + 2
        else:
            neg = name.split(".")[-1].startswith("no-")
            if neg:
                parts = name.split(".")
                parts[-1] = parts[-1][3:]
                name = ".".join(parts)
            value, i = (not neg), i + 1
        parts = [p.replace("-", "_") for p in name.split(".")]
        node = tree
        for p in parts[:-1]:
            node = node.setdefault(p, {})
        leaf = parts[-1]
        # repeated flags of a list field accumulate
        ftype = None
        try:
            sub = cls
            for p in parts[:-1]:
                sub = _field_types(sub)[p]
            ftype = _field_types(sub).get(leaf)
        except (KeyError, TypeError):
            pass
        if typing.get_origin(ftype) in (list, tuple, Sequence):
            node.setdefault(leaf, [])
            if not isinstance(node[leaf], list):
                node[leaf] = [node[leaf]]
            node[leaf].append(value)
        else:
            node[leaf] = value
    return tree


def _merge(a: dict, b: dict) -> dict:
    out = dict(a)
    for k, v in b.items():
        out[k] = _merge(out[k], v) if isinstance(v, dict) and isinstance(out.get(k), dict) else v
    return out


class LayeredConfigLoader:
    def __init__(self, *, config_arg_names: Sequence[str] = ("--config", "--user-config", "--config-file"),
                 auto_config_resolver: Callable[[Sequence[str]], Path | None] | None = None):
        self.config_arg_names = tuple(config_arg_names)
        self.auto_config_resolver = auto_config_resolver

    def load(self, cls: type[T], argv: Sequence[str] | None = None) -> T:
        argv = list(argv or [])
        path, rest = None, []
        i = 0
        while i < len(argv):
            if argv[i] in self.config_arg_names and i + 1 < len(argv):
                path = path or Path(argv[i + 1])
                i += 2
                continue
            rest.append(argv[i])
            i += 1
        if path is None and self.auto_config_resolver is not None:
            path = self.auto_config_resolver(rest)
        file_tree = {}
        if path is not None:
            if not path.is_file():
                raise FileNotFoundError(f"configuration file not found: {path}")
            file_tree = _args_to_tree(cls, dict_to_cli_args(_read_file(path)))
        tree = _merge(file_tree, _args_to_tree(cls, rest))
        return build_dataclass(cls, tree)


def parse_group_counts(arg: str, groups: Sequence[str], *, default: int | None = None,
                       what: str = "count") -> dict[str, int]:
    """``"8"`` (every group) or ``"users:2,items:1"`` (per group, the rest ``default``) -> {group: count}.

    Counts are positive integers; unknown or repeated groups are errors.  The same knob grammar as
    the reference's sparse worker counts (recipes/recsys/ranking/schema/sparse_features.py:14-43)."""
    def positive(v: str, label: str) -> int:
        try:
            n = int(v)
        except ValueError:
            raise ValueError(f"{label} must be a positive integer, got {v!r}") from None
        if n < 1:
            raise ValueError(f"{label} must be a positive integer, got {v!r}")
        return n

    names = list(dict.fromkeys(groups))
    out = {} if default is None else dict.fromkeys(names, default)
    arg = arg.strip()
    if not arg:
        return out
    if ":" not in arg:
        return dict.fromkeys(names, positive(arg, what))
    seen: set[str] = set()
    for item in arg.split(","):
        parts = [x.strip() for x in item.split(":")]
        if len(parts) != 2:
            raise ValueError(f"{what} overrides are name:count, got {item!r}")
        name, v = parts
        if name not in names:
            raise ValueError(f"unknown group {name!r} (known: {names})")
        if name in seen:
            raise ValueError(f"group {name!r} given twice")
        out[name] = positive(v, f"{what} of {name!r}")
        seen.add(name)
    return out


def load_model_config(source: str | Path | Mapping[str, Any]):
    """Model-structure file -> (model name, config dataclass) for ``dlrm``, ``dcn`` or ``seqrec``."""
    raw = dict(source) if isinstance(source, Mapping) else _read_file(Path(source))
    name = raw.pop("model", None)
    if name == "dlrm":
        from ..models.dlrm import DLRMConfig as C
    elif name == "dcn":
        from ..models.dcn import DCNConfig as C
    elif name == "seqrec":
        from ..models.seqrec import SeqRecConfig as C
    else:
        raise ValueError(f"model must be one of dlrm, dcn, seqrec; got {name!r}")
    return name, build_dataclass(C, raw)


__all__ = ["LayeredConfigLoader", "build_dataclass", "dict_to_cli_args", "load_model_config", "parse_group_counts",
           "resolve_environment"]
