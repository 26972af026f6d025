"""YAML configuration loading (avgen/config/loader.py:58-758 behaviour).

* ``_base_``: a path or list of paths merged first (deep merge; lists replace),
  relative to the including file; cycles are errors.
* ``${env:NAME}`` / ``${env:NAME:default}`` interpolation in strings.
* Dotted command-line overrides ``a.b[0].c=value`` (values parsed as YAML);
  list entries must already exist.
* Annotation-driven coercion into the frozen schema: bools, ints (no silent
  truncation), floats, tuples, nested dataclasses, ``Optional``.
* Unknown keys are fatal and suggest the closest known key; a few renamed keys
  redirect (``parallel.pipeline_schedule`` also accepts ``parallel.pipeline``
  as a mapping).
"""
from __future__ import annotations

import copy
import dataclasses
import difflib
import os
import re
import types
import typing
from collections.abc import Mapping, Sequence
from pathlib import Path
from typing import Any, get_args, get_origin

import yaml

from avgen_b200.config.schema import RunConfig

__all__ = ["ConfigError", "apply_overrides", "coerce", "deep_merge", "load_config", "load_mapping",
           "parse_override"]

BASE_KEY = "_base_"
_ENV = re.compile(r"\$\{env:([A-Za-z_][A-Za-z0-9_]*)(?::([^}]*))?\}")
_SEGMENT = re.compile(r"^([A-Za-z_][A-Za-z0-9_]*)((?:\[\d+\])*)$")
_TRUE = {"true", "yes", "on", "1"}
_FALSE = {"false", "no", "off", "0"}


class ConfigError(ValueError):
    """A configuration problem, with the dotted location in the message."""


def deep_merge(base: Mapping[str, Any], override: Mapping[str, Any]) -> dict[str, Any]:
    out = dict(base)
    for key, value in override.items():
        cur = out.get(key)
        out[key] = deep_merge(cur, value) if isinstance(cur, Mapping) and isinstance(value, Mapping) else value
    return out


def _interp(value: Any, where: str) -> Any:
    if isinstance(value, str):
        def sub(m: re.Match[str]) -> str:
            name, default = m.group(1), m.group(2)
            if name in os.environ:
                return os.environ[name]
            if default is not None:
                return default
            raise ConfigError(f"{where} references environment variable {name!r}, which is unset and has no default")

        return _ENV.sub(sub, value)
    if isinstance(value, dict):
        return {k: _interp(v, f"{where}.{k}") for k, v in value.items()}
    if isinstance(value, list):
        return [_interp(v, f"{where}[{i}]") for i, v in enumerate(value)]
    return value


def load_mapping(path: str | Path, *, _seen: tuple[Path, ...] = ()) -> dict[str, Any]:
    """Read a YAML file with its ``_base_`` chain merged and env vars interpolated."""
    p = Path(path).expanduser()
    if not p.is_file():
        raise ConfigError(f"config file not found: {p}")
    p = p.resolve()
    if p in _seen:
        raise ConfigError("_base_ composition is cyclic: " + " -> ".join(str(x) for x in (*_seen, p)))
    try:
        payload = yaml.safe_load(p.read_text(encoding="utf-8"))
    except yaml.YAMLError as exc:
        raise ConfigError(f"{p} is not valid YAML: {exc}") from exc
    payload = payload or {}
    if not isinstance(payload, dict):
        raise ConfigError(f"{p} must contain a mapping at the top level")
    bases = payload.pop(BASE_KEY, None)
    merged: dict[str, Any] = {}
    if bases is not None:
        entries = [bases] if isinstance(bases, str) else bases
        if not isinstance(entries, list) or not all(isinstance(e, str) for e in entries):
            raise ConfigError(f"{p}: {BASE_KEY} must be a path or a list of paths")
        for entry in entries:
            merged = deep_merge(merged, load_mapping((p.parent / entry).resolve(), _seen=(*_seen, p)))
    return typing.cast(dict, _interp(deep_merge(merged, payload), p.name))


def parse_override(text: str) -> tuple[list[str | int], Any]:
    if "=" not in text:
        raise ConfigError(f"override {text!r} is not of the form key.path=value (e.g. train.lr=1e-4)")
    key, _, raw = text.partition("=")
    key = key.strip()
    if not key:
        raise ConfigError(f"override {text!r} has an empty key")
    segments: list[str | int] = []
    for part in key.split("."):
        m = _SEGMENT.match(part)
        if m is None:
            raise ConfigError(f"override {text!r} has a malformed path segment {part!r}")
        segments.append(m.group(1))
        segments.extend(int(i) for i in re.findall(r"\[(\d+)\]", m.group(2)))
    stripped = raw.strip()
    if stripped in ("null", "~", "None"):
        return segments, None
    if stripped == "":
        return segments, ""
    try:
        value = yaml.safe_load(raw)
    except yaml.YAMLError:
        value = raw
    return segments, raw if value is None else value


def apply_overrides(mapping: Mapping[str, Any], overrides: Sequence[str]) -> dict[str, Any]:
    result = copy.deepcopy(dict(mapping))
    for text in overrides:
        segments, value = parse_override(text)
        cursor: Any = result
        for seg in segments[:-1]:
            if isinstance(seg, int):
                if not isinstance(cursor, list) or seg >= len(cursor):
                    raise ConfigError(f"override {text!r} indexes a list entry that does not exist in the config file")
                cursor = cursor[seg]
            else:
                if not isinstance(cursor, dict):
                    raise ConfigError(f"override {text!r} descends into a non-mapping")
                cursor = cursor.setdefault(seg, {})
        last = segments[-1]
        if isinstance(last, int):
            if not isinstance(cursor, list) or last >= len(cursor):
                raise ConfigError(f"override {text!r} assigns a list index that does not exist")
            cursor[last] = value
        else:
            if not isinstance(cursor, dict):
                raise ConfigError(f"override {text!r} assigns on a non-mapping")
            cursor[last] = value
    return result


def _unwrap_optional(ann: Any) -> tuple[Any, bool]:
    origin = get_origin(ann)
    if origin is typing.Union or origin is types.UnionType:
        members = [a for a in get_args(ann) if a is not type(None)]
        return (members[0] if len(members) == 1 else Any), True
    return ann, False


def coerce(ann: Any, value: Any, where: str) -> Any:
    """Convert a YAML value to the annotated schema type (raising with ``where``)."""
    ann, optional = _unwrap_optional(ann)
    if value is None:
        if optional or ann is Any:
            return None
        raise ConfigError(f"{where} may not be null")
    if ann is Any:
        return value
    if isinstance(ann, type) and dataclasses.is_dataclass(ann):
        if not isinstance(value, Mapping):
            raise ConfigError(f"{where} must be a mapping; got {value!r}")
        return build_dataclass(ann, value, where)
    if ann is bool:
        if isinstance(value, bool):
            return value
        if isinstance(value, str) and value.lower() in _TRUE | _FALSE:
            return value.lower() in _TRUE
        if isinstance(value, int) and value in (0, 1):
            return bool(value)
        raise ConfigError(f"{where} must be a boolean; got {value!r}")
    if ann is int:
        if isinstance(value, bool):
            raise ConfigError(f"{where} must be an integer; got {value!r}")
        if isinstance(value, int):
            return value
        if isinstance(value, float) and value.is_integer():
            return int(value)
        if isinstance(value, str):
            try:
                return int(value, 0)
            except ValueError:
                try:
                    f = float(value)
                except ValueError:
                    raise ConfigError(f"{where} must be an integer; got {value!r}") from None
                if f.is_integer():
                    return int(f)
        raise ConfigError(f"{where} must be an integer; got {value!r}")
    if ann is float:
        if isinstance(value, bool):
            raise ConfigError(f"{where} must be a float; got {value!r}")
        try:
            return float(value)
        except (TypeError, ValueError):
            raise ConfigError(f"{where} must be a float; got {value!r}") from None
    if ann is str:
        if isinstance(value, (dict, list)):
            raise ConfigError(f"{where} must be a string; got {value!r}")
        return str(value)
    origin = get_origin(ann)
    if origin is tuple:
        args = get_args(ann)
        items = value if isinstance(value, (list, tuple)) else [value]
        if len(args) == 2 and args[1] is Ellipsis:
            return tuple(coerce(args[0], v, f"{where}[{i}]") for i, v in enumerate(items))
        if len(args) != len(items):
            raise ConfigError(f"{where} must have {len(args)} entries; got {len(items)}")
        return tuple(coerce(a, v, f"{where}[{i}]") for i, (a, v) in enumerate(zip(args, items)))
    if origin in (dict, Mapping):
        if not isinstance(value, Mapping):
            raise ConfigError(f"{where} must be a mapping")
        return dict(value)
    if origin is list:
        return [coerce(get_args(ann)[0], v, f"{where}[{i}]") for i, v in enumerate(value)]
    if origin is typing.Literal:
        if value not in get_args(ann):
            raise ConfigError(f"{where} must be one of {get_args(ann)}; got {value!r}")
        return value
    return value


_REDIRECTS = {("parallel", "pipeline_schedule"): ("parallel", "pipeline")}


def build_dataclass(cls: type, values: Mapping[str, Any], where: str = "") -> Any:
    hints = typing.get_type_hints(cls)
    names = [f.name for f in dataclasses.fields(cls)]
    kwargs: dict[str, Any] = {}
    for key, value in values.items():
        path = f"{where}.{key}" if where else key
        if key not in hints:
            close = difflib.get_close_matches(key, names, n=1)
            hint = f"; did you mean {close[0]!r}?" if close else ""
            raise ConfigError(f"unknown config key {path!r}{hint} (known: {', '.join(names)})")
        kwargs[key] = coerce(hints[key], value, path)
    try:
        return cls(**kwargs)
    except (TypeError, ValueError) as exc:
        if isinstance(exc, ConfigError):
            raise
        raise ConfigError(str(exc)) from exc


def build(cls: type, mapping: Mapping[str, Any], *, where: str = "") -> Any:
    """Construct config dataclass ``cls`` from ``mapping`` (unknown keys and uncoercible values raise
    :class:`ConfigError` naming the dotted path ``where.field``); keyword form of :func:`build_dataclass`."""
    return build_dataclass(cls, mapping, where)


def _normalise(mapping: dict[str, Any]) -> dict[str, Any]:
    par = mapping.get("parallel")
    if isinstance(par, dict) and isinstance(par.get("pipeline"), dict):
        par = dict(par)
        par["pipeline_schedule"] = par.pop("pipeline")
        mapping = {**mapping, "parallel": par}
    return mapping


def load_config(path: str | Path | None = None, overrides: Sequence[str] = (), *,
                mapping: Mapping[str, Any] | None = None) -> RunConfig:
    """Load a :class:`RunConfig` from YAML (plus overrides), validating every field."""
    base: dict[str, Any] = load_mapping(path) if path is not None else {}
    if mapping is not None:
        base = deep_merge(base, mapping)
    merged = _normalise(apply_overrides(base, overrides))
    return build_dataclass(RunConfig, merged)
