"""Model registry with entry-point plugins (avgen/models/registry.py:95-282).

``@register_model("name")`` records a model class and infers its config
dataclass from the constructor annotation; ``build_model(name, mapping)``
validates keys and builds the model. Third-party models load lazily from the
``avgen.models`` entry-point group, failing loudly.
"""
from __future__ import annotations

import inspect
from collections.abc import Callable, Mapping
from dataclasses import fields, is_dataclass
from typing import Any, TypeVar, get_type_hints

from torch import nn

from avgen_b200._plugins import load_entry_points

__all__ = ["MODEL_ENTRY_POINT_GROUP", "build_model", "list_models", "model_config_class", "register_model"]

MODEL_ENTRY_POINT_GROUP = "avgen.models"
_MODELS: dict[str, type[nn.Module]] = {}
_CONFIGS: dict[str, type] = {}
_T = TypeVar("_T", bound=nn.Module)


def _config_class_for(cls: type) -> type:
    declared = getattr(cls, "config_class", None)
    if isinstance(declared, type):
        return declared
    params = list(inspect.signature(cls, eval_str=True).parameters.values())
    if not params:
        raise TypeError(f"{cls.__name__} must take a config dataclass as its first constructor argument")
    ann = params[0].annotation
    if not isinstance(ann, type) or not is_dataclass(ann):
        raise TypeError(f"{cls.__name__}.__init__ first parameter must be annotated with a config dataclass")
    return ann


def register_model(name: str) -> Callable[[type[_T]], type[_T]]:
    """Class decorator registering a model under ``name``."""
    if not name or name.strip() != name:
        raise ValueError(f"model name must be a non-empty trimmed string; got {name!r}")

    def decorate(cls: type[_T]) -> type[_T]:
        if name in _MODELS and _MODELS[name] is not cls:
            raise ValueError(f"model {name!r} is already registered")
        if not issubclass(cls, nn.Module):
            raise TypeError(f"{cls.__name__} must subclass nn.Module")
        _MODELS[name] = cls
        _CONFIGS[name] = _config_class_for(cls)
        return cls

    return decorate


def _accept(name: str, obj: object) -> None:
    if name in _MODELS:
        return
    if not (isinstance(obj, type) and issubclass(obj, nn.Module)):
        raise RuntimeError(f"model entry point {name!r} must resolve to an nn.Module subclass; got {obj!r}")
    _MODELS[name] = obj
    _CONFIGS[name] = _config_class_for(obj)


def _resolve(name: str) -> type[nn.Module]:
    import avgen_b200.models.dit  # noqa: F401  (registers the built-in models)

    if name not in _MODELS:
        load_entry_points(MODEL_ENTRY_POINT_GROUP, _accept, skip=set(_MODELS))
    try:
        return _MODELS[name]
    except KeyError:
        raise KeyError(f"unknown model {name!r}; registered models: {', '.join(sorted(_MODELS)) or '<none>'}. "
                       f"Third-party models must advertise an entry point in {MODEL_ENTRY_POINT_GROUP!r}.") from None


def list_models() -> tuple[str, ...]:
    import avgen_b200.models.dit  # noqa: F401

    load_entry_points(MODEL_ENTRY_POINT_GROUP, _accept, skip=set(_MODELS))
    return tuple(sorted(_MODELS))


def model_config_class(name: str) -> type:
    _resolve(name)
    return _CONFIGS[name]


def _coerce(config_class: type, values: Mapping[str, Any]) -> dict[str, Any]:
    known = {f.name for f in fields(config_class)}
    unknown = sorted(set(values) - known)
    if unknown:
        raise ValueError(f"unknown config field(s) for {config_class.__name__}: {', '.join(unknown)}; "
                         f"known fields: {', '.join(sorted(known))}")
    hints = get_type_hints(config_class)
    out: dict[str, Any] = {}
    for key, value in values.items():
        ftype = hints.get(key)
        if isinstance(value, Mapping) and isinstance(ftype, type) and is_dataclass(ftype):
            out[key] = ftype(**value)
        else:
            out[key] = value
    return out


def build_model(name: str, config: Mapping[str, Any] | None = None) -> nn.Module:
    """Build a registered model from a plain mapping of config fields."""
    cls = _resolve(name)
    cfg_cls = _CONFIGS[name]
    return cls(cfg_cls(**_coerce(cfg_cls, config or {})))
