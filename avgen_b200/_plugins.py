"""Entry-point plugin loading shared by every registry (avgen/_plugins.py:36-88).

Groups: ``avgen.models``, ``avgen.metrics``, ``avgen.samplers``, ``avgen.rewards``.
A plugin that fails to import is an error naming the entry point, never a
silently missing component.
"""
from __future__ import annotations

from collections.abc import Callable
from importlib import metadata

__all__ = ["ENTRY_POINT_GROUPS", "load_entry_points"]

ENTRY_POINT_GROUPS = ("avgen.models", "avgen.metrics", "avgen.samplers", "avgen.rewards")
_LOADED: set[str] = set()


def load_entry_points(group: str, accept: Callable[[str, object], None], *, skip: set[str] | None = None,
                      force: bool = False) -> int:
    """Load every entry point of ``group`` once, handing ``(name, object)`` to ``accept``.

    Returns:
        The number of entry points loaded by this call.
    """
    if group in _LOADED and not force:
        return 0
    _LOADED.add(group)
    count = 0
    for point in sorted(metadata.entry_points(group=group), key=lambda ep: ep.name):
        if skip and point.name in skip:
            continue
        try:
            obj = point.load()
        except Exception as exc:
            raise RuntimeError(f"failed to load entry point {point.name!r} ({point.value}) from {group!r}") from exc
        accept(point.name, obj)
        count += 1
    return count
