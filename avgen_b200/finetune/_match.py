"""Module-name patterns: a pattern matches when it equals a dotted component path
suffix (``"q_proj"`` matches ``blocks.3.attention.q_proj``) or, if it contains
glob characters, when ``fnmatch`` accepts the full name."""
from __future__ import annotations

import fnmatch
from collections.abc import Iterable, Sequence

__all__ = ["matches_any", "normalize_patterns"]


def normalize_patterns(patterns: Iterable[str]) -> tuple[str, ...]:
    """Strip, drop empties and duplicates, keep order."""
    out: dict[str, None] = {}
    for p in patterns:
        p = p.strip()
        if p:
            out.setdefault(p, None)
    return tuple(out)


def matches_any(name: str, patterns: Sequence[str]) -> bool:
    parts = name.split(".")
    for p in patterns:
        if any(ch in p for ch in "*?["):
            if fnmatch.fnmatchcase(name, p):
                return True
            continue
        want = p.split(".")
        n = len(want)
        if any(parts[i:i + n] == want for i in range(len(parts) - n + 1)):
            return True
    return False
