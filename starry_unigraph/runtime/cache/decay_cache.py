"""Version-stamped cache of fetched rows that expire after ``max_versions``
steps (reference runtime/cache/decay_cache.py, a stub)."""
from __future__ import annotations

from typing import Any

from torch import Tensor


class DecayCache:
    def __init__(self, max_versions: int = 2):
        self.max_versions = int(max_versions)
        self.entries: dict[int, tuple[Tensor, Tensor]] = {}

    def put(self, version: int, ids: Tensor, rows: Tensor) -> None:
        self.entries[int(version)] = (ids, rows)

    def get(self, version: int) -> tuple[Tensor, Tensor] | None:
        return self.entries.get(int(version))

    def expire(self, current: int) -> None:
        for v in [v for v in self.entries if v <= current - self.max_versions]:
            del self.entries[v]

    def clear(self) -> None:
        self.entries.clear()

    def describe(self) -> dict[str, Any]:
        return {"versions": sorted(self.entries), "max_versions": self.max_versions}
