"""Chunk utilities (reference backends/chunk/utils/utils.py)."""
from __future__ import annotations

import torch


def chunk_ranges(n: int, parts: int) -> list[tuple[int, int]]:
    per = max(1, (n + parts - 1) // max(1, parts))
    return [(i, min(n, i + per)) for i in range(0, n, per)]


def cat_or_empty(ts: list[torch.Tensor]) -> torch.Tensor:
    return torch.cat(ts) if ts else torch.zeros(0, dtype=torch.long)
