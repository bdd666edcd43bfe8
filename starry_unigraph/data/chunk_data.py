"""Serialised chunk collections (reference data/chunk_data.py, broken there)."""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import torch

from .chunk_atomic import ChunkAtomic


@dataclass
class ChunkData:
    chunks: list[ChunkAtomic]

    def __len__(self) -> int:
        return len(self.chunks)

    def by_time(self) -> dict[int, list[ChunkAtomic]]:
        out: dict[int, list[ChunkAtomic]] = {}
        for c in self.chunks:
            out.setdefault(c.chunk_id[0], []).append(c)
        return out

    def save(self, path: str | Path) -> None:
        Path(path).parent.mkdir(parents=True, exist_ok=True)
        torch.save(self, path)

    @classmethod
    def load(cls, path: str | Path) -> "ChunkData":
        return torch.load(path, weights_only=False)
