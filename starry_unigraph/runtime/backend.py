"""Graph-mode abstractions of the unified pipeline (reference runtime/backend.py:15-96)."""
from __future__ import annotations

from typing import Any, Iterator, Protocol

from torch import Tensor

from starry_unigraph.data.chunk_atomic import ChunkAtomic


class GraphBackend(Protocol):
    """Provides the chunks of an epoch (CTDG batches, DTDG windows, chunks)."""

    def iter_batches(self, split: str, batch_size: int) -> Iterator[ChunkAtomic]: ...

    def reset(self) -> None: ...

    def describe(self) -> dict[str, Any]: ...


class StateManager(Protocol):
    """Prepares model state for a batch and applies updates after it."""

    def prepare(self, node_ids: Tensor, timestamps: Tensor | None = None) -> dict[str, Any]: ...

    def update(self, model_output: dict[str, Tensor], chunk: ChunkAtomic) -> None: ...

    def reset(self) -> None: ...

    def describe(self) -> dict[str, Any]: ...
