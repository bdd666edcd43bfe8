"""Model protocols for task-agnostic temporal GNNs (reference models/base.py:13-50)."""
from __future__ import annotations

from typing import Any, Protocol

from torch import Tensor

from starry_unigraph.data.batch_data import BatchData


class TemporalModel(Protocol):
    """Backbone computing node embeddings from a message-flow graph and state."""

    def forward(self, mfg: Any, state: dict[str, Tensor]) -> Tensor: ...

    def compute_state_update(self, embeddings: Tensor, batch: BatchData) -> dict[str, Tensor]: ...
