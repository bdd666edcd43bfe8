"""State-manager contract of the unified runtime (reference runtime/state/base.py:32):
prepare (gather state for a batch), patch (merge fetched remote rows), update
(write results back), step (advance versions)."""
from __future__ import annotations

from typing import Any, Protocol

from torch import Tensor


class StateManagerBase(Protocol):
    def prepare(self, node_ids: Tensor, timestamps: Tensor | None = None) -> dict[str, Any]: ...

    def patch(self, node_ids: Tensor, rows: Tensor) -> None: ...

    def update(self, model_output: dict[str, Tensor], chunk: Any) -> None: ...

    def step(self) -> None: ...

    def reset(self) -> None: ...

    def describe(self) -> dict[str, Any]: ...
