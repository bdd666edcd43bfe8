"""TaskAdapter protocol: task logic independent of the graph mode
(reference registry/task_adapter.py:73-178)."""
from __future__ import annotations

from typing import Any, Protocol

from torch import Tensor

from starry_unigraph.data.batch_data import BatchData
from starry_unigraph.data.sample_config import SampleConfig


class TaskAdapter(Protocol):
    def build_sample_config(self, chunk: Any, sample_params: dict[str, Any]) -> SampleConfig: ...

    def compute_loss(self, model_output: dict[str, Tensor], batch: BatchData | None = None) -> Any: ...

    def compute_metrics(self, model_output: dict[str, Tensor], batch: BatchData | None = None) -> dict[str, float]: ...

    def format_output(self, model_output: dict[str, Tensor], batch: BatchData | None = None) -> dict[str, Any]: ...


__all__ = ["TaskAdapter", "SampleConfig", "BatchData"]
