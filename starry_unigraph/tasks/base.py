"""Base task adapter (reference tasks/base.py:13-62).

``compute_loss`` accepts either a model-output dict (new API: score/prediction
tensors) or a runtime step result that already carries ``"loss"`` (the form the
session loop passes), so both call sites of the reference keep working.
"""
from __future__ import annotations

from typing import Any

from starry_unigraph.data.batch_data import BatchData
from starry_unigraph.data.sample_config import SampleConfig


class BaseTaskAdapter:
    task_name = "base"

    def build_sample_config(self, chunk: Any, sample_params: dict[str, Any]) -> SampleConfig:
        return SampleConfig(
            num_neighbors=list(sample_params.get("num_neighbors", [10])),
            num_layers=int(sample_params.get("num_layers", 1)),
            sample_type=str(sample_params.get("sample_type", "temporal")),
        )

    def compute_loss(self, model_output: dict[str, Any], batch: BatchData | None = None) -> Any:
        if "loss" in model_output:
            return float(model_output["loss"])
        raise NotImplementedError

    def compute_metrics(self, model_output: dict[str, Any], batch: BatchData | None = None) -> dict[str, float]:
        return dict(model_output.get("meta", {}).get("metrics", {}))

    def format_output(self, model_output: dict[str, Any], batch: BatchData | None = None) -> dict[str, Any]:
        return model_output

    def compute_loss_old_api(self, output: dict[str, Any]) -> float:
        return float(output.get("loss", 0.0))

    def format_prediction(self, output: dict[str, Any]) -> dict[str, Any]:
        return output
