"""Node regression task (reference tasks/node_regression.py:15-110): MSE loss, MAE/RMSE metrics."""
from __future__ import annotations

from typing import Any

import torch
import torch.nn.functional as F

from starry_unigraph.data.batch_data import BatchData

from .base import BaseTaskAdapter


class NodeRegressionTaskAdapter(BaseTaskAdapter):
    task_name = "node_regression"

    def compute_loss(self, model_output: dict[str, Any], batch: BatchData | None = None) -> Any:
        if "loss" in model_output and "predictions" not in model_output:
            return float(model_output["loss"])
        if "loss" in model_output and not isinstance(model_output.get("predictions"), torch.Tensor):
            return float(model_output["loss"])
        pred = model_output["predictions"].float().flatten()
        target = (batch.labels if batch is not None else model_output["targets"]).float().flatten().to(pred.device)
        return F.mse_loss(pred, target)

    def compute_metrics(self, model_output: dict[str, Any], batch: BatchData | None = None) -> dict[str, float]:
        pred = model_output.get("predictions")
        target = batch.labels if batch is not None else model_output.get("targets")
        if pred is None or target is None:
            return super().compute_metrics(model_output, batch)
        pred = torch.as_tensor(pred, dtype=torch.float32).flatten()
        target = torch.as_tensor(target, dtype=torch.float32).flatten()
        n = min(pred.numel(), target.numel())
        if n == 0:
            return {}
        err = pred[:n] - target[:n]
        return {"mae": float(err.abs().mean()), "rmse": float(err.pow(2).mean().sqrt())}


NodeRegressAdapter = NodeRegressionTaskAdapter
