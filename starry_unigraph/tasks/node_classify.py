"""Node classification task (reference tasks/node_classify.py:15-110): CE (or BCE for
one logit) loss, accuracy metric."""
from __future__ import annotations

from typing import Any

import torch
import torch.nn.functional as F

from starry_unigraph.data.batch_data import BatchData

from .base import BaseTaskAdapter


class NodeClassifyAdapter(BaseTaskAdapter):
    task_name = "node_classification"

    def compute_loss(self, model_output: dict[str, Any], batch: BatchData | None = None) -> Any:
        logits = model_output.get("logits")
        if logits is None or not isinstance(logits, torch.Tensor):
            return float(model_output.get("loss", 0.0))
        labels = (batch.labels if batch is not None else model_output["targets"]).to(logits.device)
        if logits.dim() == 1 or logits.size(-1) == 1:
            return F.binary_cross_entropy_with_logits(logits.flatten(), labels.float().flatten())
        return F.cross_entropy(logits, labels.long().flatten())

    def compute_metrics(self, model_output: dict[str, Any], batch: BatchData | None = None) -> dict[str, float]:
        logits = model_output.get("logits")
        labels = batch.labels if batch is not None else model_output.get("targets")
        if logits is None or labels is None or not isinstance(logits, torch.Tensor):
            return super().compute_metrics(model_output, batch)
        labels = torch.as_tensor(labels).to(logits.device).flatten()
        if logits.dim() == 1 or logits.size(-1) == 1:
            pred = (logits.flatten() > 0).long()
        else:
            pred = logits.argmax(-1)
        return {"accuracy": float((pred == labels.long()).float().mean())}
