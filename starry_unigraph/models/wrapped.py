"""Backbone + head composition (reference models/wrapped.py:12-63)."""
from __future__ import annotations

from typing import Any

import torch.nn as nn
from torch import Tensor

from starry_unigraph.data.batch_data import BatchData


class WrappedModel(nn.Module):
    def __init__(self, backbone: nn.Module, head: nn.Module):
        super().__init__()
        self.backbone = backbone
        self.head = head

    def predict(self, state: dict[str, Any], batch: BatchData) -> dict[str, Tensor]:
        embeddings = self.backbone(batch.mfg, state)
        return self.head(embeddings, batch)

    def forward(self, *args, **kwargs):
        if len(args) == 2:
            return self.predict(args[0], args[1])
        return self.predict(**kwargs)
