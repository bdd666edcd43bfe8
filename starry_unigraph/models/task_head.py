"""Task heads (reference models/task_head.py:13-137)."""
from __future__ import annotations

import torch
import torch.nn as nn
from torch import Tensor

from starry_unigraph.data.batch_data import BatchData


class EdgePredictHead(nn.Module):
    """Dot-product edge scorer: score(u, v) = <z_u, z_v>."""

    def __init__(self, embedding_dim: int):
        super().__init__()
        self.embedding_dim = embedding_dim
        self.scorer = nn.Identity()

    def forward(self, embeddings: Tensor, batch: BatchData) -> dict[str, Tensor]:
        def score(a, b):
            if a is None or b is None:
                return torch.tensor([], device=embeddings.device)
            return (embeddings[a] * embeddings[b]).sum(dim=1)

        return {"pos_score": score(batch.pos_src, batch.pos_dst), "neg_score": score(batch.neg_src, batch.neg_dst)}


class NodeRegressHead(nn.Module):
    def __init__(self, embedding_dim: int, output_dim: int = 1):
        super().__init__()
        self.embedding_dim = embedding_dim
        self.output_dim = output_dim
        self.mlp = nn.Linear(embedding_dim, output_dim)

    def forward(self, embeddings: Tensor, batch: BatchData) -> dict[str, Tensor]:
        x = embeddings[batch.target_nodes] if batch.target_nodes is not None else embeddings
        return {"node_pred": self.mlp(x)}


class NodeClassifyHead(nn.Module):
    def __init__(self, embedding_dim: int, num_classes: int):
        super().__init__()
        self.embedding_dim = embedding_dim
        self.num_classes = num_classes
        self.mlp = nn.Linear(embedding_dim, num_classes)

    def forward(self, embeddings: Tensor, batch: BatchData) -> dict[str, Tensor]:
        x = embeddings[batch.target_nodes] if batch.target_nodes is not None else embeddings
        return {"logits": self.mlp(x)}
