"""Edge / temporal link prediction task (reference tasks/temporal_link_prediction.py:15-153).

Loss: BCE with logits over positive (label 1) and negative (label 0) scores.
Metrics: pairwise AUC (fraction of (pos, neg) pairs with pos > neg, ties 1/2)
and average precision with scikit-learn semantics (the reference's adapter uses a
mean-difference stand-in for AP; the online runtime uses the real AP, which is
what is computed here).
"""
from __future__ import annotations

from typing import Any

import torch
import torch.nn.functional as F

from starry_unigraph.data.batch_data import BatchData
from starry_unigraph.data.sample_config import SampleConfig

from .base import BaseTaskAdapter


def average_precision(scores: torch.Tensor, labels: torch.Tensor) -> float:
    """AP = sum over thresholds of (R_k - R_{k-1}) P_k (scikit-learn definition)."""
    scores = scores.detach().float().cpu()
    labels = labels.detach().float().cpu()
    npos = float(labels.sum())
    if npos <= 0:
        return 0.0
    ge = scores.unsqueeze(0) >= scores.unsqueeze(1)  # [i, j]: s_j >= s_i
    pos_ge = (ge & (labels.unsqueeze(0) > 0)).sum(1).float()
    all_ge = ge.sum(1).float()
    prec = pos_ge / all_ge
    return float((prec * labels).sum() / npos)


def pairwise_auc(pos: torch.Tensor, neg: torch.Tensor) -> float:
    pos = pos.detach().float().flatten().cpu()
    neg = neg.detach().float().flatten().cpu()
    if pos.numel() == 0 or neg.numel() == 0:
        return 0.0
    gt = (pos[:, None] > neg[None, :]).float()
    eq = (pos[:, None] == neg[None, :]).float()
    return float((gt + 0.5 * eq).mean())


class EdgePredictAdapter(BaseTaskAdapter):
    task_name = "edge_predict"

    def __init__(self, neg_ratio: int = 1) -> None:
        self.neg_ratio = int(neg_ratio)

    def build_sample_config(self, chunk: Any, sample_params: dict[str, Any]) -> SampleConfig:
        cfg = super().build_sample_config(chunk, sample_params)
        cfg.pos_src = getattr(chunk, "pos_src", None)
        cfg.pos_dst = getattr(chunk, "pos_dst", None)
        cfg.neg_strategy = str(sample_params.get("neg_strategy", "random"))
        cfg.neg_ratio = self.neg_ratio
        return cfg

    def compute_loss(self, model_output: dict[str, Any], batch: BatchData | None = None) -> Any:
        if "loss" in model_output and "pos_score" not in model_output:
            return float(model_output["loss"])
        pos, neg = model_output.get("pos_score"), model_output.get("neg_score")
        if pos is None or neg is None:
            return torch.tensor(0.0)
        scores = torch.cat([pos.flatten(), neg.flatten()])
        labels = torch.cat([torch.ones_like(pos.flatten()), torch.zeros_like(neg.flatten())])
        return F.binary_cross_entropy_with_logits(scores, labels)

    def compute_metrics(self, model_output: dict[str, Any], batch: BatchData | None = None) -> dict[str, float]:
        pos, neg = model_output.get("pos_score"), model_output.get("neg_score")
        if pos is None or neg is None:
            return super().compute_metrics(model_output, batch)
        scores = torch.cat([pos.flatten(), neg.flatten()]).sigmoid()
        labels = torch.cat([torch.ones_like(pos.flatten()), torch.zeros_like(neg.flatten())])
        return {"auc": pairwise_auc(pos, neg), "ap": average_precision(scores, labels)}

    def format_output(self, model_output: dict[str, Any], batch: BatchData | None = None) -> dict[str, Any]:
        def cpu(t):
            return None if t is None else t.detach().cpu()

        return {
            "pos_score": cpu(model_output.get("pos_score")),
            "neg_score": cpu(model_output.get("neg_score")),
            "pos_src": cpu(batch.pos_src) if batch is not None else None,
            "pos_dst": cpu(batch.pos_dst) if batch is not None else None,
        }


TemporalLinkPredictionTaskAdapter = EdgePredictAdapter
