"""Adaptive time split front-end (reference backends/chunk/prepare/time_split.py:5-27)."""
from __future__ import annotations

import torch


def adaptive_split(src: torch.Tensor, dst: torch.Tensor, ts: torch.Tensor, base_batch_size: int = 1000,
                   graph_feature: float = 0.5, **kw):
    from starry_unigraph.ops import native_ext

    nat = native_ext()
    if nat is None:
        raise RuntimeError("starry_unigraph._native is not built")
    return nat.adaptive_split(src.long(), dst.long(), ts.double(), int(base_batch_size), float(graph_feature), **kw)
