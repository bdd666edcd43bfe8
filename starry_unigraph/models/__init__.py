"""Task-agnostic model protocol, task heads and the backbone+head wrapper.

The CTDG (TGN-family) and DTDG (Flare) model implementations live with their
runtimes in ``starry_unigraph.backends.{ctdg,dtdg}.runtime.models``; reusable
layers are in ``starry_unigraph.runtime.modules``.
"""
from .base import TemporalModel
from .task_head import EdgePredictHead, NodeClassifyHead, NodeRegressHead
from .wrapped import WrappedModel

__all__ = ["TemporalModel", "EdgePredictHead", "NodeRegressHead", "NodeClassifyHead", "WrappedModel"]
