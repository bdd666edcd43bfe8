"""Temporal attention layer shared by the CTDG models
(reference runtime/modules/temporal_conv.py:24-148)."""
from starry_unigraph.backends.ctdg.runtime.models import TemporalTransformerConv

__all__ = ["TemporalTransformerConv"]
