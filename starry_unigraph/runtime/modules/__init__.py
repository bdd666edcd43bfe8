"""Reusable layers (reference runtime/modules/__init__.py:15-27)."""
from .gcn_layers import GCNStack
from .rnn_cells import MatGRUCell, _LSTMCell
from .time_encode import TimeEncode


def __getattr__(name):
    if name == "TemporalTransformerConv":
        from .temporal_conv import TemporalTransformerConv

        return TemporalTransformerConv
    raise AttributeError(name)


__all__ = ["TimeEncode", "GCNStack", "MatGRUCell", "_LSTMCell", "TemporalTransformerConv"]
