from .base import StateManagerBase
from .memory_state import CTDGStateManager
from .rnn_state import DTDGStateManager

__all__ = ["StateManagerBase", "CTDGStateManager", "DTDGStateManager"]
