"""DTDG window state (the reference's runtime/store/RNNState.py is empty): the
window-slot state manager of the Flare pipeline under its store-module name."""
from starry_unigraph.backends.dtdg.runtime.state import RNNStateManager as RNNState
from starry_unigraph.backends.dtdg.runtime.state import STGraphBlob

__all__ = ["RNNState", "STGraphBlob"]
