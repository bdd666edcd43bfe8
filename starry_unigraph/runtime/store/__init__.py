"""Node-state stores of the unified runtime (reference runtime/store/): a plain
per-node memory bank with a K-slot mailbox (``MemoryBank``), a dense state view
over it (``MemoryState``), the DTDG window-state manager (``RNNState``) and the
feature-store protocol (``FeatureStore``)."""
from starry_unigraph.runtime.store.MemoryState import MemoryBank, MemoryState
from starry_unigraph.runtime.store.RNNState import RNNState, STGraphBlob
from starry_unigraph.runtime.store.feature import FeatureStore, TensorFeatureStore

__all__ = ["MemoryBank", "MemoryState", "RNNState", "STGraphBlob", "FeatureStore", "TensorFeatureStore"]
