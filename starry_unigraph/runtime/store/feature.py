"""Feature stores (the reference's runtime/store/feature.py is empty): the
feature-store protocol and its tensor-backed implementation."""
from starry_unigraph.data.feature_store import FeatureStore, TensorFeatureStore

__all__ = ["FeatureStore", "TensorFeatureStore"]
