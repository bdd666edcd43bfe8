from .batch_data import BatchData
from .chunk_atomic import ChunkAtomic, RemoteManifest, SpatialDeps, StateDeps
from .chunk_builder import ChunkBuilder
from .feature_store import FeatureStore, TensorFeatureStore
from .raw_temporal import (
    NodeTemporalFeatureTable,
    RawTemporalEvents,
    build_snapshot_dataset_from_events,
    load_raw_temporal_events,
)
from .sample_config import SampleConfig


def __getattr__(name):
    if name in ("PartitionData", "RouteData", "TensorData", "SnapshotBlock"):
        from . import partition

        return getattr(partition, name)
    raise AttributeError(name)


__all__ = ["BatchData", "SampleConfig", "NodeTemporalFeatureTable", "RawTemporalEvents",
           "build_snapshot_dataset_from_events", "load_raw_temporal_events", "ChunkAtomic", "RemoteManifest",
           "SpatialDeps", "StateDeps", "ChunkBuilder", "FeatureStore", "TensorFeatureStore", "PartitionData",
           "RouteData", "TensorData", "SnapshotBlock"]
