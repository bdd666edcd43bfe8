from .batch_data import BatchData
from .raw_temporal import (
    NodeTemporalFeatureTable,
    RawTemporalEvents,
    build_snapshot_dataset_from_events,
    load_raw_temporal_events,
)
from .sample_config import SampleConfig

__all__ = ["BatchData", "SampleConfig", "NodeTemporalFeatureTable", "RawTemporalEvents",
           "build_snapshot_dataset_from_events", "load_raw_temporal_events"]
