"""Stable library surface (reference lib_stable.py:1-130): every name here keeps
its signature across patch versions."""
from __future__ import annotations

from starry_unigraph.data.batch_data import BatchData
from starry_unigraph.data.chunk_atomic import ChunkAtomic
from starry_unigraph.data.partition import PartitionData, RouteData, TensorData
from starry_unigraph.data.raw_temporal import NodeTemporalFeatureTable, RawTemporalEvents
from starry_unigraph.data.sample_config import SampleConfig
from starry_unigraph.models.base import TemporalModel
from starry_unigraph.models.task_head import EdgePredictHead, NodeClassifyHead, NodeRegressHead
from starry_unigraph.models.wrapped import WrappedModel
from starry_unigraph.registry.task_adapter import TaskAdapter
from starry_unigraph.registry.task_registry import TaskRegistry
from starry_unigraph.runtime.backend import GraphBackend, StateManager
from starry_unigraph.runtime.engine import PipelineEngine
from starry_unigraph.runtime.modules import GCNStack, MatGRUCell, TimeEncode, _LSTMCell
from starry_unigraph.session import SchedulerSession

__version__ = "0.2.0"
__stability__ = "stable"

__all__ = [
    "__version__", "__stability__", "BatchData", "SampleConfig", "PartitionData", "RouteData", "TensorData",
    "ChunkAtomic", "NodeTemporalFeatureTable", "RawTemporalEvents", "GraphBackend", "StateManager", "TaskAdapter",
    "TemporalModel", "WrappedModel", "EdgePredictHead", "NodeRegressHead", "NodeClassifyHead", "TimeEncode",
    "GCNStack", "MatGRUCell", "_LSTMCell", "SchedulerSession", "PipelineEngine", "TaskRegistry",
]


def get_stability_info() -> str:
    return (f"starry_unigraph library API v{__version__} ({__stability__}).\n"
            "Stable: data structures, protocols, PipelineEngine / SchedulerSession, task heads, reusable modules.\n"
            "Internal: backend implementations, kernels, command-line tools.")


if __name__ == "__main__":
    print(get_stability_info())
