"""Task registry (reference registry/task_registry.py:11-35)."""
from __future__ import annotations

from starry_unigraph.tasks import (
    EdgePredictAdapter,
    NodeClassifyAdapter,
    NodeRegressionTaskAdapter,
    TemporalLinkPredictionTaskAdapter,
)


class TaskRegistry:
    _tasks: dict[str, type] = {
        "temporal_link_prediction": TemporalLinkPredictionTaskAdapter,
        "edge_predict": EdgePredictAdapter,
        "snapshot_node_regression": NodeRegressionTaskAdapter,
        "node_regression": NodeRegressionTaskAdapter,
        "node_classification": NodeClassifyAdapter,
    }

    @classmethod
    def resolve(cls, task_type: str) -> type:
        if task_type not in cls._tasks:
            raise KeyError(f"Unknown task type: {task_type!r}")
        return cls._tasks[task_type]

    @classmethod
    def list_tasks(cls) -> list[str]:
        return list(cls._tasks.keys())
