from .base import BaseTaskAdapter
from .node_classify import NodeClassifyAdapter
from .node_regression import NodeRegressAdapter, NodeRegressionTaskAdapter
from .temporal_link_prediction import EdgePredictAdapter, TemporalLinkPredictionTaskAdapter

__all__ = [
    "BaseTaskAdapter",
    "EdgePredictAdapter",
    "TemporalLinkPredictionTaskAdapter",
    "NodeRegressionTaskAdapter",
    "NodeRegressAdapter",
    "NodeClassifyAdapter",
]
