from .loader import STGraphLoader
from .models import (MODEL_SPECS, FlareEvolveGCN, FlareModelSpec, FlareMPNNLSTM, FlareTGCN, build_flare_model,
                     extract_graph_labels)
from .route import Route, RouteExchange, set_route_transport
from .session_loader import DTDGBatch, DTDGWindowState, FlareRuntimeLoader, SnapshotRoutePlan
from .state import RNNStateManager, STGraphBlob, STWindowState
from .training import (FlareOptimizer, init_flare_training, run_flare_eval_step, run_flare_predict_step,
                       run_flare_train_step)

__all__ = ["STGraphLoader", "MODEL_SPECS", "FlareEvolveGCN", "FlareModelSpec", "FlareMPNNLSTM", "FlareTGCN",
           "build_flare_model", "extract_graph_labels", "Route", "RouteExchange", "set_route_transport", "DTDGBatch",
           "DTDGWindowState", "FlareRuntimeLoader", "SnapshotRoutePlan", "RNNStateManager", "STGraphBlob",
           "STWindowState", "FlareOptimizer", "init_flare_training", "run_flare_eval_step", "run_flare_predict_step",
           "run_flare_train_step"]
