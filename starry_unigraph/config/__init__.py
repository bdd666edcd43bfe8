from .schema import (
    ConfigError,
    MODEL_GRAPH_MODES,
    REQUIRED_PATHS,
    detect_graph_mode,
    get_by_path,
    load_config,
    load_default_config,
    merge_config,
    set_by_path,
    validate_config,
)

__all__ = [
    "ConfigError",
    "MODEL_GRAPH_MODES",
    "REQUIRED_PATHS",
    "detect_graph_mode",
    "get_by_path",
    "load_config",
    "load_default_config",
    "merge_config",
    "set_by_path",
    "validate_config",
]
