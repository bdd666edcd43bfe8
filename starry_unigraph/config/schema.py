"""YAML configuration: load, deep-merge, validate, infer the graph mode.

Schema and merge semantics follow the reference (config/schema.py:12-150):
``default.yaml`` <- user file <- overrides; required paths are checked; the
graph mode is inferred from ``model.family`` when ``data.graph_mode`` is null;
fields that only matter for the other graph mode produce warnings.
"""
from __future__ import annotations

from copy import deepcopy
from pathlib import Path
from typing import Any

import yaml

DEFAULT_CONFIG_PATH = Path(__file__).with_name("default.yaml")

MODEL_GRAPH_MODES: dict[str, str] = {
    "tgn": "ctdg",
    "dyrep": "ctdg",
    "jodie": "ctdg",
    "tgat": "ctdg",
    "apan": "ctdg",
    "evolvegcn": "dtdg",
    "tgcn": "dtdg",
    "mpnn_lstm": "dtdg",
    "gcn": "dtdg",
}

REQUIRED_PATHS = (
    "model.name",
    "model.family",
    "model.task",
    "data.root",
    "data.name",
    "train.epochs",
    "train.batch_size",
    "runtime.backend",
    "runtime.device",
)

CTDG_ACTIVE_PREFIXES = ("sampling.", "model.memory.", "runtime.state_sync", "ctdg.")
DTDG_ACTIVE_PREFIXES = ("train.snaps", "graph.storage", "model.window.size", "runtime.cache", "dtdg.")


class ConfigError(ValueError):
    """Raised for a missing required path or an unknown graph mode."""


def load_default_config() -> dict[str, Any]:
    with DEFAULT_CONFIG_PATH.open("r", encoding="utf-8") as handle:
        return yaml.safe_load(handle)


def _deep_merge(base: dict[str, Any], override: dict[str, Any]) -> dict[str, Any]:
    merged = deepcopy(base)
    for key, value in override.items():
        if isinstance(value, dict) and isinstance(merged.get(key), dict):
            merged[key] = _deep_merge(merged[key], value)
        else:
            merged[key] = deepcopy(value)
    return merged


def merge_config(config: dict[str, Any], overrides: dict[str, Any] | None) -> dict[str, Any]:
    return _deep_merge(config, overrides or {})


def load_config(config_or_path: str | Path | dict[str, Any], overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    """Load a config dict or YAML path and merge it over the defaults."""
    if isinstance(config_or_path, dict):
        config = deepcopy(config_or_path)
    else:
        with Path(config_or_path).open("r", encoding="utf-8") as handle:
            config = yaml.safe_load(handle) or {}
    return merge_config(load_default_config(), merge_config(config, overrides))


def get_by_path(config: dict[str, Any], path: str) -> Any:
    cur: Any = config
    for part in path.split("."):
        if not isinstance(cur, dict) or part not in cur:
            raise ConfigError(f"Missing required config path: {path}")
        cur = cur[part]
    return cur


def set_by_path(config: dict[str, Any], path: str, value: Any) -> None:
    cur = config
    parts = path.split(".")
    for part in parts[:-1]:
        cur = cur.setdefault(part, {})
    cur[parts[-1]] = value


def detect_graph_mode(config: dict[str, Any]) -> str:
    explicit = config.get("data", {}).get("graph_mode")
    if explicit:
        return str(explicit)
    family = str(get_by_path(config, "model.family")).lower()
    if family in MODEL_GRAPH_MODES:
        mode = MODEL_GRAPH_MODES[family]
        set_by_path(config, "data.graph_mode", mode)
        return mode
    raise ConfigError(f"Unable to infer graph mode for model.family={family!r}")


def _flatten(config: dict[str, Any], prefix: str = "") -> dict[str, Any]:
    flat: dict[str, Any] = {}
    for key, value in config.items():
        path = f"{prefix}.{key}" if prefix else key
        if isinstance(value, dict):
            flat.update(_flatten(value, path))
        else:
            flat[path] = value
    return flat


def _warn_inactive(config: dict[str, Any], active: tuple[str, ...], inactive: tuple[str, ...]) -> list[str]:
    warnings: list[str] = []
    for path, value in _flatten(config).items():
        if value is None:
            continue
        if any(path.startswith(p) for p in inactive) and not any(path.startswith(p) for p in active):
            warnings.append(f"Inactive config field for selected graph mode: {path}")
    return warnings


def validate_config(config: dict[str, Any]) -> list[str]:
    """Check required paths; return warnings (never raises for inactive fields)."""
    for path in REQUIRED_PATHS:
        get_by_path(config, path)
    mode = detect_graph_mode(config)
    storage = config.get("graph", {}).get("storage")
    warnings: list[str] = []
    if mode == "dtdg" and storage != "snapshots":
        warnings.append("DTDG mode usually expects graph.storage=snapshots; continuing with configured value.")
    if mode == "ctdg" and storage == "snapshots":
        warnings.append("CTDG mode received graph.storage=snapshots; sampling pipeline will ignore snapshot storage.")
    # default.yaml carries both ctdg.* and dtdg.* sections; only user-set deviations are interesting,
    # so compare against the defaults before warning.
    defaults = _flatten(load_default_config())
    user_flat = {k: v for k, v in _flatten(config).items() if defaults.get(k, object()) != v}
    active = CTDG_ACTIVE_PREFIXES if mode == "ctdg" else DTDG_ACTIVE_PREFIXES
    inactive = DTDG_ACTIVE_PREFIXES if mode == "ctdg" else CTDG_ACTIVE_PREFIXES
    warnings.extend(_warn_inactive(_unflatten(user_flat), active, inactive))
    return warnings


def _unflatten(flat: dict[str, Any]) -> dict[str, Any]:
    out: dict[str, Any] = {}
    for path, value in flat.items():
        set_by_path(out, path, value)
    return out
