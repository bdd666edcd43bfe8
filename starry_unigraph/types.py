"""Core dataclasses shared by every layer (reference: types.py:9-84)."""
from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path
from typing import Any


@dataclass
class DistributedContext:
    backend: str
    world_size: int = 1
    rank: int = 0
    local_rank: int = 0
    local_world_size: int = 1
    master_addr: str = "127.0.0.1"
    master_port: int = 29500
    init_method: str = "env://"
    launcher: str = "single_process"
    initialized: bool = False
    timeout_s: float = 600.0

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1


@dataclass
class PredictionResult:
    predictions: list[Any]
    targets: list[Any] | None = None
    meta: dict[str, Any] = field(default_factory=dict)


@dataclass
class SessionContext:
    config: dict[str, Any]
    project_root: Path
    dataset_path: Path | None
    artifact_root: Path
    dist: DistributedContext
    warnings: list[str] = field(default_factory=list)
    provider_state: dict[str, Any] = field(default_factory=dict)
    prepared_artifacts: "PreparedArtifacts | None" = None


@dataclass
class RuntimeBundle:
    model: Any = None
    optimizer: Any = None
    scheduler: Any = None
    state: dict[str, Any] = field(default_factory=dict)


@dataclass
class PreparedArtifacts:
    """Handle on ``<artifact_root>``: ``meta/artifacts.json`` plus the existing
    sub-directories (meta, partitions, routes, sampling, snapshots, flare, clusters).

    ``provider_meta`` carries ``graph_mode``, ``artifact_version`` and ``num_parts``
    for every mode, plus mode-specific fields written by the preprocessors.
    """

    meta_path: Path
    directories: dict[str, Path]
    provider_meta: dict[str, Any]
