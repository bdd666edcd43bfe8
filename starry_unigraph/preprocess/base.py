"""Preprocessors that turn a raw dataset into the artifact tree a runtime loads
(reference interface: preprocess/base.py:13-89).

Artifact tree under ``<artifact_root>``: ``meta/artifacts.json`` (the provider
meta, read back by ``load_prepared_from_disk``) and one directory per artifact
family (``partitions``, ``routes``, ``sampling``, ``snapshots``, plus ``flare``
and ``clusters`` written by some modes). Every file is written to a temporary
name and renamed into place, so an interrupted preprocessing run never leaves a
truncated artifact that a later run would load.
"""
from __future__ import annotations

import json
import os
from abc import ABC, abstractmethod
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable

import torch

from starry_unigraph.types import PreparedArtifacts, SessionContext

KNOWN_ARTIFACT_DIRS = ("meta", "partitions", "routes", "sampling", "snapshots", "flare", "clusters")
META_FILE = ("meta", "artifacts.json")


def _dump_json(payload: Any, handle) -> None:
    handle.write(json.dumps(payload, indent=2, sort_keys=True, default=str).encode("utf-8"))


def _dump_torch(payload: Any, handle) -> None:
    torch.save(payload, handle)


# serializer name -> writer(payload, binary file handle)
SERIALIZERS: dict[str, Callable[[Any, Any], None]] = {"json": _dump_json, "torch": _dump_torch}


def write_artifact(path: Path, payload: Any, serializer: str = "json") -> Path:
    """Write one artifact atomically (temporary file in the same directory, then rename)."""
    writer = SERIALIZERS.get(serializer)
    if writer is None:
        raise ValueError(f"Unsupported artifact serializer: {serializer} (known: {sorted(SERIALIZERS)})")
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    staging = path.with_name(f".{path.name}.{os.getpid()}.partial")
    with staging.open("wb") as handle:
        writer(payload, handle)
    os.replace(staging, path)
    return path


@dataclass
class ArtifactLayout:
    root: Path
    directories: dict[str, Path]

    @property
    def meta_path(self) -> Path:
        return self.directories[META_FILE[0]] / META_FILE[1]


@dataclass
class ArtifactOutput:
    relative_path: str
    payload: Any
    serializer: str = "json"


@dataclass
class ArtifactPayload:
    provider_meta: dict[str, Any]
    outputs: list[ArtifactOutput]


class GraphPreprocessor(ABC):
    """Three stages run in order by ``run``: read the raw data, partition it, and
    build the runtime artifacts (the last stage usually ends in ``emit_artifacts``)."""

    artifact_dirs: tuple[str, ...] = ("meta", "partitions", "routes", "sampling", "snapshots")

    @abstractmethod
    def prepare_raw(self, session_ctx: SessionContext) -> None: ...

    @abstractmethod
    def build_partitions(self, session_ctx: SessionContext) -> None: ...

    @abstractmethod
    def build_runtime_artifacts(self, session_ctx: SessionContext) -> PreparedArtifacts: ...

    def run(self, session_ctx: SessionContext) -> PreparedArtifacts:
        stages = (self.prepare_raw, self.build_partitions)
        for stage in stages:
            stage(session_ctx)
        return self.build_runtime_artifacts(session_ctx)

    def ensure_artifact_layout(self, session_ctx: SessionContext) -> ArtifactLayout:
        root = Path(session_ctx.artifact_root)
        layout = ArtifactLayout(root=root, directories={d: root / d for d in self.artifact_dirs})
        for directory in layout.directories.values():
            directory.mkdir(parents=True, exist_ok=True)
        return layout

    def emit_artifacts(self, session_ctx: SessionContext, payload: ArtifactPayload) -> PreparedArtifacts:
        """Write every output, then the provider meta last: a tree whose meta exists is complete."""
        layout = self.ensure_artifact_layout(session_ctx)
        for output in payload.outputs:
            write_artifact(layout.root / output.relative_path, output.payload, output.serializer)
        write_artifact(layout.meta_path, payload.provider_meta, "json")
        return PreparedArtifacts(meta_path=layout.meta_path, directories=layout.directories,
                                 provider_meta=payload.provider_meta)


def read_artifact_meta(meta_path: Path) -> dict[str, Any]:
    return json.loads(Path(meta_path).read_text(encoding="utf-8"))


def load_prepared_from_disk(artifact_root: Path) -> PreparedArtifacts:
    root = Path(artifact_root)
    meta_path = root.joinpath(*META_FILE)
    if not meta_path.is_file():
        raise RuntimeError("Data not prepared. Call prepare_data() first.")
    present = {name: root / name for name in KNOWN_ARTIFACT_DIRS if (root / name).is_dir()}
    return PreparedArtifacts(meta_path=meta_path, directories=present, provider_meta=read_artifact_meta(meta_path))
