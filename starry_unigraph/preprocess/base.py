"""Artifact-emitting preprocessor base (reference preprocess/base.py:13-89).

Layout under ``<artifact_root>``: ``meta/artifacts.json`` (provider meta) plus
mode-specific directories; JSON payloads are pretty-printed with sorted keys,
tensor payloads use ``torch.save``.
"""
from __future__ import annotations

import json
from abc import ABC, abstractmethod
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

from starry_unigraph.types import PreparedArtifacts, SessionContext


@dataclass
class ArtifactLayout:
    root: Path
    directories: dict[str, Path]

    @property
    def meta_path(self) -> Path:
        return self.directories["meta"] / "artifacts.json"


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
    artifact_dirs: tuple[str, ...] = ("meta", "partitions", "routes", "sampling", "snapshots")

    @abstractmethod
    def prepare_raw(self, session_ctx: SessionContext) -> None: ...

    @abstractmethod
    def build_partitions(self, session_ctx: SessionContext) -> None: ...

    @abstractmethod
    def build_runtime_artifacts(self, session_ctx: SessionContext) -> PreparedArtifacts: ...

    def ensure_artifact_layout(self, session_ctx: SessionContext) -> ArtifactLayout:
        dirs = {name: session_ctx.artifact_root / name for name in self.artifact_dirs}
        for p in dirs.values():
            p.mkdir(parents=True, exist_ok=True)
        return ArtifactLayout(root=session_ctx.artifact_root, directories=dirs)

    def emit_artifacts(self, session_ctx: SessionContext, payload: ArtifactPayload) -> PreparedArtifacts:
        layout = self.ensure_artifact_layout(session_ctx)
        self._write_json(layout.meta_path, payload.provider_meta)
        for out in payload.outputs:
            self._write_output(layout.root / out.relative_path, out.payload, out.serializer)
        return PreparedArtifacts(meta_path=layout.meta_path, directories=layout.directories,
                                 provider_meta=payload.provider_meta)

    def run(self, session_ctx: SessionContext) -> PreparedArtifacts:
        self.prepare_raw(session_ctx)
        self.build_partitions(session_ctx)
        return self.build_runtime_artifacts(session_ctx)

    @staticmethod
    def _write_json(path: Path, payload: dict[str, Any]) -> None:
        path.parent.mkdir(parents=True, exist_ok=True)
        with path.open("w", encoding="utf-8") as handle:
            json.dump(payload, handle, indent=2, sort_keys=True, default=str)

    @classmethod
    def _write_output(cls, path: Path, payload: Any, serializer: str) -> None:
        path.parent.mkdir(parents=True, exist_ok=True)
        if serializer == "json":
            cls._write_json(path, payload)
        elif serializer == "torch":
            torch.save(payload, path)
        else:
            raise ValueError(f"Unsupported artifact serializer: {serializer}")


def read_artifact_meta(meta_path: Path) -> dict[str, Any]:
    with Path(meta_path).open("r", encoding="utf-8") as handle:
        return json.load(handle)


KNOWN_ARTIFACT_DIRS = ("meta", "partitions", "routes", "sampling", "snapshots", "flare", "clusters")


def load_prepared_from_disk(artifact_root: Path) -> PreparedArtifacts:
    meta_path = Path(artifact_root) / "meta" / "artifacts.json"
    if not meta_path.exists():
        raise RuntimeError("Data not prepared. Call prepare_data() first.")
    dirs = {n: Path(artifact_root) / n for n in KNOWN_ARTIFACT_DIRS if (Path(artifact_root) / n).exists()}
    return PreparedArtifacts(meta_path=meta_path, directories=dirs, provider_meta=read_artifact_meta(meta_path))
