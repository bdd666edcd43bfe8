from .base import (
    ArtifactLayout,
    ArtifactOutput,
    ArtifactPayload,
    GraphPreprocessor,
    load_prepared_from_disk,
    read_artifact_meta,
)

__all__ = ["ArtifactLayout", "ArtifactOutput", "ArtifactPayload", "GraphPreprocessor", "load_prepared_from_disk",
           "read_artifact_meta"]
