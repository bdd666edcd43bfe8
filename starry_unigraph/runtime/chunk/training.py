"""Chunk-mode training steps (reference runtime/chunk/training.py:19-96)."""
from __future__ import annotations

from typing import Any


def run_chunk_train_step(loader: Any, runtime: Any, batch: Any) -> dict[str, Any]:
    return loader.run_train_step(runtime, batch)


def run_chunk_eval_step(loader: Any, runtime: Any, batch: Any) -> dict[str, Any]:
    return loader.run_eval_step(runtime, batch)
