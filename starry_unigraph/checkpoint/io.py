"""Checkpoint IO (reference checkpoint/io.py:9-20: pickle of a payload dict).

Payloads are written with ``torch.save`` (a pickle container that also stores
tensors efficiently) and read back with ``weights_only=False`` so both
state-dict payloads and the reference's live-object payloads load.
"""
from __future__ import annotations

import pickle
from pathlib import Path
from typing import Any

import torch


def save_checkpoint(path: str | Path, payload: dict[str, Any]) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(payload, tmp)
    tmp.replace(path)
    return path


def load_checkpoint(path: str | Path) -> dict[str, Any]:
    path = Path(path)
    try:
        return torch.load(path, map_location="cpu", weights_only=False)
    except Exception:
        with path.open("rb") as handle:
            return pickle.load(handle)
