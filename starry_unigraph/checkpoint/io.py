"""Checkpoint IO (reference checkpoint/io.py:9-20: pickle of a payload dict).

Payloads are written with ``pickle.dump``, the reference's format, so the
reference's ``load_checkpoint`` (``pickle.load``) reads them; tensors pickle
through torch's own reduction. Files written by ``torch.save`` (earlier
builds of this framework, the CTDG checkpoint) also load.
"""
from __future__ import annotations

import pickle
import zipfile
from pathlib import Path
from typing import Any

import torch


def save_checkpoint(path: str | Path, payload: dict[str, Any]) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    with tmp.open("wb") as handle:
        pickle.dump(payload, handle, protocol=pickle.HIGHEST_PROTOCOL)
    tmp.replace(path)
    return path


def load_checkpoint(path: str | Path) -> dict[str, Any]:
    path = Path(path)
    if zipfile.is_zipfile(path):  # torch.save container
        return torch.load(path, map_location="cpu", weights_only=False)
    with path.open("rb") as handle:
        return pickle.load(handle)
