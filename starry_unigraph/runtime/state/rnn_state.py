"""Per-node recurrent state for DTDG models across snapshots (reference
runtime/state/rnn_state.py:26, a stub there): states are dense [N, H] tensors
padded / truncated to the current snapshot's node count."""
from __future__ import annotations

from typing import Any

from torch import Tensor

from starry_unigraph.backends.dtdg.runtime.state import RNNStateManager


class DTDGStateManager:
    def __init__(self, mode: str = "pad"):
        self.mode = mode
        self.state: Any = None
        self.steps = 0

    def prepare(self, node_ids: Tensor, timestamps: Tensor | None = None) -> dict[str, Any]:
        if self.state is None:
            return {"state": None}
        return {"state": RNNStateManager.state_padding(self.state, int(node_ids.numel()))}

    def patch(self, node_ids: Tensor, rows: Tensor) -> None:
        return None

    def update(self, model_output: dict[str, Any], chunk: Any) -> None:
        if "state" in model_output:
            self.state = RNNStateManager.state_detach(model_output["state"])

    def step(self) -> None:
        self.steps += 1

    def reset(self) -> None:
        self.state = None
        self.steps = 0

    def describe(self) -> dict[str, Any]:
        return {"manager": "dtdg_rnn", "mode": self.mode, "steps": self.steps, "has_state": self.state is not None}
