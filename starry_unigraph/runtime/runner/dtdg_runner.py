"""Runner over the Flare DTDG loader (reference runtime/runner/dtdg_runner.py, a stub)."""
from __future__ import annotations

from typing import Any, Iterable


class DTDGRunner:
    def __init__(self, loader: Any, runtime_bundle: Any):
        self.loader = loader
        self.bundle = runtime_bundle
        self.history: list[float] = []

    def build_sequence(self, split: str) -> Iterable[Any]:
        return self.loader.iter_train() if split == "train" else self.loader.iter_eval(split)

    def prepare_data(self, unit: Any) -> Any:
        return unit

    def sync_data(self, prepared: Any) -> Any:
        return prepared

    def compute(self, synced: Any, training: bool) -> dict[str, Any]:
        if training:
            return self.loader.run_train_step(self.bundle, synced)
        return self.loader.run_eval_step(self.bundle, synced)

    def post_compute(self, result: dict[str, Any]) -> None:
        if "loss" in result:
            self.history.append(float(result["loss"]))
