"""Runner over the CTDG online runtime (reference runtime/runner/ctdg_runner.py, a stub)."""
from __future__ import annotations

from typing import Any, Iterable


class CTDGRunner:
    def __init__(self, online_runtime: Any, batch_size: int):
        self.rt = online_runtime
        self.batch_size = batch_size
        self.history: list[float] = []

    def build_sequence(self, split: str) -> Iterable[Any]:
        return self.rt.iter_batches(split, self.batch_size)

    def prepare_data(self, unit: Any) -> Any:
        return unit

    def sync_data(self, prepared: Any) -> Any:
        self.rt.memory.wait_pending_syncs()
        return prepared

    def compute(self, synced: Any, training: bool) -> dict[str, Any]:
        return self.rt.train_step(synced) if training else self.rt.eval_step(synced, synced.split)

    def post_compute(self, result: dict[str, Any]) -> None:
        self.history.append(float(result.get("loss", 0.0)))
