"""Runner protocol (reference runtime/runner/base.py:35): build_sequence ->
prepare_data -> sync_data -> compute -> post_compute for each unit of work."""
from __future__ import annotations

from typing import Any, Iterable, Protocol


class Runner(Protocol):
    def build_sequence(self, split: str) -> Iterable[Any]: ...

    def prepare_data(self, unit: Any) -> Any: ...

    def sync_data(self, prepared: Any) -> Any: ...

    def compute(self, synced: Any, training: bool) -> dict[str, Any]: ...

    def post_compute(self, result: dict[str, Any]) -> None: ...


def run_units(runner: Runner, split: str, training: bool) -> list[dict[str, Any]]:
    out = []
    for unit in runner.build_sequence(split):
        res = runner.compute(runner.sync_data(runner.prepare_data(unit)), training)
        runner.post_compute(res)
        out.append(res)
    return out
