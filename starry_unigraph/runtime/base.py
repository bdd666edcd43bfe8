"""Runtime protocol shared by the online and snapshot runtimes (reference runtime/base.py:13-30)."""
from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any, Iterable


class RuntimeProtocol(ABC):
    @abstractmethod
    def iter_batches(self, split: str, **kwargs: Any) -> Iterable[Any]: ...

    @abstractmethod
    def step(self, batch: Any, training: bool) -> dict[str, Any]: ...

    @abstractmethod
    def state_dict(self) -> dict[str, Any]: ...

    @abstractmethod
    def load_state_dict(self, state: dict[str, Any]) -> None: ...
