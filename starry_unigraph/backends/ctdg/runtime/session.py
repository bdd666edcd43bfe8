"""Thin CTDG session (reference backends/ctdg/runtime/session.py:16-93)."""
from __future__ import annotations

from pathlib import Path
from typing import Any

import torch

from starry_unigraph.types import PreparedArtifacts, RuntimeBundle, SessionContext

from .factory import build_ctdg_runtime
from .runtime import CTDGOnlineRuntime


class CTDGSession:
    def __init__(self) -> None:
        self.online_runtime: CTDGOnlineRuntime | None = None
        self.prepared: PreparedArtifacts | None = None
        self._runtime = RuntimeBundle()

    def prepare_data(self, session_ctx: SessionContext) -> PreparedArtifacts:
        from starry_unigraph.backends.ctdg.preprocess import CTDGPreprocessor

        self.prepared = CTDGPreprocessor().run(session_ctx)
        session_ctx.prepared_artifacts = self.prepared
        return self.prepared

    def build_runtime(self, session_ctx: SessionContext) -> None:
        if self.prepared is not None:
            session_ctx.prepared_artifacts = self.prepared
        self.online_runtime, self._runtime = build_ctdg_runtime(session_ctx)

    def _bs(self, ctx: SessionContext) -> int:
        return int(ctx.config["train"]["batch_size"])

    def iter_train(self, ctx: SessionContext):
        yield from self.online_runtime.iter_batches("train", self._bs(ctx))

    def iter_eval(self, ctx: SessionContext, split: str = "val"):
        yield from self.online_runtime.iter_batches(split, self._bs(ctx))

    def iter_predict(self, ctx: SessionContext, split: str = "test"):
        yield from self.online_runtime.iter_batches(split, self._bs(ctx))

    def train_batches(self, batches: list[Any]) -> list[dict[str, Any]]:
        """Train on a list of batches (pinned host tensors): asynchronous per-step
        host -> device inputs and device -> host loss/metrics, one synchronisation at
        the end (CUDA engine); the per-step path elsewhere."""
        rt = self.online_runtime
        if rt.engine is not None:
            return rt.run_batches_device(list(batches), "train", True)
        return [self.train_step(b) for b in batches]

    def train_step(self, batch: Any) -> dict[str, Any]:
        return self.online_runtime.train_step(batch)

    def eval_step(self, batch: Any) -> dict[str, Any]:
        return self.online_runtime.eval_step(batch, split=batch.split)

    def predict_step(self, batch: Any) -> dict[str, Any]:
        return self.online_runtime.predict_step(batch)

    def save_checkpoint(self, path: str | Path, extra: dict[str, Any] | None = None) -> None:
        rt = self.online_runtime
        model = rt.model.module if hasattr(rt.model, "module") else rt.model
        ckpt: dict[str, Any] = {"model": {k: v.detach().cpu() for k, v in model.state_dict().items()}}
        if rt.memory_updater is not None:
            ckpt["memory_updater"] = {k: v.detach().cpu() for k, v in rt.memory_updater.state_dict().items()}
        if extra:
            ckpt.update(extra)
        torch.save(ckpt, str(path))

    def load_checkpoint(self, path: str | Path) -> dict[str, Any]:
        rt = self.online_runtime
        ckpt = torch.load(str(path), map_location="cpu", weights_only=False)
        model = rt.model.module if hasattr(rt.model, "module") else rt.model
        with torch.no_grad():
            for k, v in model.state_dict().items():  # copy in place: parameters may be views of a flat buffer
                v.copy_(ckpt["model"][k])
            if rt.memory_updater is not None and "memory_updater" in ckpt:
                for k, v in rt.memory_updater.state_dict().items():
                    v.copy_(ckpt["memory_updater"][k])
            if "memory_bank" in ckpt:
                mb = ckpt["memory_bank"]
                for name in ("memory", "memory_ts", "mailbox", "mailbox_ts", "next_mail_pos"):
                    getattr(rt.memory, name).copy_(mb[name])
        return ckpt
