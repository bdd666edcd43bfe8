"""Unified pipeline engine: GraphBackend x TaskAdapter x StateManager x model
(reference runtime/engine.py:20-243). Unlike the reference it also takes the
optimiser step when one is given, so an epoch through this engine trains."""
from __future__ import annotations

from typing import Any, Iterator

import torch

from starry_unigraph.data.batch_data import BatchData


class PipelineEngine:
    def __init__(self, backend: Any, state_manager: Any, model: Any, task_adapter: Any, device: str = "cpu",
                 optimizer: Any = None, feature_store: Any = None, fetch_remote: Any = None):
        """`feature_store` (a ``FeatureStore`` of this rank's rows) makes every batch carry
        its neighbours' feature rows (``BatchData.nbr_feat``); `fetch_remote(manifest)`
        returns ``{"node_ids", "rows"}`` for the rows the manifest lists on other ranks."""
        self.feature_store = feature_store
        self.fetch_remote = fetch_remote
        self.backend = backend
        self.state_manager = state_manager
        self.model = model
        self.task_adapter = task_adapter
        self.device = device
        self.optimizer = optimizer

    def _materialize_batch(self, chunk: Any, sample_config: Any) -> BatchData:
        batch, manifest = chunk.materialize(sample_config)
        batch.source = chunk
        if self.feature_store is not None:
            remote = self.fetch_remote(manifest) if self.fetch_remote is not None and \
                manifest.remote_node_ids.numel() else None
            batch = chunk.complete(batch, remote, self.feature_store)
        return batch

    def iter_batches_with_step(self, split: str = "train", batch_size: int = 64) -> Iterator[tuple[BatchData, Any]]:
        for chunk in self.backend.iter_batches(split, batch_size):
            cfg = self.task_adapter.build_sample_config(chunk, {"num_neighbors": [10], "num_layers": 1})
            yield self._materialize_batch(chunk, cfg), chunk

    def run_epoch(self, split: str = "train", batch_size: int = 64) -> dict[str, Any]:
        is_train = split == "train"
        if hasattr(self.model, "train"):
            self.model.train(is_train)
        if hasattr(self.model, "current_split"):
            self.model.current_split = split
        outputs, losses, metric_acc = [], [], {}
        for batch, chunk in self.iter_batches_with_step(split, batch_size):
            state = self.state_manager.prepare(node_ids=batch.node_ids, timestamps=batch.timestamps)
            predict = getattr(self.model, "predict", None)
            if not callable(predict):
                raise TypeError(f"{type(self.model).__name__} has no predict(state, batch) for the engine to call")
            with torch.set_grad_enabled(is_train):
                out = predict(state, batch)
            if isinstance(out, dict) and (not out or out.get("meta", {}).get("batch_size", 1) == 0):
                continue  # a unit that only advanced state (lock-step padding, RNN warm-up): no loss
            loss = self.task_adapter.compute_loss(out, batch)
            if is_train and isinstance(loss, torch.Tensor) and loss.requires_grad:
                if self.optimizer is not None:
                    self.optimizer.zero_grad()
                loss.backward()
                if self.optimizer is not None:
                    self.optimizer.step()
            losses.append(float(loss.detach()) if isinstance(loss, torch.Tensor) else float(loss))
            for k, v in self.task_adapter.compute_metrics(out, batch).items():
                metric_acc.setdefault(k, []).append(float(v))
            self.state_manager.update(out, chunk)
            outputs.append(self.task_adapter.format_output(out, batch))
        return {"split": split, "loss": sum(losses) / len(losses) if losses else 0.0, "losses": losses,
                "num_batches": len(outputs), "metrics": {k: sum(v) / len(v) for k, v in metric_acc.items()},
                "outputs": outputs}
