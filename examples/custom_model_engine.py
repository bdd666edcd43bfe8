"""A user-defined model trained through the unified pipeline engine.

The session prepares the data and provides the graph backend; the model is your own
``nn.Module`` with ``predict(state, batch)``. Every unit of the backend is
materialised into a ``BatchData``: its roots (the events' endpoints), a temporal
neighbour block (``batch.mfg``, most recent neighbours strictly before the unit) and,
because the engine is given a feature store, the feature rows of every sampled
neighbour (``batch.nbr_feat``, [roots, k, F]). The task adapter turns the model's
scores into the loss; the engine runs backward and the optimizer.

    python examples/custom_model_engine.py --config configs/tgn_wiki.yaml --events 20000 --device cpu

The model here is deliberately small: a root's embedding is an MLP of its own features
and the mean of its neighbours' features, and an event's score is a bilinear form of
its endpoints' embeddings against a random negative destination.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch
from torch import nn


class MeanNeighbourLinkModel(nn.Module):
    def __init__(self, store, hidden: int = 64):
        super().__init__()
        self.store = store
        f = store.feat_dim()
        self.mlp = nn.Sequential(nn.Linear(2 * f, hidden), nn.ReLU(), nn.Linear(hidden, hidden))
        self.bilinear = nn.Parameter(torch.eye(hidden))

    def embed(self, batch) -> torch.Tensor:
        blk = batch.mfg
        mask = blk.mask().unsqueeze(-1).float()
        nbr = (batch.nbr_feat * mask).sum(1) / mask.sum(1).clamp(min=1.0)
        own = self.store.get_node_feat(blk.roots)
        return self.mlp(torch.cat([own, nbr], dim=1))

    def predict(self, state, batch) -> dict:
        roots = batch.mfg.roots  # sorted unique endpoints of the unit's events
        h = self.embed(batch)
        src = torch.searchsorted(roots, batch.pos_src.long())
        dst = torch.searchsorted(roots, batch.pos_dst.long())
        neg = torch.randint(0, roots.numel(), dst.shape)
        hs = h[src] @ self.bilinear
        return {"pos_score": (hs * h[dst]).sum(-1), "neg_score": (hs * h[neg]).sum(-1)}


def main(argv=None) -> dict:
    from starry_unigraph import SchedulerSession
    from starry_unigraph.data import TensorFeatureStore
    from starry_unigraph.runtime.backend_adapters import CTDGGraphBackend, DummyStateManager
    from starry_unigraph.runtime.engine import PipelineEngine
    from starry_unigraph.tasks import EdgePredictAdapter

    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--config", default=str(Path(__file__).resolve().parents[1] / "configs" / "tgn_wiki.yaml"))
    p.add_argument("--events", type=int, default=None, help="synthetic streams: first N events only")
    p.add_argument("--device", default="cpu")
    p.add_argument("--epochs", type=int, default=2)
    p.add_argument("--batch-size", type=int, default=200, dest="batch_size")
    p.add_argument("--artifact-root", default=None)
    a = p.parse_args(argv)
    over = {"runtime": {"device": a.device}, "train": {"batch_size": a.batch_size}}
    if a.events:
        over["data"] = {"synthetic": {"num_events": a.events}}
    s = SchedulerSession.from_config(a.config, overrides=over)
    if a.artifact_root:
        s.ctx.artifact_root = Path(a.artifact_root)
    s.prepare_data()
    s.build_runtime()
    num_nodes = s.ctdg_session.online_runtime.dataset.num_nodes
    store = TensorFeatureStore(torch.randn(num_nodes, 16, generator=torch.Generator().manual_seed(0)))
    model = MeanNeighbourLinkModel(store)
    engine = PipelineEngine(backend=CTDGGraphBackend(s.ctdg_session), state_manager=DummyStateManager(), model=model,
                            task_adapter=EdgePredictAdapter(), optimizer=torch.optim.Adam(model.parameters(), lr=1e-3),
                            feature_store=store)
    result = {}
    for epoch in range(a.epochs):
        tr = engine.run_epoch("train", batch_size=a.batch_size)
        va = engine.run_epoch("val", batch_size=a.batch_size)
        print(f"epoch {epoch + 1} | train loss {tr['loss']:.4f} | val loss {va['loss']:.4f} "
              f"auc {va['metrics'].get('auc', 0.0):.4f} ap {va['metrics'].get('ap', 0.0):.4f}", flush=True)
        result = {"train": tr["losses"], "val": va}
    return result


if __name__ == "__main__":
    main()
