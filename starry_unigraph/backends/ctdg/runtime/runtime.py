"""CTDG online runtime: TGN-family temporal link prediction
(reference backends/ctdg/runtime/runtime.py:39-391).

Per batch: drain pending memory syncs -> negatives -> temporal sampling ->
memory update (GRU over the mailbox, written detached with ts = max batch ts)
-> mailbox write from the pre-update memories -> temporal attention over the
updated memory -> link scores -> BCE loss -> backward -> Adam -> push updates
of remote-owned nodes to their owners.

On CUDA devices the whole step runs as the fused sm_100a kernel sequence of
``starry_unigraph.ops.tgn.TGNCudaEngine`` (captured in a CUDA graph); on CPU
the same math runs as plain PyTorch (this path is also the numerical oracle).
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Iterable

import torch
import torch.nn.functional as F

from starry_unigraph.tasks.temporal_link_prediction import average_precision, pairwise_auc
from starry_unigraph.types import DistributedContext

from .data import CTDGDataBatch, TGTemporalDataset
from .memory import CTDGMemoryBank
from .models import CTDGLinkPredictor
from .route import CTDGFeatureRoute
from .sampler import CTDGSampleOutput, NativeTemporalSampler


@dataclass
class CTDGPreparedBatch:
    batch: CTDGDataBatch
    neg_dst: torch.Tensor
    sample: CTDGSampleOutput | None
    roots: torch.Tensor | None = None
    root_ts: int = 0
    prev_ts: torch.Tensor | None = None  # memory_ts of the roots before this step's update (JODIE)


def _grad_allreduce(params: list[torch.nn.Parameter], world_size: int) -> None:
    import torch.distributed as dist

    grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in params]
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat)
    flat /= world_size
    off = 0
    for p, g in zip(params, grads):
        n = g.numel()
        if p.grad is None:
            p.grad = flat[off:off + n].view_as(p).clone()
        else:
            p.grad.copy_(flat[off:off + n].view_as(p))
        off += n


class CTDGOnlineRuntime:
    def __init__(self, dataset: TGTemporalDataset, sampler: NativeTemporalSampler, memory: CTDGMemoryBank,
                 model: CTDGLinkPredictor, optimizer: Any, route: CTDGFeatureRoute, device: str,
                 dist_ctx: DistributedContext, memory_updater: torch.nn.Module | None = None, engine: Any = None,
                 memory_grad: bool = False, seed: int = 0, adaptive_alpha: bool = False):
        self.dataset = dataset
        self.sampler = sampler
        self.memory = memory
        self.model = model
        self.optimizer = optimizer
        self.route = route
        self.device = device
        self.dist_ctx = dist_ctx
        self.memory_updater = memory_updater
        self.engine = engine
        self.memory_grad = memory_grad
        # with a historical cache: move its push threshold with each step's sync / compute time
        self.adaptive_alpha = adaptive_alpha
        self._gen = torch.Generator().manual_seed(seed)
        self._dst_node_pool: torch.Tensor | None = None
        self._edge_feat_dev: torch.Tensor | None = None

    # ------------------------------------------------------------------ helpers
    @property
    def _core(self) -> CTDGLinkPredictor:
        return self.model.module if hasattr(self.model, "module") else self.model

    def iter_batches(self, split: str, batch_size: int) -> Iterable[CTDGDataBatch]:
        yield from self.dataset.iter_batches(split=split, batch_size=batch_size)

    def _negative_sample(self, batch: CTDGDataBatch) -> torch.Tensor:
        if self._dst_node_pool is None:
            self._dst_node_pool = self.dataset.dst_pool()
        pool = self._dst_node_pool
        idx = torch.randint(0, pool.numel(), batch.dst.shape, generator=self._gen)
        neg = pool[idx]
        coll = neg.eq(batch.dst.cpu())
        if bool(coll.any()):
            idx[coll] = (idx[coll] + 1) % pool.numel()
            neg = pool[idx]
        return neg

    @property
    def _jodie(self) -> bool:
        from .models import CTDGJodiePredictor

        return isinstance(self._core, CTDGJodiePredictor)

    def _prepare(self, batch: CTDGDataBatch) -> CTDGPreparedBatch:
        neg = self._negative_sample(batch)
        roots = torch.unique(torch.cat([batch.src, batch.dst])).long()
        root_ts = int(batch.ts.max().item())
        if self._jodie:  # time-projection embedding: no neighbour sampling
            prev = self.memory.memory_ts[roots.to(self.memory.memory_ts.device)].clone()
            return CTDGPreparedBatch(batch, neg, None, roots, root_ts, prev)
        ts = torch.full((roots.numel(),), root_ts, dtype=torch.long)
        split = batch.split if batch.split != "predict" else "test"
        return CTDGPreparedBatch(batch, neg, self.sampler.sample(split, roots, ts), roots, root_ts)

    def _pull(self, prepared: CTDGPreparedBatch | None) -> None:
        """Remote reads (``ctdg.remote_fetch``, several ranks): refresh the rows this step
        reads from their owners, the roots and every sampled neighbour. A collective:
        every rank calls it once per step, with nothing to ask for on an empty step."""
        if prepared is None:
            ids = torch.empty(0, dtype=torch.long)
        elif prepared.sample is not None:
            ids = prepared.sample.sampled_nodes
        else:
            ids = prepared.roots
        self.memory.pull_remote(self.dist_ctx, ids)

    def _edge_feats(self) -> torch.Tensor:
        if self._edge_feat_dev is None:
            ef = self.dataset.edge_feat.float()
            if ef.dim() == 1:
                ef = ef.view(-1, 1)
            E = self.memory.edge_feat_dim
            if ef.size(1) < E:
                ef = torch.cat([ef, torch.zeros(ef.size(0), E - ef.size(1))], dim=1)
            self._edge_feat_dev = ef[:, :E].to(self.device)
        return self._edge_feat_dev

    def _conv_output(self, nodes: torch.Tensor, roots: torch.Tensor, conv_all: torch.Tensor) -> torch.Tensor:
        nodes = nodes.to(roots.device)
        idx = torch.searchsorted(roots, nodes).clamp(0, max(0, roots.numel() - 1))
        valid = roots[idx] == nodes if roots.numel() else torch.zeros_like(nodes, dtype=torch.bool)
        out = conv_all[idx] if roots.numel() else torch.zeros(nodes.numel(), conv_all.size(1))
        return out * valid.unsqueeze(1)

    def _conv_all(self, prepared: CTDGPreparedBatch) -> tuple[torch.Tensor, torch.Tensor]:
        if self._jodie:
            roots = prepared.roots.to(self.device)
            h = self.memory.gather(roots)
            if not self.memory_grad:
                h = h.detach()
            prev = prepared.prev_ts.to(self.device)
            dt = torch.where(prev >= 0, float(prepared.root_ts) - prev, torch.zeros_like(prev))
            return roots, self._core.embed(h, dt)
        blk = prepared.sample.blocks[0]
        roots = blk.roots.to(self.device)
        mask = blk.mask().to(self.device)
        nbr = blk.nbr.to(self.device).clamp(min=0)
        h_root = self.memory.gather(roots)
        h_nbr = self.memory.gather(nbr.reshape(-1)).view(*nbr.shape, -1) * mask.unsqueeze(-1)
        if not self.memory_grad:
            h_root, h_nbr = h_root.detach(), h_nbr.detach()
        ef = self._edge_feats()[blk.eid.to(self.device).clamp(min=0)] * mask.unsqueeze(-1)
        conv = self._core.conv.forward_dense(h_root, h_nbr, ef, blk.dt.to(self.device), mask)
        return roots, conv

    def _scores(self, prepared: CTDGPreparedBatch) -> tuple[torch.Tensor, torch.Tensor]:
        roots, conv = self._conv_all(prepared)
        b = prepared.batch
        out = self.model(src_conv=self._conv_output(b.src, roots, conv), dst_conv=self._conv_output(b.dst, roots, conv),
                         neg_conv=self._conv_output(prepared.neg_dst, roots, conv))
        return out.pos_logits, out.neg_logits

    @staticmethod
    def _metric_dict(pos: torch.Tensor, neg: torch.Tensor) -> dict[str, float]:
        p, n = torch.sigmoid(pos).detach().cpu(), torch.sigmoid(neg).detach().cpu()
        scores = torch.cat([p, n])
        labels = torch.cat([torch.ones_like(p), torch.zeros_like(n)])
        return {"ap": average_precision(scores, labels), "auc": pairwise_auc(p, n),
                "mrr": float((p.unsqueeze(1) > n.unsqueeze(0)).float().mean()) if p.numel() else 0.0}

    def _update_memory(self, batch: CTDGDataBatch) -> None:
        dev = self.device
        src, dst = batch.src.to(dev), batch.dst.to(dev)
        src_prev = self.memory.gather(src).detach().clone()
        dst_prev = self.memory.gather(dst).detach().clone()
        all_nodes = torch.unique(torch.cat([src, dst]))
        mail = self.memory.read_mailbox(all_nodes)
        cur = self.memory.gather(all_nodes)
        with torch.set_grad_enabled(self.memory_grad and torch.is_grad_enabled()):
            upd = self.memory_updater(mail, cur)
        ts_scalar = float(batch.ts.max().item())
        self.memory._apply_memory_update(all_nodes, upd.detach(),
                                         torch.full((all_nodes.numel(),), ts_scalar, device=dev))
        self.memory.write_mailbox(src, dst, src_prev, dst_prev, batch.edge_feat.to(dev), batch.ts.to(dev))

    def _sync_updater_params(self) -> None:
        """Updater parameters receive no gradient (memory is written detached), so the
        reference's per-step rank-0 broadcast is a no-op after the first; one
        broadcast at construction keeps every rank identical."""
        return

    def broadcast_updater_params(self) -> None:
        import torch.distributed as dist

        if self.memory_updater is None or not (self.dist_ctx.is_distributed and dist.is_initialized()):
            return
        for p in self.memory_updater.parameters():
            dist.broadcast(p.data, src=0)

    def _submit_syncs(self, batch: CTDGDataBatch) -> None:
        if not self.dist_ctx.is_distributed:
            return
        dev = self.device
        ids = torch.unique(torch.cat([batch.src, batch.dst]).to(dev)) if batch.size else \
            torch.empty(0, dtype=torch.long, device=dev)
        ts_scalar = float(batch.ts.max().item()) if batch.size else 0.0
        vals = self.memory.memory[ids] if ids.numel() else torch.zeros(0, self.memory.hidden_dim, device=dev)
        self.memory.submit_async_memory_sync(self.dist_ctx, ids, vals, torch.full((ids.numel(),), ts_scalar, device=dev))
        self.memory.submit_async_mail_sync(self.dist_ctx, ids, self.memory.mailbox[ids], self.memory.mailbox_ts[ids])

    def _empty_result(self, split: str) -> dict[str, Any]:
        return {"loss": 0.0, "predictions": [], "targets": [],
                "meta": {"split": split, "batch_size": 0, "metrics": {}, "memory": self.memory.describe(),
                         "empty_batch": True}}

    # ------------------------------------------------------------------ steps
    def train_step(self, batch: CTDGDataBatch) -> dict[str, Any]:
        if self.engine is not None:
            return self._engine_step(batch, "train", train=True)
        self.model.train()
        t0 = time.perf_counter()
        self.memory.wait_pending_syncs()
        wait_ms = (time.perf_counter() - t0) * 1000.0
        if batch.is_empty:
            self._pull(None)
            self.optimizer.zero_grad(set_to_none=False)
            zero = sum(p.sum() * 0.0 for p in self._core.parameters())
            zero.backward()
            if self.dist_ctx.is_distributed:
                _grad_allreduce(list(self._core.parameters()), self.dist_ctx.world_size)
            self.optimizer.step()
            self._submit_syncs(batch)
            res = self._empty_result(batch.split)
            res["meta"].update(sync_wait_ms=wait_ms, sync_submit_ms=0.0, step_ms=(time.perf_counter() - t0) * 1e3)
            return res
        prepared = self._prepare(batch)
        self._pull(prepared)
        self._update_memory(batch)
        pos, neg = self._scores(prepared)
        loss = F.binary_cross_entropy_with_logits(pos, torch.ones_like(pos)) + \
            F.binary_cross_entropy_with_logits(neg, torch.zeros_like(neg))
        self.optimizer.zero_grad(set_to_none=True)
        loss.backward()
        if self.dist_ctx.is_distributed:
            _grad_allreduce(list(self._core.parameters()), self.dist_ctx.world_size)
        self.optimizer.step()
        t1 = time.perf_counter()
        self._submit_syncs(batch)
        submit_ms = (time.perf_counter() - t1) * 1000.0
        step_ms = (time.perf_counter() - t0) * 1000.0
        cache = self.memory.historical_cache
        if cache is not None and self.adaptive_alpha:
            cache.ada_param.update_from_latency(wait_ms + submit_ms, step_ms - wait_ms - submit_ms)
        return {"loss": float(loss.item()), "predictions": torch.sigmoid(pos).detach().cpu().tolist(),
                "targets": [1] * batch.size,
                "meta": {"split": batch.split, "batch_size": batch.size, "sample": prepared.sample.describe() if prepared.sample is not None else None,
                         "metrics": self._metric_dict(pos, neg), "memory": self.memory.describe(),
                         "sync_wait_ms": wait_ms, "sync_submit_ms": submit_ms, "step_ms": step_ms,
                         "historical_alpha": cache.ada_param.alpha if cache is not None else None}}

    def eval_step(self, batch: CTDGDataBatch, split: str) -> dict[str, Any]:
        if self.engine is not None:
            return self._engine_step(batch, split, train=False)
        self.memory.wait_pending_syncs()
        self.model.eval()
        with torch.no_grad():
            if batch.is_empty:
                self._pull(None)
                self._submit_syncs(batch)
                return self._empty_result(split)
            prepared = self._prepare(batch)
            self._pull(prepared)
            self._update_memory(batch)
            pos, neg = self._scores(prepared)
            loss = F.binary_cross_entropy_with_logits(pos, torch.ones_like(pos)) + \
                F.binary_cross_entropy_with_logits(neg, torch.zeros_like(neg))
        self._submit_syncs(batch)
        return {"loss": float(loss.item()), "predictions": torch.sigmoid(pos).cpu().tolist(),
                "targets": [1] * batch.size,
                "meta": {"split": split, "batch_size": batch.size, "metrics": self._metric_dict(pos, neg),
                         "memory": self.memory.describe()}}

    def predict_step(self, batch: CTDGDataBatch) -> dict[str, Any]:
        res = self.eval_step(batch, split=batch.split)
        res["meta"]["predict"] = True
        return res

    # ------------------------------------------------------------------ CUDA engine path
    def _engine_step(self, batch: CTDGDataBatch, split: str, train: bool, want_outputs: bool = True) -> dict[str, Any]:
        eng = self.engine
        split = "test" if split == "predict" else split
        nccl_sync = self.dist_ctx.is_distributed and eng.peer is None  # the NVLink path syncs inside the step
        if nccl_sync:
            self.memory.wait_pending_syncs()
            if self.memory.remote_fetch:
                self.memory.pull_remote(self.dist_ctx, torch.cat([batch.src, batch.dst]))
        eng.load_batch(batch.src, batch.dst, batch.ts, batch.event_ids)
        if train:
            self.model.train()
        eng.step(split, train)
        if nccl_sync:
            self._submit_syncs(batch)
        if not want_outputs:
            return {}
        loss, metrics = eng.read_scalars()
        if batch.is_empty:
            res = self._empty_result(split)
            res["loss"] = loss
            return res
        return {"loss": loss, "predictions": eng.pos_probs(batch.size).cpu().tolist(), "targets": [1] * batch.size,
                "meta": {"split": split, "batch_size": batch.size, "metrics": metrics,
                         "memory": self.memory.describe()}}

    def run_batches_device(self, batches: list[CTDGDataBatch], split: str = "train", train: bool = True,
                           on_step: Any = None) -> list[dict[str, Any]]:
        """Stream given batches through the CUDA engine: per step the inputs are copied
        host -> device (asynchronously from pinned memory) and the step's loss and
        metrics device -> host into a pinned buffer, without a host synchronisation
        between steps; one synchronisation at the end returns every step's result."""
        eng = self.engine
        n = len(batches)
        res = torch.empty(n, 4, dtype=torch.float32, pin_memory=True)
        if train:
            self.model.train()
        split = "test" if split == "predict" else split
        for i, b in enumerate(batches):
            if on_step is not None:
                on_step(i)
            eng.load_batch(b.src, b.dst, b.ts, b.event_ids)
            eng.step(split, train)
            res[i, 0:1].copy_(eng.loss, non_blocking=True)   # stream-ordered before the next step overwrites it
            res[i, 1:4].copy_(eng.metrics, non_blocking=True)
        eng.drain()
        out = []
        for i, b in enumerate(batches):
            loss, ap, auc, mrr = res[i].tolist()
            out.append({"loss": loss, "meta": {"split": split, "batch_size": b.size,
                                               "metrics": {"ap": ap, "auc": auc, "mrr": mrr} if b.size else {}}})
        return out

    def run_split_device(self, split: str, batch_size: int, train: bool, max_steps: int | None = None,
                         collect_predictions: bool = False, on_step: Any = None) -> dict[str, Any]:
        """Epoch over a split without per-step host synchronisation (CUDA engine only):
        losses and metrics accumulate on the device and are read once at the end."""
        eng = self.engine
        losses, mets, preds, sizes = [], [], [], []
        for i, batch in enumerate(self.iter_batches(split, batch_size)):
            if max_steps is not None and i >= max_steps:
                break
            if on_step is not None:
                on_step(i)
            self._engine_step(batch, split, train, want_outputs=False)
            losses.append(eng.loss.clone())
            mets.append(eng.metrics.clone())
            sizes.append(batch.size)
            if collect_predictions:
                preds.append(eng.pos_probs(batch.size).clone())
        eng.drain()  # multi-GPU: every peer's last pushes have landed before the caller reads anything
        if not losses:
            return {"losses": [], "metrics": [], "sizes": [], "predictions": []}
        L = torch.cat(losses).tolist()
        M = torch.stack(mets).tolist()
        P = [p.cpu().tolist() for p in preds] if collect_predictions else []
        return {"losses": L, "metrics": M, "sizes": sizes, "predictions": P}
