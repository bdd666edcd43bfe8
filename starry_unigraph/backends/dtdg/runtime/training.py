"""Flare DTDG training / eval / predict steps (reference backends/dtdg/runtime/training.py:31-295).

Data parallelism: parameters live in one flat buffer; after backward the flat
gradient is averaged across ranks in one collective (the peer-memory all-reduce
kernel on CUDA with ``comm.path: p2p``, NCCL otherwise) and one fused Adam
kernel updates everything. The loss is scaled by local/total nodes
(``part_loss_scale``). Regression tasks use MSE (reference); classification
tasks (``node_classification``) use BCE on one logit / CE on several.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
import torch.nn.functional as F

from starry_unigraph.types import RuntimeBundle, SessionContext

from .models import build_flare_model
from .session_loader import DTDGBatch
from .state import STGraphBlob


def _infer_dims(partition_data: Any) -> tuple[int, int]:
    input_size = int(partition_data.node_data["x"].data.size(-1))
    labels = partition_data.node_data.get("y")
    if labels is None:
        return input_size, 1
    y = labels.data
    if y.dtype == torch.long:
        return input_size, int(y.max().item() + 1 if y.dim() == 1 else y.size(-1))
    return input_size, int(1 if y.dim() == 1 else y.size(-1))


def _compute_part_loss_scale(local_nodes: int, device: str) -> float:
    if not dist.is_available() or not dist.is_initialized():
        return 1.0
    dev = device if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(local_nodes)], device=dev)
    dist.all_reduce(t)
    total = float(t.item())
    return local_nodes / total if total > 0 else 1.0


class FlareOptimizer:
    """Flat-buffer Adam with one gradient all-reduce per step."""

    def __init__(self, model: torch.nn.Module, lr: float, device: torch.device, comm_path: str = "nccl"):
        self.model = model
        self.world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        self.cuda = device.type == "cuda"
        self.comm_path = comm_path
        self._allreduce = None
        if self.cuda:
            from starry_unigraph.ops.flat import FlatParams, FusedAdam

            self.flat = FlatParams([model], device)
            self.opt = FusedAdam(self.flat, lr=lr)
            if self.world > 1 and comm_path == "p2p":
                from starry_unigraph.parallel.allreduce import PeerAllReduceAdam

                self._allreduce = PeerAllReduceAdam(self.flat, self.opt, device)
        else:
            self.opt = torch.optim.Adam(model.parameters(), lr=lr, fused=device.type == "cpu")
        self.param_groups = self.opt.param_groups

    def zero_grad(self, set_to_none: bool = False) -> None:
        if self.cuda:
            self.flat.zero_grad()
        else:
            self.opt.zero_grad(set_to_none=set_to_none)

    def step(self) -> None:
        if self.cuda:
            if self._allreduce is not None:  # fused NVLink all-reduce + Adam
                self._allreduce.step()
                return
            scale = 1.0
            if self.world > 1:
                dist.all_reduce(self.flat.grad)
                scale = 1.0 / self.world
            self.opt.step(grad_scale=scale)
        else:
            if self.world > 1:
                for p in self.model.parameters():
                    if p.grad is None:
                        p.grad = torch.zeros_like(p)
                    dist.all_reduce(p.grad)
                    p.grad /= self.world
            self.opt.step()

    def state_dict(self) -> dict:
        """Full optimizer state. On the NVLink path the moments are sharded by rank
        and this is a collective: every rank must call it."""
        if self._allreduce is not None:
            return self._allreduce.gather_state()
        return self.opt.state_dict()

    def load_state_dict(self, state: dict) -> None:
        self.opt.load_state_dict(state)


def init_flare_training(runtime: RuntimeBundle, session_ctx: SessionContext, partition_data: Any,
                        device: str | None = None) -> None:
    input_size, output_size = _infer_dims(partition_data)
    cfg = session_ctx.config
    device = device or cfg["runtime"]["device"]
    torch.manual_seed(int(cfg.get("train", {}).get("seed", 0)))
    model = build_flare_model(cfg["model"]["name"], input_size, int(cfg["model"]["hidden_dim"]), output_size)
    model = model.to(device)
    opt = FlareOptimizer(model, float(cfg.get("train", {}).get("lr", 1e-3)), torch.device(device),
                         str(cfg.get("comm", {}).get("path", "nccl")))
    if dist.is_available() and dist.is_initialized():
        for p in model.parameters():  # identical initial weights on every rank
            dist.broadcast(p.data, src=0)
    scale = _compute_part_loss_scale(int(partition_data.num_dst_nodes), device)
    task = str(cfg["model"]["task"])
    runtime.model = model
    runtime.optimizer = opt
    runtime.state["flare_model"] = {"name": cfg["model"]["name"], "input_size": input_size,
                                    "hidden_size": int(cfg["model"]["hidden_dim"]), "output_size": output_size,
                                    "part_loss_scale": scale, "task": task}
    runtime.state["part_loss_scale"] = scale
    runtime.state["task"] = task
    dev = torch.device(device)
    comm = str(cfg.get("comm", {}).get("path", "nccl"))
    world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    graphs_ok = dev.type == "cuda" and bool(cfg.get("runtime", {}).get("cuda_graphs", True)) and \
        (world == 1 or comm == "p2p")
    runtime.state["cuda_graphs"] = graphs_ok
    precision = str(cfg.get("runtime", {}).get("precision", "tf32"))
    if precision not in ("tf32", "bf16"):
        raise ValueError(f"runtime.precision must be tf32 or bf16, got {precision!r}")
    runtime.state["precision_tf32"] = (precision == "tf32") if dev.type == "cuda" else None
    runtime.state["step_graphs"] = StepGraphs(dev) if graphs_ok else None


def _get_labels(graph: Any) -> torch.Tensor | None:
    y = graph.dstdata.get("y")
    if y is None:
        y = graph.srcdata.get("y")
        y = None if y is None else y[: graph.num_dst_nodes]
    if y is None:
        return None
    return y.view(-1, 1) if y.dim() == 1 else y


def _forward_single_graph(runtime: RuntimeBundle, graph: Any, state: Any):
    """One snapshot outside a window (evaluation): the state passes through unchanged."""
    model = runtime.model.module if hasattr(runtime.model, "module") else runtime.model
    return model(graph, state)


def _precision(runtime: RuntimeBundle):
    """Context selecting the run's tensor-core operand precision (no-op on CPU)."""
    from contextlib import nullcontext

    if runtime.state.get("precision_tf32") is None:
        return nullcontext()
    from starry_unigraph.ops import gemm_precision

    return gemm_precision(bool(runtime.state["precision_tf32"]))


def _loss_and_predictions(runtime: RuntimeBundle, blob_or_batch, training: bool, need_host: bool = True):
    model = runtime.model
    model.train(training)
    if isinstance(blob_or_batch, STGraphBlob):
        preds, _ = model(blob_or_batch)
        last = blob_or_batch.current_graph
    else:
        graph = blob_or_batch.graph
        if graph is None:
            raise RuntimeError("flare_native batch.graph is not available")
        preds, new_state = _forward_single_graph(runtime, graph, runtime.state.get("eval_rnn_state"))
        runtime.state["eval_rnn_state"] = new_state
        last = graph
    pred = preds[-1] if isinstance(preds, list) else preds
    labels = _get_labels(last)
    pred_values = pred.detach().view(-1).cpu().tolist() if need_host else pred.detach()
    if labels is None:
        return None, pred_values, None
    labels = labels.to(pred.device)
    if pred.size(-1) != labels.size(-1):
        labels = labels[..., : pred.size(-1)]
    scale = float(runtime.state.get("part_loss_scale", 1.0))
    if labels.numel() == 0:  # no labelled row of this partition in the snapshot: zero loss, zero gradients
        loss = pred.sum() * 0.0
    elif runtime.state.get("task") == "node_classification":
        if pred.size(-1) == 1:
            loss = F.binary_cross_entropy_with_logits(pred, labels.float()) * scale
        else:
            loss = F.cross_entropy(pred, labels.long().view(-1)) * scale
    else:
        loss = F.mse_loss(pred, labels.float()) * scale
    targets = labels.detach().view(-1).cpu().tolist() if need_host else labels.detach()
    return loss, pred_values, targets


class StepGraphs:
    """Whole DTDG training steps (forward, backward, optimizer) as CUDA graphs,
    one per training window.

    An eager step issues a few hundred kernels from Python (~50 us of host time
    each), which bounds the step once its GPU work is split over several ranks.
    A window's step is captured the first time it is seen after two eager
    warm-up steps and replayed afterwards (every epoch visits the same windows).
    All graphs share one memory pool: only transient activations live there;
    parameters, gradients, optimizer moments and halo buffers are allocated
    before capture, and each replay's loss / predictions are copied out of the
    pool before the next one can overwrite them. Host-side per-snapshot caches
    (CSR orders, halo pull plans) are built eagerly before a capture.

    Used on CUDA for ``pad``-mode windows (the state is not carried between
    windows) on one GPU or with the NVLink collectives (``comm.path: p2p``)."""

    WARMUP = 2

    def __init__(self, device: torch.device) -> None:
        self.device = torch.device(device)
        self.graphs: dict[tuple, tuple] = {}
        self.pool = torch.cuda.graph_pool_handle()
        self.eager = 0
        self.captures = 0
        self.launches_per_step = 0  # this library's kernel launches in one captured step

    @staticmethod
    def supported(runtime: RuntimeBundle, blob: Any) -> bool:
        if not isinstance(blob, STGraphBlob) or not bool(runtime.state.get("cuda_graphs", False)):
            return False
        # windows with decayed (truncated) slots come from a chunk order drawn anew every epoch:
        # their graphs would never replay, so they run eagerly
        return getattr(blob.state, "mode", "pad") == "pad" and all(st.full for st in blob.steps)

    @staticmethod
    def key(blob: Any) -> tuple:
        return tuple((st.snapshot_id, st.slot, int(st.graph.num_src_nodes), int(st.graph.num_dst_nodes),
                      int(st.graph.num_edges())) for st in blob.steps)

    @staticmethod
    def _prepare(blob: Any) -> None:
        from starry_unigraph.parallel.halo import get_halo_context

        hc = get_halo_context()
        for g in blob:
            g.csr()
            if hc is not None and getattr(g, "route", None) is not None and g.num_src_nodes > g.num_dst_nodes:
                hc.pull_plan(g, g.num_dst_nodes)

    def _step(self, runtime: RuntimeBundle, blob: Any):
        with _precision(runtime):
            loss, preds, targets = _loss_and_predictions(runtime, blob, training=True, need_host=False)
            runtime.optimizer.zero_grad(set_to_none=True)
            loss.backward()
            runtime.optimizer.step()
        return loss.detach(), preds, targets

    def run(self, runtime: RuntimeBundle, blob: Any):
        key = self.key(blob)
        entry = self.graphs.get(key)
        if entry is None:
            if self.eager < self.WARMUP:
                self.eager += 1
                return self._step(runtime, blob)
            self._prepare(blob)
            torch.cuda.synchronize(self.device)
            from starry_unigraph.ops import cuda_ext

            n0 = cuda_ext().launch_count()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, pool=self.pool):
                out = self._step(runtime, blob)
            self.launches_per_step = int(cuda_ext().launch_count() - n0)
            entry = (graph, out, blob)  # the blob keeps the captured tensors alive
            self.graphs[key] = entry
            self.captures += 1
        graph, (loss, preds, targets), _ = entry
        graph.replay()
        return loss.clone(), preds.clone(), (None if targets is None else targets.clone())

    def reset(self) -> None:
        self.graphs.clear()


def run_flare_train_step(runtime: RuntimeBundle, batch: Any, kernel_output: dict[str, Any],
                         need_host: bool = True) -> dict[str, Any]:
    graphs = runtime.state.get("step_graphs")
    if graphs is not None and StepGraphs.supported(runtime, batch):
        loss, preds, targets = graphs.run(runtime, batch)
        if need_host:
            preds = preds.view(-1).cpu().tolist()
            targets = None if targets is None else targets.view(-1).cpu().tolist()
        return {"loss": float(loss.item()) if need_host else loss, "predictions": preds, "targets": targets,
                "meta": kernel_output.get("meta", {}) | {"model": runtime.state["flare_model"],
                                                          "sequence_state": "updated", "cuda_graph": True}}
    with _precision(runtime):
        loss, preds, targets = _loss_and_predictions(runtime, batch, training=True, need_host=need_host)
        if loss is None:
            raise RuntimeError("Training labels are required for flare_native train_step")
        runtime.optimizer.zero_grad(set_to_none=True)
        loss.backward()
        runtime.optimizer.step()
    return {"loss": float(loss.detach().item()) if need_host else loss.detach(), "predictions": preds,
            "targets": targets,
            "meta": kernel_output.get("meta", {}) | {"model": runtime.state["flare_model"],
                                                      "sequence_state": "updated"}}


def run_flare_eval_step(runtime: RuntimeBundle, batch: Any, kernel_output: dict[str, Any]) -> dict[str, Any]:
    with torch.no_grad(), _precision(runtime):
        if getattr(batch, "chain", "") == "snapshot_warmup":
            _, new_state = _forward_single_graph(runtime, batch.graph, runtime.state.get("eval_rnn_state"))
            runtime.state["eval_rnn_state"] = new_state
            return {}
        loss, preds, targets = _loss_and_predictions(runtime, batch, training=False)
    out = {"predictions": preds, "targets": targets,
           "meta": kernel_output.get("meta", {}) | {"model": runtime.state["flare_model"]}}
    if loss is not None:
        out["loss"] = float(loss.detach().item())
        if targets is not None:
            out["meta"]["metrics"] = _eval_metrics(runtime.state.get("task"), torch.tensor(preds),
                                                   torch.tensor(targets))
    return out


def _eval_metrics(task: str | None, p: torch.Tensor, t: torch.Tensor) -> dict[str, float]:
    """Regression: MAE / RMSE. Classification: accuracy (one logit per node: positive means
    class 1; C logits per node: the arg-max)."""
    if t.numel() == 0:
        return {}
    if task == "node_classification":
        if p.numel() == t.numel():
            hit = (p > 0).float() == t.float()
        else:
            hit = p.view(t.numel(), -1).argmax(1) == t.long()
        return {"accuracy": float(hit.float().mean())}
    p, t = p.float(), t.float()
    return {"mae": float((p - t).abs().mean()), "rmse": float((p - t).pow(2).mean().sqrt())}


def run_flare_predict_step(runtime: RuntimeBundle, batch: Any, kernel_output: dict[str, Any]) -> dict[str, Any]:
    with torch.no_grad(), _precision(runtime):
        if getattr(batch, "chain", "") == "snapshot_warmup":
            _, new_state = _forward_single_graph(runtime, batch.graph, runtime.state.get("eval_rnn_state"))
            runtime.state["eval_rnn_state"] = new_state
            return {}
        _, preds, targets = _loss_and_predictions(runtime, batch, training=False)
    return {"predictions": preds, "targets": targets,
            "meta": kernel_output.get("meta", {}) | {"model": runtime.state["flare_model"]}}
