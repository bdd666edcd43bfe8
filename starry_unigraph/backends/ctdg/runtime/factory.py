"""Build a CTDG online runtime from a session context
(reference backends/ctdg/runtime/factory.py:20-178)."""
from __future__ import annotations

from pathlib import Path

import torch

from starry_unigraph.types import RuntimeBundle, SessionContext

from .cache import AdaParameter, CTDGHistoricalCache
from .data import TGTemporalDataset
from .memory import CTDGMemoryBank
from .models import build_ctdg_model, build_memory_updater
from .route import CTDGFeatureRoute
from .runtime import CTDGOnlineRuntime
from .sampler import NativeTemporalSampler


def _load_parts(session_ctx: SessionContext, name: str, flag: str):
    pa = session_ctx.prepared_artifacts
    if pa is None or not pa.provider_meta.get(flag):
        return None
    path = pa.directories.get("partitions", session_ctx.artifact_root / "partitions") / name
    return torch.load(path, weights_only=True) if path.exists() else None


def _engine_bmax(session_ctx: SessionContext, batch_size: int, world_size: int, owner_events: bool) -> int:
    """Events the CUDA step's static buffers hold. With the owner rule a rank's share of a
    global window varies: the largest share, as the preprocessor recorded it (in this
    process, or in the artifacts' metadata when another process prepared them)."""
    if world_size <= 1 or not owner_events:
        return batch_size
    known = session_ctx.provider_state.get("max_local_batch")
    if known is None and session_ctx.prepared_artifacts is not None:
        known = session_ctx.prepared_artifacts.provider_meta.get("max_local_batch")
    return max(batch_size, int(known)) if known else 2 * batch_size


def build_ctdg_runtime(session_ctx: SessionContext, dataset: TGTemporalDataset | None = None):
    cfg = session_ctx.config
    root = session_ctx.dataset_path or Path(cfg["data"]["root"]).expanduser().resolve()
    if dataset is None:
        dataset = TGTemporalDataset(root, cfg["data"]["name"], split_ratio=cfg.get("data", {}).get("split_ratio"),
                                    config=cfg, raw=session_ctx.provider_state.get("raw_events"))
    device = str(cfg["runtime"]["device"])
    if device.startswith("cuda") and not torch.cuda.is_available():
        device = "cpu"
    if device == "cuda":
        device = f"cuda:{session_ctx.dist.local_rank}" if session_ctx.dist.is_distributed else "cuda:0"
    strategy = str(cfg["sampling"]["strategy"])
    if device.startswith("cuda") and strategy not in ("recent", "uniform"):
        raise ValueError(f"sampling.strategy {strategy!r} runs in the host sampler only; the CUDA step samples "
                         "'recent' or 'uniform' (use runtime.device: cpu for the other policies)")
    hidden = int(cfg["model"]["hidden_dim"])
    dctx = session_ctx.dist
    c = cfg.get("ctdg", {})
    slots = int(c.get("mailbox_slots", 4))
    edim = max(1, dataset.edge_feat_dim)
    node_parts = _load_parts(session_ctx, "node_parts.pt", "has_node_parts")
    edge_parts = _load_parts(session_ctx, "edge_parts.pt", "has_edge_parts")
    if dctx.world_size > 1 and node_parts is None:
        node_parts = torch.arange(dataset.num_nodes, dtype=torch.long) % dctx.world_size
        edge_parts = node_parts[dataset.src]
    # events per rank: "owner" = the events whose source this rank owns (reference rule;
    # per-rank batch sizes follow the stream's skew), "balanced" = an equal share of each
    # global window (needs every rank to read and push any node's rows); "auto" picks
    # balanced on the NVLink path with remote reads, owner elsewhere
    assignment = str(c.get("event_partition", "auto"))
    if assignment == "auto":
        nvlink = device.startswith("cuda") and str(cfg.get("comm", {}).get("path", "p2p")) == "p2p"
        assignment = "balanced" if (nvlink and bool(c.get("remote_fetch", True))) else "owner"
    dataset.configure_partition(node_parts=node_parts, edge_parts=edge_parts, rank=dctx.rank,
                                world_size=dctx.world_size, assignment=assignment)
    memory = CTDGMemoryBank(num_nodes=dataset.num_nodes, hidden_dim=hidden, device=device, mailbox_slots=slots,
                            edge_feat_dim=edim, rank=dctx.rank, world_size=dctx.world_size,
                            async_sync=bool(c.get("async_sync", True)), node_parts=node_parts,
                            remote_fetch=bool(c.get("remote_fetch", True)))
    family = str(cfg["model"]["family"])
    seed = int(cfg.get("train", {}).get("seed", 0))
    torch.manual_seed(seed)
    embedding = str(c.get("embedding") or ("time_projection" if family == "jodie" else "attention"))
    model = build_ctdg_model(family, num_nodes=dataset.num_nodes, hidden_dim=hidden, edge_feat_dim=edim,
                             dim_time=int(c.get("dim_time", 100)), num_head=int(c.get("num_head", 2)),
                             dropout=float(c.get("dropout", 0.1)), att_dropout=float(c.get("att_dropout", 0.1)),
                             embedding=embedding)
    if hasattr(model, "dt_scale"):
        span = float(dataset.ts.max() - dataset.ts.min()) if dataset.ts.numel() else 1.0
        model.dt_scale = 1.0 / max(span, 1.0)
    model = model.to(device)
    mem_type = str(cfg["model"].get("memory", {}).get("type", "gru"))
    if embedding == "time_projection":
        mem_type = "rnn"  # JODIE: tanh-RNN memory updater
    updater = build_memory_updater(mem_type, hidden_dim=hidden, mailbox_slot_dim=2 * hidden + edim,
                                   mailbox_slots=slots).to(device)
    for p in updater.parameters():
        p.requires_grad_(bool(c.get("memory_grad", False)))
    sampling = cfg["sampling"]
    fanout = list(sampling["neighbor_limit"])
    strategy = str(sampling["strategy"])
    sampler = NativeTemporalSampler(dataset, fanout=fanout, history=int(sampling["history"]), strategy=strategy,
                                    workers=max(1, min(4, dctx.local_world_size)), device=device,
                                    boundary_p=float(sampling.get("boundary_p", 1.0)))
    lr = float(cfg.get("train", {}).get("lr", 1e-3))
    route = CTDGFeatureRoute(route_type=str(cfg["graph"]["route"]), world_size=dctx.world_size)
    engine = None
    fused_ok = (embedding == "time_projection") == (mem_type == "rnn")  # TGN+GRU or JODIE+RNN
    if device.startswith("cuda") and fused_ok:
        from starry_unigraph.ops.tgn import TGNCudaEngine

        grad_sync = None
        peer = None
        comm_path = str(cfg.get("comm", {}).get("path", "p2p"))
        if dctx.is_distributed and comm_path == "p2p":
            from starry_unigraph.parallel.ctdg_peer import PeerCTDGContext

            owner = node_parts if node_parts is not None else \
                torch.arange(dataset.num_nodes, dtype=torch.long) % dctx.world_size
            peer = PeerCTDGContext(num_nodes=dataset.num_nodes, hidden_dim=hidden, slot_width=memory.slot_width,
                                   mailbox_slots=slots, grad_numel=sum(p.numel() for p in model.parameters()),
                                   owner=owner, device=torch.device(device))
            peer.attach(memory)
            if bool(c.get("historical_filter", True)):
                peer.enable_historical_filter(float(c.get("historical_alpha", 0.5)))
        elif dctx.is_distributed:
            import torch.distributed as dist

            world = dctx.world_size

            def grad_sync(flat_grad: torch.Tensor) -> float:
                dist.all_reduce(flat_grad)
                return 1.0 / world

        bmax = _engine_bmax(session_ctx, int(cfg["train"]["batch_size"]), dctx.world_size,
                            edge_parts is not None and assignment == "owner")
        engine = TGNCudaEngine(model=model, updater=updater, memory=memory, edge_feat=dataset.edge_feat,
                               neg_pool=dataset.dst_pool(), csr_provider=sampler.csr, bmax=bmax, fanout=fanout[0],
                               policy=str(sampling["strategy"]), lr=lr, dropout=float(c.get("dropout", 0.1)),
                               att_dropout=float(c.get("att_dropout", 0.1)), num_head=int(c.get("num_head", 2)),
                               seed=seed, use_graphs=bool(cfg["runtime"].get("cuda_graphs", True)),
                               grad_sync=grad_sync, peer=peer,
                               precision=str(cfg["runtime"].get("precision", "tf32")))
        optimizer = engine.opt
    else:
        # host path: torch's fused CPU Adam, one pass over all parameters instead of a loop of small ops
        optimizer = torch.optim.Adam(list(model.parameters()) + [p for p in updater.parameters() if p.requires_grad],
                                     lr=lr, fused=device == "cpu")
    if dctx.is_distributed and node_parts is not None:
        shared = torch.nonzero(node_parts != dctx.rank).view(-1).to(device)
        # the configured alpha holds either way; ada_param_enabled only lets the runtime move it
        ada = AdaParameter(alpha=float(c.get("historical_alpha", 0.5)))
        if not bool(c.get("remote_fetch", True)):
            memory.historical_cache = CTDGHistoricalCache(shared.numel(), hidden, device, dataset.num_nodes, shared,
                                                          ada)
    online = CTDGOnlineRuntime(dataset=dataset, sampler=sampler, memory=memory, model=model, optimizer=optimizer,
                               route=route, device=device, dist_ctx=dctx, memory_updater=updater, engine=engine,
                               memory_grad=bool(c.get("memory_grad", False)), seed=seed,
                               adaptive_alpha=bool(c.get("ada_param_enabled", True)))
    online.broadcast_updater_params()
    bundle = RuntimeBundle(model=model, optimizer=optimizer,
                           state={"pipeline": "ctdg_online_native", "dataset": dataset.describe(),
                                  "memory_state": memory.describe(), "route_state": route.describe(),
                                  "engine": "sm100a_fused" if engine is not None else "torch_cpu"})
    return online, bundle
