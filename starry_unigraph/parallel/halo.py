"""DTDG halo exchange fused into the neighbour aggregation over NVLink
(reference: Route.forward = all_to_all of boundary rows, then DGL SpMM,
backends/dtdg/runtime/route.py:297-322, runtime/modules/gcn_layers.py:62-94).

Every rank copies its layer input rows into a symmetric staging buffer; after a
bounded device barrier one kernel pulls each halo row of the block once from
its owner's buffer over NVLink (P2P loads, no collective), and the aggregation
reads local rows from the layer input and halo rows from the pulled copy, with
the block's columns remapped once to [local rows | halo rows]. (Reading every
halo edge's source row straight from the owner inside the aggregation, the
other form kept in `spmm_peer_gather`, moves each halo row once per edge
instead of once: on a degree-10 graph about five times the NVLink bytes.)
Backward runs the transposed aggregation and pushes each source row's gradient
into the owner's gradient buffer with remote atomic adds (one push per source
row); after a barrier each rank takes its rows out.

Staging and gradient buffers alternate between two copies, so a rank may start
writing call k+1 while a slower peer still reads call k: a buffer is reused
two calls later, after a barrier that every peer passes only once it finished
reading it. Buffers are as wide as the widest exchanging layer; a narrower layer
uses the first columns of each row (the kernels take the row stride), so any
width up to that one (a multiple of 4) takes this path.

Row order: a partition's rows follow ascending node id unless the training
loader permutes them (chunk order with temporal decay); ``set_row_order``
publishes every rank's current order (one all-gather) so peers address the
owner's rows where they are.
"""
from __future__ import annotations

import torch
import torch.autograd as autograd
import torch.distributed as dist

from starry_unigraph.data.partition import NID
from starry_unigraph.ops import cuda_ext
from starry_unigraph.parallel.ctdg_peer import DEFAULT_BARRIER_BUDGET
from starry_unigraph.parallel.symmetric import SymmetricArena


class PeerHaloContext:
    def __init__(self, node_parts: torch.Tensor, features: int, device: torch.device,
                 group: dist.ProcessGroup | None = None, barrier_budget: int = DEFAULT_BARRIER_BUDGET):
        self.device = torch.device(device)
        node_parts = node_parts.long().cpu()
        world = dist.get_world_size(group)
        counts = torch.bincount(node_parts, minlength=world)
        max_rows = int(counts.max()) if counts.numel() else 1
        self.F = int(features)
        specs = {f"x{i}": ((max_rows, self.F), torch.float32) for i in range(2)}
        specs.update({f"g{i}": ((max_rows, self.F), torch.float32) for i in range(2)})
        specs["flags"] = ((32,), torch.int64)
        self.arena = SymmetricArena(specs, self.device, group)
        self.rank, self.world = self.arena.rank, self.arena.world_size
        for n in ("x0", "x1", "g0", "g1", "flags"):
            self.arena[n].zero_()
        self.tables = {n: self.arena.peer_table(n) for n in specs}
        # owner and row-in-owner of every global node (rows of a partition follow ascending node id)
        local_index = torch.empty_like(node_parts)
        for q in range(world):
            ids = torch.nonzero(node_parts == q).view(-1)
            local_index[ids] = torch.arange(ids.numel())
        self.owner = node_parts.to(self.device, torch.int32)
        self.local_index = local_index.to(self.device, torch.int32)
        self._default_index = self.local_index
        self._node_parts = node_parts
        self.order_version = 0  # bumped whenever a rank's row order changes (invalidates pull plans)
        self._group = group
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.budget = int(barrier_budget)
        self.fwd_calls = 0
        self.bwd_calls = 0
        self._C = cuda_ext()
        torch.cuda.synchronize(self.device)
        self.arena.barrier_host()

    def barrier(self) -> None:
        self._C.peer_barrier(self.tables["flags"], self.rank, self.world, self.epoch, self.budget)

    def supports(self, width: int) -> bool:
        """Layer widths this context exchanges over NVLink."""
        return width == self.F or (width <= self.F and width % 4 == 0)

    def set_row_order(self, local_ids: torch.Tensor | None) -> None:
        """Collective: this rank's local rows are the global nodes `local_ids` in
        this order (None: ascending node id, the partition's stored order). Every
        rank calls it with its own order; afterwards `local_index[gid]` is the
        row of gid in its owner's current order."""
        counts = torch.bincount(self._node_parts, minlength=self.world)
        rows = int(counts.max())
        mine = torch.full((rows,), -1, dtype=torch.int64, device=self.device)
        if local_ids is not None:
            ids = local_ids.to(self.device, torch.int64).view(-1)
            if ids.numel() != int(counts[self.rank]):
                raise ValueError(f"row order of {ids.numel()} nodes for a partition of {int(counts[self.rank])}")
            mine[: ids.numel()] = ids
        flag = torch.tensor([0 if local_ids is None else 1], dtype=torch.int64, device=self.device)
        flags = [torch.zeros_like(flag) for _ in range(self.world)]
        dist.all_gather(flags, flag, group=self._group)
        if not any(int(f) for f in flags):
            if self.local_index is not self._default_index:
                self.local_index = self._default_index
                self.order_version += 1
            return
        orders = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(orders, mine, group=self._group)
        index = self._default_index.clone()
        for order in orders:
            valid = order >= 0
            index[order[valid]] = torch.arange(int(valid.sum()), dtype=torch.int32, device=self.device)
        self.local_index = index
        self.order_version += 1

    def src_maps(self, graph) -> tuple[torch.Tensor, torch.Tensor]:
        gid = graph.srcdata[NID].to(self.device).long()
        return self.owner[gid].contiguous(), self.local_index[gid].contiguous()

    def pull_plan(self, graph, n_local: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(halo_src, col): the block's source rows owned by other ranks (pulled
        once per call, in this order) and the aggregation columns remapped to
        [row of a local source in the layer input | n_local + pull slot].
        Cached on the block."""
        key = ("_halo_pull", self.rank, self.world, int(n_local), self.order_version)
        meta = graph.graph_meta
        if meta.get("_halo_pull_key") != key:
            owner, row = self.src_maps(graph)
            remote = owner != self.rank
            halo_src = torch.nonzero(remote).view(-1).int()
            slot = torch.cumsum(remote.int(), 0) - 1
            remap = torch.where(remote, n_local + slot, row.long())
            col = remap[graph.csr()["col"].long()].int().contiguous()
            meta["_halo_pull_key"] = key
            meta["_halo_pull"] = (halo_src, col)
        return meta["_halo_pull"]


class _HaloAggregate(autograd.Function):
    @staticmethod
    def forward(ctx, x_local: torch.Tensor, graph, hc: PeerHaloContext):
        C = hc._C
        buf = f"x{hc.fwd_calls % 2}"
        hc.fwd_calls += 1
        n_local, F = x_local.shape
        if not hc.supports(F):
            raise ValueError(f"halo staging rows hold {hc.F} features; layer width {F} is not exchanged here")
        stage = hc.arena[buf]
        stage[:n_local, :F].copy_(x_local)  # rows at the staging stride hc.F
        hc.barrier()
        csr = graph.csr()
        owner, row = hc.src_maps(graph)
        if F % 4 == 0:
            halo_src, col = hc.pull_plan(graph, n_local)
            halo = C.halo_pull(hc.tables[buf], owner, row, halo_src, F, hc.F)
            out = C.spmm_two_tables(csr["rowptr"], col, csr["val"], x_local, halo, graph.num_dst_nodes,
                                    csr.get("plan"))
        else:  # F == hc.F (supports): per-edge peer reads at the staging stride
            out = C.spmm_peer_gather(csr["rowptr"], csr["col"], csr["val"], hc.tables[buf], owner, row,
                                     graph.num_dst_nodes, F)
        ctx.hc, ctx.graph, ctx.n_local = hc, graph, n_local
        ctx.save_for_backward(owner, row)
        return out

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        hc = ctx.hc
        C = hc._C
        owner, row = ctx.saved_tensors
        buf = f"g{hc.bwd_calls % 2}"
        hc.bwd_calls += 1
        csr = ctx.graph.csr()
        F = grad.size(1)
        C.spmm_peer_push(csr["rowptr_t"], csr["col_t"], csr["val_t"], grad.contiguous(), ctx.graph.num_src_nodes,
                         hc.tables[buf], owner, row, hc.F, csr.get("plan_t"))
        hc.barrier()
        g = hc.arena[buf]
        gx = g[: ctx.n_local, :F].clone()
        g[: ctx.n_local, :F].zero_()  # ready for its next use, two calls later
        return gx, None, None


def halo_width(model, default: int) -> int:
    """Feature width of the rows that exchange halo rows: the outputs of a GCN
    stack's second and later layers, which run their linear map before the
    exchange (the first layer aggregates the block's stored source features and
    exchanges nothing). T-GCN's stack is 3 x hidden wide, MPNN-LSTM's hidden."""
    from starry_unigraph.runtime.modules.gcn_layers import GCNStack

    widths = [int(layer.weight.shape[0]) for m in model.modules() if isinstance(m, GCNStack)
              for layer in list(m.layers)[1:]]
    return max(widths) if widths else int(default)


_CONTEXT: dict[str, PeerHaloContext | None] = {"ctx": None}


def set_halo_context(hc: PeerHaloContext | None) -> None:
    _CONTEXT["ctx"] = hc


def get_halo_context() -> PeerHaloContext | None:
    return _CONTEXT["ctx"]


def halo_aggregate(graph, x_local: torch.Tensor) -> torch.Tensor:
    """Normalised neighbour sum of `graph` whose halo source rows come from the
    peers' staging buffers (requires an active PeerHaloContext)."""
    hc = _CONTEXT["ctx"]
    if hc is None:
        raise RuntimeError("no PeerHaloContext is active")
    return _HaloAggregate.apply(x_local.float().contiguous(), graph, hc)
