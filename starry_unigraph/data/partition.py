"""Partitioned snapshot containers for distributed DTDG training
(reference data/partition.py:43-589), without DGL.

* ``TensorData``: N variable-length tensors packed into one tensor + pointers.
* ``RouteData``: per-snapshot send/recv sizes and packed send indices.
* ``PartitionData``: one partition's snapshots (local dst ids, remote src ids,
  edge topology, node/edge feature dicts, routes); slicing, ``to``,
  ``pin_memory``, ``save``/``load``, ``to_blocks``/``from_blocks``.
* ``SnapshotBlock``: the bipartite message-flow block of one snapshot — source
  rows are ``[local dst nodes ; remote halo nodes]``, destination rows the local
  nodes, edges in COO with lazily built destination- and source-sorted CSR used
  by the aggregation kernels.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch
from torch import Tensor

NID = "_ID"
EID = "_ID"


@dataclass
class TensorData:
    ptr: list[int]
    data: Tensor

    def __post_init__(self) -> None:
        if not self.ptr:
            raise ValueError("ptr must not be empty")
        if self.ptr[-1] != int(self.data.size(0)):
            raise ValueError(f"ptr[-1] != data.size(0): {self.ptr[-1]} != {self.data.size(0)}")

    def __len__(self) -> int:
        return len(self.ptr) - 1

    def __getitem__(self, index: int | slice) -> "TensorData":
        if not isinstance(index, slice):
            if index < 0:
                index += len(self)
            index = slice(index, index + 1)
        if index.step not in (None, 1):
            raise ValueError("Only step size of 1 is supported")
        start = 0 if index.start is None else index.start
        stop = len(self) if index.stop is None else index.stop
        a, b = self.ptr[start], self.ptr[stop]
        return type(self)(ptr=[v - a for v in self.ptr[start:stop + 1]], data=self.data[a:b])

    def item(self) -> Tensor:
        items = self.to_tensors()
        if len(items) != 1:
            raise ValueError(f"Expected 1 tensor, got {len(items)}")
        return items[0]

    def to_tensors(self) -> list[Tensor]:
        return [self.data[self.ptr[i]:self.ptr[i + 1]] for i in range(len(self))]

    def pin_memory(self, device: str | None = None) -> "TensorData":
        return type(self)(ptr=self.ptr, data=self.data.pin_memory())

    def to(self, device=None, dtype=None, non_blocking: bool = False, copy: bool = False) -> "TensorData":
        data = self.data
        if dtype is not None and data.is_floating_point():
            data = data.to(dtype=dtype)
        return type(self)(ptr=self.ptr, data=data.to(device=device, non_blocking=non_blocking, copy=copy))

    @classmethod
    def from_tensors(cls, tensors: list[Tensor]) -> "TensorData":
        if not tensors:
            raise ValueError("tensors must not be empty")
        ptr = [0]
        for t in tensors:
            ptr.append(ptr[-1] + int(t.size(0)))
        return cls(ptr=ptr, data=torch.cat(tensors, dim=0))


@dataclass
class RouteData:
    send_sizes: list[list[int]]
    recv_sizes: list[list[int]]
    send_index_ind: Tensor | None = None
    send_index_ptr: list[int] | None = None

    def __len__(self) -> int:
        return len(self.send_sizes)

    def __getitem__(self, index: int | slice) -> "RouteData":
        if not isinstance(index, slice):
            if index < 0:
                index += len(self)
            index = slice(index, index + 1)
        start = 0 if index.start is None else index.start
        stop = len(self) if index.stop is None else index.stop
        ind = ptr = None
        if self.send_index_ind is not None and self.send_index_ptr is not None:
            a, b = self.send_index_ptr[start], self.send_index_ptr[stop]
            ind = self.send_index_ind[a:b]
            ptr = [v - a for v in self.send_index_ptr[start:stop + 1]]
        return type(self)(self.send_sizes[start:stop], self.recv_sizes[start:stop], ind, ptr)

    def item(self):
        from starry_unigraph.backends.dtdg.runtime.route import Route

        if len(self) != 1:
            raise ValueError(f"Expected 1 route, got {len(self)}")
        return Route(send_sizes=list(self.send_sizes[0]), recv_sizes=list(self.recv_sizes[0]),
                     send_index=self.send_index_ind)

    def to(self, device=None, dtype=None, non_blocking: bool = False, copy: bool = False) -> "RouteData":
        ind = None if self.send_index_ind is None else self.send_index_ind.to(device=device, non_blocking=non_blocking)
        return type(self)(self.send_sizes, self.recv_sizes, ind, self.send_index_ptr)

    def pin_memory(self, device: str | None = None) -> "RouteData":
        ind = None if self.send_index_ind is None else self.send_index_ind.pin_memory()
        return type(self)(self.send_sizes, self.recv_sizes, ind, self.send_index_ptr)

    @classmethod
    def from_routes(cls, routes: list[Any]) -> "RouteData":
        send = [list(map(int, r.send_sizes)) for r in routes]
        recv = [list(map(int, r.recv_sizes)) for r in routes]
        if any(r.send_index is None for r in routes):
            return cls(send, recv, None, None)
        td = TensorData.from_tensors([r.send_index.long() for r in routes])
        return cls(send, recv, td.data, td.ptr)


def spmm_plan(rowptr: Tensor, max_edges: int = 128, warps: int | None = None) -> list[Tensor]:
    """Work plan of the item-based aggregation kernel over a CSR (device tensors):
    every row cut into items of at most `max_edges` edges (a row without edges is
    one empty item, which writes its zero row), items handed to the warps of a
    fixed grid in runs of about equal edge count (8 edges of overhead per item).
    Returns [items (row or -row-1 for rows split over several items, first edge,
    end edge; int32, 3 x n_items), warp offsets (int32, warps + 1), split rows
    (int32)]."""
    from starry_unigraph.ops import cuda_ext

    dev = rowptr.device
    if warps is None:
        warps = int(cuda_ext().spmm_plan_warps())
    n = rowptr.numel() - 1
    deg = rowptr[1:] - rowptr[:-1]
    k = torch.clamp((deg + max_edges - 1) // max_edges, min=1)
    row = torch.repeat_interleave(torch.arange(n, device=dev), k)
    n_items = int(row.numel())
    first = torch.cumsum(k, 0) - k
    j = torch.arange(n_items, device=dev) - first[row]
    e0 = rowptr[row] + j * max_edges
    e1 = torch.minimum(e0 + max_edges, rowptr[row + 1])
    split = k > 1
    renc = torch.where(split[row], -row - 1, row)
    cw = torch.cumsum(e1 - e0 + 8, 0)
    targets = torch.arange(1, warps, device=dev, dtype=torch.int64) * int(cw[-1]) // warps
    bounds = torch.searchsorted(cw, targets, right=True)
    woff = torch.cat([torch.zeros(1, dtype=torch.int64, device=dev), bounds,
                      torch.full((1,), n_items, dtype=torch.int64, device=dev)])
    items = torch.stack([renc, e0, e1]).int().contiguous().view(-1)
    return [items, woff.int().contiguous(), torch.nonzero(split).view(-1).int().contiguous()]


@dataclass
class SnapshotBlock:
    """Bipartite block of one snapshot on one partition."""

    num_src_nodes: int
    num_dst_nodes: int
    edge_src: Tensor   # [E] index into source rows
    edge_dst: Tensor   # [E] index into destination rows
    srcdata: dict[str, Tensor] = field(default_factory=dict)
    dstdata: dict[str, Tensor] = field(default_factory=dict)
    edata: dict[str, Tensor] = field(default_factory=dict)
    route: Any = None
    is_block: bool = True
    graph_meta: dict[str, Any] = field(default_factory=dict)
    _csr: dict[str, Tensor] | None = field(default=None, repr=False)

    def num_edges(self) -> int:
        return int(self.edge_src.numel())

    def num_nodes(self) -> int:
        return self.num_dst_nodes

    def edges(self) -> tuple[Tensor, Tensor]:
        return self.edge_src, self.edge_dst

    @property
    def device(self) -> torch.device:
        return self.edge_src.device

    def edge_norm(self) -> Tensor:
        """gcn_norm if precomputed, else w / max(1, sum of incoming w) (reference _gcn_norm)."""
        if "gcn_norm" in self.edata:
            return self.edata["gcn_norm"].float().view(-1)
        w = self.edata["w"].float().view(-1) if "w" in self.edata else \
            torch.ones(self.num_edges(), device=self.device)
        deg = torch.zeros(self.num_dst_nodes, device=self.device).index_add_(0, self.edge_dst.long(), w)
        return w / deg.clamp_min(1.0)[self.edge_dst.long()]

    def csr(self) -> dict[str, Tensor]:
        """Destination-sorted CSR (forward aggregation) and source-sorted CSR
        (backward aggregation), both with int32 columns and fp32 values; on the
        GPU also the item plans of the 64-feature aggregation kernel for both
        ("plan", "plan_t", see ``spmm_plan``)."""
        if self._csr is None:
            dst = self.edge_dst.long()
            src = self.edge_src.long()
            val = self.edge_norm()
            order = torch.argsort(dst, stable=True)
            rowptr = torch.zeros(self.num_dst_nodes + 1, dtype=torch.int64, device=dst.device)
            rowptr[1:] = torch.cumsum(torch.bincount(dst, minlength=self.num_dst_nodes), 0)
            order_t = torch.argsort(src, stable=True)
            rowptr_t = torch.zeros(self.num_src_nodes + 1, dtype=torch.int64, device=dst.device)
            rowptr_t[1:] = torch.cumsum(torch.bincount(src, minlength=self.num_src_nodes), 0)
            self._csr = {"rowptr": rowptr, "col": src[order].int().contiguous(), "val": val[order].contiguous(),
                         "rowptr_t": rowptr_t, "col_t": dst[order_t].int().contiguous(),
                         "val_t": val[order_t].contiguous()}
            if rowptr.is_cuda and int(rowptr[-1]) < 2 ** 31:
                self._csr["plan"] = spmm_plan(rowptr)
                self._csr["plan_t"] = spmm_plan(rowptr_t)
        return self._csr

    def local_scope(self):
        import contextlib

        return contextlib.nullcontext()


@dataclass
class PartitionData:
    src_ids: TensorData
    dst_ids: TensorData
    edge_ids: TensorData
    edge_src: TensorData
    edge_dst: TensorData
    node_data: dict[str, TensorData] = field(default_factory=dict)
    edge_data: dict[str, TensorData] = field(default_factory=dict)
    routes: RouteData | None = None

    def __post_init__(self) -> None:
        n = len(self.dst_ids)
        for name in ("src_ids", "edge_ids", "edge_src", "edge_dst"):
            if len(getattr(self, name)) != n:
                raise ValueError(f"Expected {n} entries for {name}")
        for kind, d in (("node_data", self.node_data), ("edge_data", self.edge_data)):
            for k, v in d.items():
                if len(v) != n:
                    raise ValueError(f"Expected {n} entries for {kind}[{k}], got {len(v)}")
        if self.routes is not None and len(self.routes) != n:
            raise ValueError(f"Expected {n} entries for routes, got {len(self.routes)}")

    def __len__(self) -> int:
        return len(self.dst_ids)

    def __getitem__(self, index: int | slice) -> "PartitionData":
        return type(self)(self.src_ids[index], self.dst_ids[index], self.edge_ids[index], self.edge_src[index],
                          self.edge_dst[index], {k: v[index] for k, v in self.node_data.items()},
                          {k: v[index] for k, v in self.edge_data.items()},
                          None if self.routes is None else self.routes[index])

    @property
    def num_snaps(self) -> int:
        return len(self)

    @property
    def num_dst_nodes(self) -> int:
        return int(self.dst_ids[0].item().numel())

    def add_ndata(self, key: str, data: TensorData) -> None:
        if len(data) != len(self):
            raise ValueError(f"Expected {len(self)} entries for node_data[{key}], got {len(data)}")
        self.node_data[key] = data

    def pop_ndata(self, key: str) -> TensorData | None:
        return self.node_data.pop(key, None)

    def add_edata(self, key: str, data: TensorData) -> None:
        if len(data) != len(self):
            raise ValueError(f"Expected {len(self)} entries for edge_data[{key}], got {len(data)}")
        self.edge_data[key] = data

    def _map(self, fn) -> "PartitionData":
        return type(self)(fn(self.src_ids), fn(self.dst_ids), fn(self.edge_ids), fn(self.edge_src), fn(self.edge_dst),
                          {k: fn(v) for k, v in self.node_data.items()}, {k: fn(v) for k, v in self.edge_data.items()},
                          None if self.routes is None else fn(self.routes))

    def to(self, device=None, dtype=None, non_blocking: bool = False, copy: bool = False) -> "PartitionData":
        return self._map(lambda t: t.to(device=device, dtype=dtype, non_blocking=non_blocking, copy=copy))

    def pin_memory(self, device: str | None = None) -> "PartitionData":
        return self._map(lambda t: t.pin_memory())

    def to_blocks(self, node_perm: Tensor | None = None, keep_ids: bool = False) -> list[SnapshotBlock]:
        from starry_unigraph.backends.dtdg.runtime.route import Route

        blocks = []
        for i in range(len(self)):
            orig_dst = self.dst_ids[i].item()
            dst_ids = orig_dst
            suffix = self.src_ids[i].item()
            src = self.edge_src[i].item().long()
            dst = self.edge_dst[i].item().long()
            n_dst = int(dst_ids.numel())
            if node_perm is not None:
                if int(node_perm.numel()) != n_dst:
                    raise ValueError(f"Expected node_perm size {n_dst}, got {node_perm.numel()}")
                imap = torch.empty_like(node_perm)
                imap[node_perm] = torch.arange(node_perm.numel(), dtype=node_perm.dtype, device=node_perm.device)
                dst = imap[dst]
                inner = src < n_dst
                src = src.clone()
                src[inner] = imap[src[inner]]
                dst_ids = dst_ids[node_perm]
            src_ids = torch.cat([dst_ids, suffix])
            blk = SnapshotBlock(num_src_nodes=int(src_ids.numel()), num_dst_nodes=n_dst, edge_src=src, edge_dst=dst)
            if keep_ids:
                blk.srcdata[NID] = src_ids
                blk.dstdata[NID] = dst_ids
                blk.edata[EID] = self.edge_ids[i].item()
            for k, v in self.node_data.items():
                it = v[i].item()
                if it.size(0) == src_ids.size(0) and src_ids.size(0) != n_dst:
                    if node_perm is not None:
                        it = torch.cat([it[:n_dst][node_perm], it[n_dst:]])
                    blk.srcdata[k] = it
                elif it.size(0) == n_dst:
                    blk.dstdata[k] = it[node_perm] if node_perm is not None else it
                elif it.size(0) == src_ids.size(0):
                    blk.srcdata[k] = it
                else:
                    raise ValueError(f"Unexpected node_data[{k}] size: {tuple(it.size())}")
            for k, v in self.edge_data.items():
                blk.edata[k] = v[i].item()
            if self.routes is not None:
                route = self.routes[i].item()
                if node_perm is not None and route.send_index is not None:
                    remap = torch.empty_like(node_perm)
                    remap[node_perm] = torch.arange(node_perm.numel(), dtype=node_perm.dtype, device=node_perm.device)
                    send = route.send_index.clone()
                    local = send < n_dst
                    send[local] = remap[send[local]].to(send.dtype)
                    route = Route(send_sizes=route.send_sizes, recv_sizes=route.recv_sizes, send_index=send,
                                  group=route.group)
                blk.route = route
            blocks.append(blk)
        return blocks

    def item(self, node_perm: Tensor | None = None, keep_ids: bool = False) -> SnapshotBlock:
        blocks = self.to_blocks(node_perm=node_perm, keep_ids=keep_ids)
        if len(blocks) != 1:
            raise ValueError(f"Expected 1 block, got {len(blocks)}")
        return blocks[0]

    def save(self, path: str | Path) -> None:
        path = Path(path).expanduser().resolve()
        path.parent.mkdir(parents=True, exist_ok=True)
        torch.save(self, path)

    @classmethod
    def load(cls, path: str | Path, mmap: bool = False) -> "PartitionData":
        obj = torch.load(Path(path).expanduser().resolve(), mmap=mmap, weights_only=False)
        if not isinstance(obj, cls):
            raise TypeError(f"Expected {cls.__name__}, got {type(obj).__name__}")
        return obj

    @classmethod
    def from_blocks(cls, blocks: list[SnapshotBlock]) -> "PartitionData":
        src_ids, dst_ids, edge_ids, esrc, edst = [], [], [], [], []
        snd: dict[str, list[Tensor]] = {}
        dnd: dict[str, list[Tensor]] = {}
        ed: dict[str, list[Tensor]] = {}
        routes = []
        for b in blocks:
            s_id = b.srcdata.get(NID, torch.arange(b.num_src_nodes))
            d_id = b.dstdata.get(NID, torch.arange(b.num_dst_nodes))
            e_id = b.edata.get(EID, torch.arange(b.num_edges()))
            if torch.any(s_id[:d_id.numel()] != d_id):
                raise ValueError("prefix of src_ids and dst_ids must be the same")
            src_ids.append(s_id[d_id.numel():])
            dst_ids.append(d_id)
            edge_ids.append(e_id)
            esrc.append(b.edge_src)
            edst.append(b.edge_dst)
            for k, v in b.srcdata.items():
                if k != NID:
                    snd.setdefault(k, []).append(v)
            for k, v in b.dstdata.items():
                if k != NID:
                    dnd.setdefault(k, []).append(v)
            for k, v in b.edata.items():
                if k != EID:
                    ed.setdefault(k, []).append(v)
            if b.route is not None:
                routes.append(b.route)
        nd = {k: TensorData.from_tensors(v) for k, v in dnd.items() if len(v) == len(blocks)}
        nd.update({k: TensorData.from_tensors(v) for k, v in snd.items() if len(v) == len(blocks)})
        return cls(TensorData.from_tensors(src_ids), TensorData.from_tensors(dst_ids),
                   TensorData.from_tensors(edge_ids), TensorData.from_tensors(esrc), TensorData.from_tensors(edst),
                   nd, {k: TensorData.from_tensors(v) for k, v in ed.items() if len(v) == len(blocks)},
                   RouteData.from_routes(routes) if len(routes) == len(blocks) else None)
