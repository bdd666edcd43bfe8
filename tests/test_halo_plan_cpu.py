"""Host-side logic of the NVLink halo path, checked on CPU: the pull plan of a
partitioned snapshot block (which source rows are pulled from other ranks, and
the aggregation columns remapped to [local rows | pulled rows]) must give the
same aggregation as indexing every source row by its global id; and the
in-place weight-gradient routing of the DTDG autograd ops."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from starry_unigraph.data.partition import NID, SnapshotBlock
from starry_unigraph.parallel.halo import PeerHaloContext


def _plan_ctx(node_parts: torch.Tensor, rank: int, world: int | None = None) -> PeerHaloContext:
    # the plan needs only the ownership maps, not the symmetric buffers
    hc = PeerHaloContext.__new__(PeerHaloContext)
    hc.device = torch.device("cpu")
    hc.rank, hc.world = rank, world or int(node_parts.max()) + 1
    local_index = torch.empty_like(node_parts)
    for q in range(hc.world):
        ids = torch.nonzero(node_parts == q).view(-1)
        local_index[ids] = torch.arange(ids.numel())
    hc.owner = node_parts.int()
    hc.local_index = local_index.int()
    hc._default_index = hc.local_index
    hc._node_parts = node_parts.long()
    hc._group = None
    hc.order_version = 0
    return hc


def _orders(parts: torch.Tensor, world: int, permuted: bool, g: torch.Generator) -> list[torch.Tensor]:
    """Each rank's current row order (global ids of its local rows)."""
    out = []
    for q in range(world):
        ids = torch.nonzero(parts == q).view(-1)
        out.append(ids[torch.randperm(ids.numel(), generator=g)] if permuted else ids)
    return out


@pytest.mark.parametrize("permuted", [False, True])
def test_pull_plan_matches_global_indexing(permuted):
    g = torch.Generator().manual_seed(3)
    n, F, world = 300, 6, 3
    parts = torch.randint(0, world, (n,), generator=g)
    x_global = torch.randn(n, F, generator=g)
    orders = _orders(parts, world, permuted, g)
    for rank in range(world):
        hc = _plan_ctx(parts, rank)
        if permuted:  # what set_row_order computes from the gathered orders
            index = hc.local_index.clone()
            for order in orders:
                index[order] = torch.arange(order.numel(), dtype=torch.int32)
            hc.local_index = index
        mine = orders[rank]
        # block: destination rows = this rank's nodes; sources = its nodes plus some
        # other ranks' nodes, in an arbitrary order (the plan must not rely on one)
        others = torch.nonzero(parts != rank).view(-1)
        halo = others[torch.randperm(others.numel(), generator=g)[:40]]
        src_nodes = torch.cat([halo[:20], mine, halo[20:]])
        m = 500
        edge_src = torch.randint(0, src_nodes.numel(), (m,), generator=g)
        edge_dst = torch.randint(0, mine.numel(), (m,), generator=g)
        block = SnapshotBlock(num_src_nodes=int(src_nodes.numel()), num_dst_nodes=int(mine.numel()),
                              edge_src=edge_src, edge_dst=edge_dst, srcdata={NID: src_nodes},
                              edata={"gcn_norm": torch.rand(m, generator=g)})
        x_local = x_global[mine]
        halo_src, col = hc.pull_plan(block, int(mine.numel()))
        owner, row = hc.src_maps(block)
        assert (owner[halo_src.long()] != rank).all()
        assert int((owner != rank).sum()) == halo_src.numel()
        # what the pull kernel gathers: row `row[c]` of owner[c]'s layer input
        pulled = torch.stack([x_global[orders[int(owner[c])]][row[c]] for c in halo_src.tolist()]) \
            if halo_src.numel() else torch.zeros(0, F)
        table = torch.cat([x_local, pulled])
        csr = block.csr()
        dst_of_edge = torch.repeat_interleave(torch.arange(block.num_dst_nodes), csr["rowptr"].diff())
        got = torch.zeros(block.num_dst_nodes, F).index_add_(0, dst_of_edge,
                                                             table[col.long()] * csr["val"][:, None])
        ref = torch.zeros(block.num_dst_nodes, F).index_add_(
            0, dst_of_edge, x_global[src_nodes[csr["col"].long()]] * csr["val"][:, None])
        torch.testing.assert_close(got, ref)
        # cached on the block for the next call, rebuilt when a row order changes
        assert hc.pull_plan(block, int(mine.numel()))[1] is col
        hc.order_version += 1
        assert hc.pull_plan(block, int(mine.numel()))[1] is not col


def _row_order_worker(rank: int, world: int, port: int, out: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(11)
        parts = torch.randint(0, world, (200,), generator=g)
        orders = _orders(parts, world, True, g)
        hc = _plan_ctx(parts, rank, world)
        default = hc.local_index.clone()
        hc.set_row_order(orders[rank] if rank == 0 else None)  # rank 1 keeps its stored order
        expect = default.clone()
        expect[orders[0]] = torch.arange(orders[0].numel(), dtype=torch.int32)
        ok = torch.equal(hc.local_index, expect) and hc.order_version == 1
        hc.set_row_order(None)  # everyone back to ascending ids
        ok = ok and torch.equal(hc.local_index, default) and hc.order_version == 2
        torch.save(ok, f"{out}/r{rank}.pt")
    finally:
        dist.destroy_process_group()


def test_set_row_order_publishes_every_ranks_order(tmp_path):
    import socket

    with socket.socket() as sock:  # a free port for the rendezvous
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    mp.spawn(_row_order_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    assert all(torch.load(tmp_path / f"r{r}.pt") for r in range(2))


def test_weight_gradients_go_to_existing_grad_in_place():
    from starry_unigraph.ops.dtdg import _grad_sink, _wgrad_buffers

    w = torch.nn.Parameter(torch.randn(4, 3))
    b = torch.nn.Parameter(torch.randn(4))
    fresh = _wgrad_buffers([w], [b])
    assert all(buf is ret for buf, ret in fresh)           # no .grad yet: fresh buffers are returned
    w.grad = torch.zeros_like(w)
    b.grad = torch.zeros_like(b)
    sink = _wgrad_buffers([w], [b])
    assert sink[0][0] is w.grad and sink[1][0] is b.grad    # kernels add into .grad ...
    assert sink[0][1] is None and sink[1][1] is None        # ... and autograd gets None
    assert _grad_sink(w.detach() * 2) is None               # computed weights get a returned gradient


def test_halo_width_of_the_flare_models():
    from starry_unigraph.backends.dtdg.runtime.models import build_flare_model
    from starry_unigraph.parallel.halo import halo_width

    assert halo_width(build_flare_model("tgcn", 128, 128, 2), 128) == 384      # GCN stack of 3 x hidden
    assert halo_width(build_flare_model("mpnn_lstm", 64, 64, 1), 64) == 64
    assert halo_width(build_flare_model("evolvegcn", 128, 128, 2), 128) == 128  # no stack: the default



def test_spmm_item_plan_covers_every_edge_once():
    """The item plan of the 64-feature aggregation kernel, built on CPU tensors:
    every row's edges are covered by its items exactly once and in order, a row
    without edges is one empty item, rows longer than the item size are split
    (and flagged, and listed for zeroing), and the warp offsets partition the
    items with roughly equal edge counts."""
    from starry_unigraph.data.partition import spmm_plan

    g = torch.Generator().manual_seed(5)
    deg = torch.randint(0, 6, (500,), generator=g)
    deg[7], deg[100], deg[101] = 1000, 0, 129
    rowptr = torch.zeros(501, dtype=torch.long)
    rowptr[1:] = deg.cumsum(0)
    max_edges, warps = 64, 13
    items, woff, split = spmm_plan(rowptr, max_edges, warps)
    it = items.view(3, -1).long()
    renc, e0, e1 = it[0], it[1], it[2]
    row = torch.where(renc >= 0, renc, -renc - 1)
    assert bool((e1 - e0 <= max_edges).all()) and bool((e1 >= e0).all())
    covered = torch.zeros(int(rowptr[-1]), dtype=torch.long)
    for r, a, b in zip(row.tolist(), e0.tolist(), e1.tolist()):
        assert int(rowptr[r]) <= a <= b <= int(rowptr[r + 1])
        covered[a:b] += 1
    assert bool((covered == 1).all())
    per_row = torch.bincount(row, minlength=500)
    assert bool((per_row >= 1).all())                       # empty rows have their zero item
    assert int(per_row[100]) == 1 and int((e1 - e0)[row == 100].sum()) == 0
    assert sorted(split.tolist()) == [7, 101]               # 1000 and 129 edges > 64
    assert bool((renc[row == 7] < 0).all()) and bool((renc[row == 3] >= 0).all())
    assert woff.numel() == warps + 1 and int(woff[0]) == 0 and int(woff[-1]) == it.size(1)
    assert bool((woff[1:] >= woff[:-1]).all())
