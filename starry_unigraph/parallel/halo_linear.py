"""A GCN layer whose dense GEMM publishes the halo rows (reference: one layer of
runtime/modules/gcn_layers.py:62-94, Route.forward all_to_all, then DGL SpMM,
then Linear(bias=False); backends/dtdg/runtime/route.py:297-322).

The layer's GEMM runs first: A (H W^T) equals (A H) W^T for a bias-free linear
map, and the activation follows the aggregation either way. The tcgen05 GEMM's
epilogue stores Z = H W^T straight into this rank's rows of the symmetric
staging buffer, the buffer the peers pull halo rows from, so no separate copy
publishes the layer's rows; after one bounded device barrier each halo row of
the block is pulled once from its owner over NVLink and the aggregation runs
over [local rows of Z in the staging buffer | pulled rows]. The exchanged rows
are the layer's output width.

Backward: the transposed aggregation pushes each source row's gradient into its
owner's gradient buffer (remote atomic adds), a barrier, then this rank's dZ
rows feed the GEMM's data and weight gradients (the weight gradient is added in
place into the parameter's gradient view, as the other DTDG ops do).
"""
from __future__ import annotations

import torch
import torch.autograd as autograd

from starry_unigraph.parallel.halo import PeerHaloContext


class _HaloLinearAggregate(autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor, graph, hc: PeerHaloContext):
        C = hc._C
        buf = f"x{hc.fwd_calls % 2}"
        hc.fwd_calls += 1
        n_local, F = x.size(0), w.size(0)
        z = hc.arena[buf][:n_local, :F]  # this rank's staging rows, row stride hc.F
        C.linear_fwd_into(x, w.contiguous(), None, 0, z)  # GEMM epilogue publishes the rows
        hc.barrier()
        csr = graph.csr()
        owner, row = hc.src_maps(graph)
        halo_src, col = hc.pull_plan(graph, n_local)
        halo = C.halo_pull(hc.tables[buf], owner, row, halo_src, F, hc.F)
        out = C.spmm_two_tables(csr["rowptr"], col, csr["val"], z, halo, graph.num_dst_nodes, csr.get("plan"))
        ctx.hc, ctx.graph, ctx.n_local, ctx.w_ref = hc, graph, n_local, w
        ctx.save_for_backward(x, w, owner, row)
        return out

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        from starry_unigraph.ops.dtdg import _grad_sink

        hc = ctx.hc
        C = hc._C
        x, w, owner, row = ctx.saved_tensors
        buf = f"g{hc.bwd_calls % 2}"
        hc.bwd_calls += 1
        csr = ctx.graph.csr()
        F = grad.size(1)
        C.spmm_peer_push(csr["rowptr_t"], csr["col_t"], csr["val_t"], grad.contiguous(), ctx.graph.num_src_nodes,
                         hc.tables[buf], owner, row, hc.F, csr.get("plan_t"))
        hc.barrier()
        g = hc.arena[buf]
        gz = g[: ctx.n_local, :F]  # read in place by both GEMMs (row stride hc.F), no copy
        gx = C.linear_dgrad(gz, w.contiguous()) if ctx.needs_input_grad[0] else None
        gw = None
        if ctx.needs_input_grad[1]:
            sink = _grad_sink(ctx.w_ref)
            target = sink if sink is not None else torch.zeros_like(w)
            C.linear_wgrad(gz, x.contiguous(), target, None, None)
            gw = None if sink is not None else target
        gz.zero_()  # after both GEMMs (same stream): ready for its next use, two calls later
        return gx, gw, None, None


def halo_linear_aggregate(graph, x: torch.Tensor, weight: torch.Tensor, hc: PeerHaloContext) -> torch.Tensor:
    """A x W^T aggregated over the block, halo rows of x W^T pulled from the peers."""
    return _HaloLinearAggregate.apply(x.float().contiguous(), weight, graph, hc)
