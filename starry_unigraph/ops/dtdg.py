"""Autograd wrappers of the DTDG sm_100a kernels.

* ``gcn_aggregate(block, x)``: normalised neighbour sum over the block's CSR
  (forward over the destination-sorted CSR, backward over the source-sorted
  one — no atomics).
* ``linear(x, w, b, act)``: tcgen05 GEMM forward, data and weight gradients.
* ``lstm_cell(x, state, cell)``: fused LSTM cell (one GEMM over [x || h] with a
  gate epilogue) with a fused backward.

On CPU tensors the same functions run the PyTorch reference math.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from starry_unigraph.ops import cuda_ext


class _SpMM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_src, csr, n_dst):
        C = cuda_ext()
        ctx.csr = csr  # CSR and item plans of the block (cached on it)
        ctx.n_src = x_src.size(0)
        return C.spmm_csr(csr["rowptr"], csr["col"], csr["val"], x_src.contiguous(), int(n_dst), None, False,
                          csr.get("plan"))

    @staticmethod
    def backward(ctx, g):
        c = ctx.csr
        gx = cuda_ext().spmm_csr(c["rowptr_t"], c["col_t"], c["val_t"], g.contiguous(), int(ctx.n_src), None, False,
                                 c.get("plan_t"))
        return gx, None, None


def gcn_aggregate(block, x_src: torch.Tensor) -> torch.Tensor:
    if x_src.is_cuda:
        return _SpMM.apply(x_src.float(), block.csr(), block.num_dst_nodes)
    norm = block.edge_norm()
    out = torch.zeros(block.num_dst_nodes, x_src.size(1), dtype=x_src.dtype, device=x_src.device)
    return out.index_add(0, block.edge_dst.long(), x_src[block.edge_src.long()] * norm.unsqueeze(1))


def _grad_sink(t: torch.Tensor | None) -> torch.Tensor | None:
    """The parameter's own .grad when the weight-gradient kernels may add into it
    in place: a leaf parameter whose gradient already exists (the flat gradient
    buffer's views). The backward then returns None for it, so autograd runs no
    zero-fill and no accumulation kernel. Otherwise None (a fresh buffer is
    returned as usual)."""
    if t is not None and t.is_leaf and t.requires_grad and t.grad is not None and t.grad.is_contiguous() \
            and t.grad.dtype == torch.float32:
        return t.grad
    return None


def _wgrad_buffers(ws, bs):
    """Per weight, then per bias: (buffer the kernel accumulates into, value the
    backward returns for it)."""
    out = []
    for t in list(ws) + list(bs):
        sink = _grad_sink(t)
        if sink is not None:
            out.append((sink, None))
        else:
            z = torch.zeros_like(t, dtype=torch.float32)
            out.append((z, z))
    return out


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, act):
        y = cuda_ext().linear_fwd(x.contiguous(), w.contiguous(), b, int(act))
        ctx.act = int(act)
        ctx.has_b = b is not None
        ctx.w_ref, ctx.b_ref = w, b  # parameters: their .grad may take the gradient in place
        ctx.save_for_backward(x, w, y if act else None)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w, y = ctx.saved_tensors
        C = cuda_ext()
        if gy.stride(-1) != 1:  # the GEMM producers read any row stride
            gy = gy.contiguous()
        mask = None
        if ctx.act == 1:
            mask = y  # ReLU derivative applied while the GEMMs pack dY
        elif ctx.act == 2:
            gy = gy * y * (1 - y)
        elif ctx.act == 3:
            gy = gy * (1 - y * y)
        gx = C.linear_dgrad(gy, w.contiguous(), mask) if ctx.needs_input_grad[0] else None
        sw = _grad_sink(ctx.w_ref)
        gw = sw if sw is not None else torch.zeros_like(w)
        gb, sb = None, None
        if ctx.has_b:
            sb = _grad_sink(ctx.b_ref)
            gb = sb if sb is not None else torch.zeros(w.size(0), device=w.device)
        C.linear_wgrad(gy, x.contiguous(), gw, gb, mask)
        return gx, (None if sw is not None else gw), (None if sb is not None else gb), None


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None, act: int = 0) -> torch.Tensor:
    if x.is_cuda and x.dtype == torch.float32:
        return _Linear.apply(x, w, b, act)
    y = F.linear(x, w, b)
    return {0: y, 1: F.relu(y), 2: torch.sigmoid(y), 3: torch.tanh(y)}[act]


class _LSTMCell(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, h, c, wi, bi, wf, bf, wg, bg, wo, bo):
        hn, cn, gates = cuda_ext().lstm_fwd(x.contiguous(), h, c, wi, bi, wf, bf, wg, bg, wo, bo, True)
        ctx.save_for_backward(x, h, c, cn, gates, wi, wf, wg, wo)
        ctx.params = (wi, bi, wf, bf, wg, bg, wo, bo)
        ctx.has_h, ctx.has_c = h is not None, c is not None
        # an output nobody used (the last cell state of a window) arrives as None, not
        # as a zero-filled tensor: the backward kernel reads a missing dh / dc as zero
        ctx.set_materialize_grads(False)
        return hn, cn

    @staticmethod
    def backward(ctx, dh, dc):
        x, h, c, cn, gates, wi, wf, wg, wo = ctx.saved_tensors
        bufs = _wgrad_buffers(ctx.params[0::2], ctx.params[1::2])  # w_i, w_f, w_g, w_o, b_i, b_f, b_g, b_o
        gw, gb = [b[0] for b in bufs[:4]], [b[0] for b in bufs[4:]]
        dx, dhp, dcp = cuda_ext().lstm_bwd(x.contiguous(), h if ctx.has_h else None, c if ctx.has_c else None, cn,
                                           gates, dh, dc, wi, wf, wg, wo, gw[0], gb[0], gw[1], gb[1], gw[2], gb[2],
                                           gw[3], gb[3])
        rw, rb = [b[1] for b in bufs[:4]], [b[1] for b in bufs[4:]]
        return (dx, dhp if ctx.has_h else None, dcp if ctx.has_c else None,
                rw[0], rb[0], rw[1], rb[1], rw[2], rb[2], rw[3], rb[3])


class _RGRUCell(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xz, xr, xc, h, wz, bz, wr, br, wc, bc):
        hn, z, r, c, rh = cuda_ext().rgru_fwd(xz, xr, xc, h, wz, bz, wr, br, wc, bc)
        ctx.save_for_backward(xz, xr, xc, h, z, r, c, rh, wz, wr, wc)
        ctx.params = (wz, bz, wr, br, wc, bc)
        return hn

    @staticmethod
    def backward(ctx, dhn):
        xz, xr, xc, h, z, r, c, rh, wz, wr, wc = ctx.saved_tensors
        bufs = _wgrad_buffers(ctx.params[0::2], ctx.params[1::2])  # w_z, w_r, w_c, b_z, b_r, b_c
        gw, gb = [b[0] for b in bufs[:3]], [b[0] for b in bufs[3:]]
        dxz, dxr, dxc, dh = cuda_ext().rgru_bwd(xz, xr, xc, h, z, r, c, rh, dhn.contiguous(), wz, wr, wc,
                                                gw[0], gb[0], gw[1], gb[1], gw[2], gb[2])
        rw, rb = [b[1] for b in bufs[:3]], [b[1] for b in bufs[3:]]
        return dxz, dxr, dxc, dh, rw[0], rb[0], rw[1], rb[1], rw[2], rb[2]


def rgru_cell(xz: torch.Tensor, xr: torch.Tensor, xc: torch.Tensor, h: torch.Tensor, wz, bz, wr, br, wc,
              bc) -> torch.Tensor:
    """Reset-gated GRU cell (T-GCN gates, EvolveGCN MatGRU):
    z = sigmoid(W_z [x_z | h] + b_z), r = sigmoid(W_r [x_r | h] + b_r),
    c = tanh(W_c [x_c | r h] + b_c), h' = z h + (1 - z) c.
    On CUDA two tcgen05 GEMMs with the gate math in their epilogues and a fused
    backward; elsewhere the same math with torch ops."""
    H = wz.size(0)
    if xz.is_cuda and xz.dtype == torch.float32 and H % 8 == 0:
        def unit(t):
            return t if t.stride(-1) == 1 else t.contiguous()
        return _RGRUCell.apply(unit(xz), unit(xr), unit(xc), unit(h), wz, bz, wr, br, wc, bc)
    z = torch.sigmoid(F.linear(torch.cat([xz, h], -1), wz, bz))
    r = torch.sigmoid(F.linear(torch.cat([xr, h], -1), wr, br))
    c = torch.tanh(F.linear(torch.cat([xc, r * h], -1), wc, bc))
    return z * h + (1 - z) * c


def lstm_cell(x: torch.Tensor, h, c, cell) -> tuple[torch.Tensor, torch.Tensor]:
    """cell: module with i_t, f_t, g_t, o_t nn.Linear(in + hidden, hidden)."""
    return _LSTMCell.apply(x.float(), h, c, cell.i_t.weight, cell.i_t.bias, cell.f_t.weight, cell.f_t.bias,
                           cell.g_t.weight, cell.g_t.bias, cell.o_t.weight, cell.o_t.bias)
