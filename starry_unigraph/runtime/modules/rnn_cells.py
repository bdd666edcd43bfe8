"""Recurrent cells for DTDG models (reference runtime/modules/rnn_cells.py:14-116).

* ``MatGRUCell``: EvolveGCN's weight-evolving GRU: with xc = [ctx rows || W],
  z = sigmoid(L_z xc), r = sigmoid(L_r xc), W~ = tanh(L_h [ctx || r * W]),
  W' = z * W + (1 - z) * W~.
* ``_LSTMCell``: four Linear(in + hidden, hidden) gates over [x || h]; on CUDA
  one fused tcgen05 GEMM with a gate epilogue.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from starry_unigraph.ops.dtdg import linear, lstm_cell, rgru_cell


class MatGRUCell(nn.Module):
    def __init__(self, in_feats: int, out_feats: int) -> None:
        super().__init__()
        self.update = nn.Linear(in_feats + out_feats, out_feats)
        self.reset = nn.Linear(in_feats + out_feats, out_feats)
        self.htilda = nn.Linear(in_feats + out_feats, out_feats)

    def forward(self, prev_w: torch.Tensor, inputs: torch.Tensor) -> torch.Tensor:
        inputs = inputs.reshape(1, -1).repeat(prev_w.size(0), 1)
        if inputs.is_cuda:
            return rgru_cell(inputs, inputs, inputs, prev_w.float(), self.update.weight, self.update.bias,
                             self.reset.weight, self.reset.bias, self.htilda.weight, self.htilda.bias)
        xc = torch.cat([inputs, prev_w], dim=1)
        z = linear(xc, self.update.weight, self.update.bias, 2)
        r = linear(xc, self.reset.weight, self.reset.bias, 2)
        h_tilde = linear(torch.cat([inputs, r * prev_w], dim=1), self.htilda.weight, self.htilda.bias, 3)
        return z * prev_w + (1 - z) * h_tilde


class _LSTMCell(nn.Module):
    def __init__(self, input_size: int, hidden_size: int) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.i_t = nn.Linear(input_size + hidden_size, hidden_size)
        self.f_t = nn.Linear(input_size + hidden_size, hidden_size)
        self.g_t = nn.Linear(input_size + hidden_size, hidden_size)
        self.o_t = nn.Linear(input_size + hidden_size, hidden_size)

    def forward(self, x: torch.Tensor, state: tuple[torch.Tensor, torch.Tensor] | None = None):
        if x.is_cuda and self.hidden_size <= 128:
            h, c = (None, None) if state is None else state
            return lstm_cell(x, h, c, self)
        if state is None:
            h = torch.zeros(x.size(0), self.hidden_size, dtype=x.dtype, device=x.device)
            c = torch.zeros_like(h)
        else:
            h, c = state
        xh = torch.cat([x, h], dim=-1)
        i = torch.sigmoid(self.i_t(xh))
        f = torch.sigmoid(self.f_t(xh))
        g = torch.tanh(self.g_t(xh))
        o = torch.sigmoid(self.o_t(xh))
        c = f * c + i * g
        return o * torch.tanh(c), c
