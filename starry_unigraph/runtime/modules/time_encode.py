"""Learnable cosine time encoding (reference runtime/modules/time_encode.py:13-58).

phi(t) = cos(w t + b), w initialised to 10^-linspace(0, 9, dim), b = 0, both
learnable (stored as an nn.Linear(1, dim) so state-dict keys match).
"""
from __future__ import annotations

import torch
import torch.nn as nn


class TimeEncode(nn.Module):
    def __init__(self, dim: int) -> None:
        super().__init__()
        self.dim = dim
        self.w = nn.Linear(1, dim)
        self.w.weight = nn.Parameter((1.0 / 10 ** torch.linspace(0, 9, dim)).reshape(dim, 1))
        self.w.bias = nn.Parameter(torch.zeros(dim))

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        return torch.cos(self.w(t.float().reshape(-1, 1))).reshape(*t.shape, self.dim)
