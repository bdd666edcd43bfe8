"""Flat parameter / gradient buffers.

All trainable parameters of a module set are re-seated as views of one fp32
buffer and their ``.grad`` as views of a second one. A fused optimiser then
updates everything in one kernel, gradient synchronisation is one collective
on one buffer, and kernels write gradients straight into the views.
"""
from __future__ import annotations

from typing import Iterable

import torch
import torch.nn as nn


class FlatParams:
    def __init__(self, modules: Iterable[nn.Module], device: torch.device, requires_grad_only: bool = True):
        params: list[tuple[str, nn.Parameter]] = []
        seen: set[int] = set()
        for mi, m in enumerate(modules):
            for name, p in m.named_parameters():
                if id(p) in seen or (requires_grad_only and not p.requires_grad):
                    continue
                seen.add(id(p))
                params.append((f"{mi}.{name}", p))
        total = sum(p.numel() for _, p in params)
        # pad to a multiple of 4 floats so vector loads in the optimiser stay aligned
        padded = (total + 3) // 4 * 4
        self.data = torch.zeros(padded, dtype=torch.float32, device=device)
        self.grad = torch.zeros(padded, dtype=torch.float32, device=device)
        self.names: list[str] = []
        self.views: dict[str, torch.Tensor] = {}
        self.grad_views: dict[str, torch.Tensor] = {}
        off = 0
        for name, p in params:
            n = p.numel()
            self.data[off:off + n].copy_(p.detach().reshape(-1).to(device=device, dtype=torch.float32))
            view = self.data[off:off + n].view_as(p)
            p.data = view
            gview = self.grad[off:off + n].view_as(p)
            p.grad = gview
            self.names.append(name)
            self.views[name] = view
            self.grad_views[name] = gview
            off += n
        self.numel = total
        self.params = [p for _, p in params]

    def rebind_grad(self, buffer: torch.Tensor) -> None:
        """Move the gradient views onto `buffer` (e.g. a symmetric allocation that
        peer GPUs read); its first ``grad.numel()`` elements are used."""
        assert buffer.numel() >= self.grad.numel() and buffer.dtype == torch.float32
        new = buffer.view(-1)[: self.grad.numel()]
        new.copy_(self.grad)
        self.grad = new
        off = 0
        for name, p in zip(self.names, self.params):
            n = p.numel()
            gview = self.grad[off:off + n].view_as(p)
            p.grad = gview
            self.grad_views[name] = gview
            off += n

    def rebind_data(self, buffer: torch.Tensor) -> None:
        """Move the parameters onto `buffer` (e.g. a symmetric allocation that
        peer GPUs write updated shards into); values are copied over."""
        assert buffer.numel() >= self.data.numel() and buffer.dtype == torch.float32
        new = buffer.view(-1)[: self.data.numel()]
        new.copy_(self.data)
        self.data = new
        off = 0
        for name, p in zip(self.names, self.params):
            n = p.numel()
            view = self.data[off:off + n].view_as(p)
            p.data = view
            self.views[name] = view
            off += n

    def zero_grad(self) -> None:
        self.grad.zero_()


class FusedAdam:
    """torch.optim.Adam semantics on a FlatParams buffer, one sm_100a kernel per step."""

    def __init__(self, flat: FlatParams, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0):
        from starry_unigraph.ops import cuda_ext

        self._C = cuda_ext()
        self.flat = flat
        self.lr, self.betas, self.eps, self.weight_decay = lr, betas, eps, weight_decay
        dev = flat.data.device
        self.exp_avg = torch.zeros_like(flat.data)
        self.exp_avg_sq = torch.zeros_like(flat.data)
        self.step_ctr = torch.zeros(1, dtype=torch.int64, device=dev)
        self.done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.param_groups = [{"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay,
                              "params": flat.params}]

    def step(self, grad_scale: float = 1.0) -> None:
        self._C.adam_flat(self.flat.data, self.flat.grad, self.exp_avg, self.exp_avg_sq, self.step_ctr, self.done,
                          float(self.param_groups[0]["lr"]), float(self.betas[0]), float(self.betas[1]),
                          float(self.eps), float(self.weight_decay), float(grad_scale))

    def zero_grad(self, set_to_none: bool = False) -> None:
        self.flat.zero_grad()

    def state_dict(self) -> dict:
        return {"exp_avg": self.exp_avg.cpu(), "exp_avg_sq": self.exp_avg_sq.cpu(), "step": self.step_ctr.cpu(),
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups]}

    def load_state_dict(self, state: dict) -> None:
        self.exp_avg.copy_(state["exp_avg"])
        self.exp_avg_sq.copy_(state["exp_avg_sq"])
        self.step_ctr.copy_(state["step"])
