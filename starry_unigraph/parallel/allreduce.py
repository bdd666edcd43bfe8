"""Data-parallel gradient all-reduce fused with Adam over NVLink (reference:
DistributedDataParallel bucketed NCCL all-reduce + torch Adam,
backends/dtdg/runtime/training.py:84-88, backends/ctdg/runtime/factory.py:115-125).

The flat gradient buffer lives in a symmetric allocation; after a device
barrier every rank reads all W gradient buffers, sums them in rank order (so
every replica gets bit-identical parameters), scales by 1/W and applies Adam
in the same kernel; a second barrier keeps a fast rank from overwriting its
gradients before the slow ones have read them.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from starry_unigraph.ops import cuda_ext
from starry_unigraph.parallel.ctdg_peer import DEFAULT_BARRIER_BUDGET
from starry_unigraph.parallel.symmetric import SymmetricArena


class PeerAllReduceAdam:
    def __init__(self, flat, opt, device: torch.device, group: dist.ProcessGroup | None = None,
                 barrier_budget: int = DEFAULT_BARRIER_BUDGET):
        self.flat, self.opt = flat, opt
        n = (flat.grad.numel() + 3) // 4 * 4
        self.arena = SymmetricArena({"grad": ((n,), torch.float32), "flags": ((32,), torch.int64)},
                                    torch.device(device), group)
        self.arena["grad"].zero_()
        self.arena["flags"].zero_()
        flat.rebind_grad(self.arena["grad"])
        self.rank, self.world = self.arena.rank, self.arena.world_size
        self.tables = {k: self.arena.peer_table(k) for k in ("grad", "flags")}
        self.epoch = torch.zeros(1, dtype=torch.int64, device=device)
        self.budget = int(barrier_budget)
        self._C = cuda_ext()
        torch.cuda.synchronize(device)
        self.arena.barrier_host()

    def _barrier(self) -> None:
        self._C.peer_barrier(self.tables["flags"], self.rank, self.world, self.epoch, self.budget)

    def step(self) -> None:
        o = self.opt
        self._barrier()
        self._C.peer_allreduce_adam(self.tables["grad"], self.world, self.flat.data, o.exp_avg, o.exp_avg_sq,
                                    o.step_ctr, o.done, float(o.param_groups[0]["lr"]), float(o.betas[0]),
                                    float(o.betas[1]), float(o.eps), float(o.weight_decay), 1.0 / self.world)
        self._barrier()
