"""Data-parallel gradient all-reduce fused with Adam over NVLink (reference:
DistributedDataParallel bucketed NCCL all-reduce + torch Adam,
backends/dtdg/runtime/training.py:84-88, backends/ctdg/runtime/factory.py:115-125).

Both the flat gradient buffer and the flat parameter buffer live in symmetric
allocations. After a device barrier (every rank's backward has finished) one
kernel does reduce-scatter + Adam + all-gather: rank r reads shard r of all W
gradient buffers over NVLink, sums them in rank order, scales by 1/W, applies
Adam to shard r with its own moments, and stores the new shard into every
rank's parameter buffer. Each gradient element crosses NVLink once and each
parameter element is written once per peer, the traffic of a ring
reduce-scatter + all-gather, and every replica receives the same bits. A
second barrier keeps a fast rank from starting its next backward (which
overwrites its gradients) or its next forward (which reads parameters) before
every shard has landed.

Adam moments are therefore valid only on the owning rank's shard;
``gather_state`` assembles the full moments (a collective) for checkpoints.
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
        self.arena = SymmetricArena({"grad": ((n,), torch.float32), "param": ((n,), torch.float32),
                                     "flags": ((32,), torch.int64)}, torch.device(device), group)
        self.arena["grad"].zero_()
        self.arena["flags"].zero_()
        flat.rebind_grad(self.arena["grad"])
        flat.rebind_data(self.arena["param"])
        self.rank, self.world = self.arena.rank, self.arena.world_size
        self._group = group
        self.tables = {k: self.arena.peer_table(k) for k in ("grad", "param", "flags")}
        self.epoch = torch.zeros(1, dtype=torch.int64, device=device)
        self.budget = int(barrier_budget)
        self._C = cuda_ext()
        torch.cuda.synchronize(device)
        self.arena.barrier_host()

    def shard(self) -> tuple[int, int]:
        """[lo, hi) elements of the flat buffers whose Adam step this rank owns."""
        n4 = self.flat.data.numel() // 4
        s4 = (n4 + self.world - 1) // self.world
        return min(n4, self.rank * s4) * 4, min(n4, (self.rank + 1) * s4) * 4

    def _barrier(self) -> None:
        self._C.peer_barrier(self.tables["flags"], self.rank, self.world, self.epoch, self.budget)

    def step(self) -> None:
        o = self.opt
        self._barrier()
        self._C.peer_rs_adam_ag(self.tables["grad"], self.tables["param"], self.world, self.rank, self.flat.data,
                                o.exp_avg, o.exp_avg_sq, o.step_ctr, o.done, float(o.param_groups[0]["lr"]),
                                float(o.betas[0]), float(o.betas[1]), float(o.eps), float(o.weight_decay),
                                1.0 / self.world)
        self._barrier()

    def gather_state(self) -> dict:
        """Collective: the optimizer state with every rank's moment shard put in place."""
        state = self.opt.state_dict()
        for key, t in (("exp_avg", self.opt.exp_avg), ("exp_avg_sq", self.opt.exp_avg_sq)):
            lo, hi = self.shard()
            mine = torch.zeros_like(t)
            mine[lo:hi] = t[lo:hi]
            dist.all_reduce(mine, group=self._group)  # shards are disjoint: the sum places each one
            state[key] = mine.cpu()
        return state
