"""Multi-GPU CTDG memory over NVLink: node memory, mailbox and their
timestamps live in symmetric allocations; each node's rows are authoritative
on its owner rank (``node_parts``, default ``id % world``).

Per step (reference semantics: remote memory/mail pushed to owners and applied
before the next step, backends/ctdg/runtime/memory.py:328-553, runtime.py:243-246):

  1. compute (all ranks, no communication call): the memory updater reads the
     roots' mailbox and memory rows straight from their owners' tables inside
     the GEMM producers and writes the new rows to a local buffer; attention
     reads neighbour rows from the owners (this step's roots from the local
     buffer); backward likewise.
  2. barrier A (tables and gradients are no longer read for this step)
  3. gradient all-reduce fused with Adam (train), memory write-back to owners
     (memory_ts = max over writers), mailbox claims: 64-bit atomicMax of
     (ts, event id) on the owner
  4. barrier B, then the claim winners write the mailbox slots
  5. barrier C (the next step reads consistent tables)

Every wait is a bounded device spin that records a status code and returns.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from starry_unigraph.parallel.symmetric import SymmetricArena

# ~1 s at B200 clocks before a barrier gives up and records kPeerTimeout
DEFAULT_BARRIER_BUDGET = 2_000_000_000


class PeerCTDGContext:
    def __init__(self, *, num_nodes: int, hidden_dim: int, slot_width: int, mailbox_slots: int, grad_numel: int,
                 owner: torch.Tensor, device: torch.device, group: dist.ProcessGroup | None = None,
                 barrier_budget: int = DEFAULT_BARRIER_BUDGET):
        if mailbox_slots != 1:
            raise ValueError("the NVLink CTDG path keeps one mailbox slot per node (ctdg.mailbox_slots: 1)")
        N, D = int(num_nodes), int(hidden_dim)
        self.device = torch.device(device)
        specs = {
            "memory": ((N, D), torch.float32),
            "memory_ts": ((N,), torch.float32),
            "mailbox": ((N, 1, int(slot_width)), torch.float32),
            "mailbox_ts": ((N, 1), torch.float32),
            "claim": ((N,), torch.int64),
            "grad": (((int(grad_numel) + 3) // 4 * 4,), torch.float32),
            "flags": ((32,), torch.int64),
        }
        self.arena = SymmetricArena(specs, self.device, group)
        self.rank, self.world = self.arena.rank, self.arena.world_size
        a = self.arena
        a["memory"].zero_()
        a["memory_ts"].fill_(-1.0)
        a["mailbox"].zero_()
        a["mailbox_ts"].zero_()
        a["claim"].zero_()
        a["grad"].zero_()
        a["flags"].zero_()
        self.owner = owner.to(self.device, torch.int32).contiguous()
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.budget = int(barrier_budget)
        self.tables = {n: a.peer_table(n) for n in ("memory", "memory_ts", "mailbox", "mailbox_ts", "claim", "grad",
                                                    "flags")}
        torch.cuda.synchronize(self.device)
        a.barrier_host()

    def enable_historical_filter(self, alpha: float) -> None:
        """Historical-cache filter of the memory push (reference
        backends/ctdg/runtime/cache.py): for every node this rank does not own, the
        last row it pushed is kept here, and a new row is pushed to the owner only
        when its cosine distance to that row exceeds 1 - alpha (or it was never
        pushed). The check runs inside the write-back kernel."""
        N, D = self.arena["memory"].shape
        shared = self.owner != self.rank
        slot_of = torch.full((N,), -1, dtype=torch.int64, device=self.device)
        n_shared = int(shared.sum())
        slot_of[shared] = torch.arange(n_shared, dtype=torch.int64, device=self.device)
        self.hist_cache = [slot_of, torch.zeros(n_shared, D, device=self.device),
                           torch.full((n_shared,), -1.0, device=self.device)]
        self.hist_thresh = 1.0 - float(alpha)

    hist_cache: list[torch.Tensor] | None = None
    hist_thresh: float = 0.5

    def attach(self, memory_bank) -> None:
        """Re-seat a CTDGMemoryBank's tables on the symmetric storage."""
        a = self.arena
        memory_bank.memory = a["memory"]
        memory_bank.memory_ts = a["memory_ts"]
        memory_bank.mailbox = a["mailbox"]
        memory_bank.mailbox_ts = a["mailbox_ts"]

    def descriptor(self, stamp: torch.Tensor, node2root: torch.Tensor, step_ctr: torch.Tensor,
                   mem_new: torch.Tensor) -> torch.Tensor:
        """CPU int64 [8] descriptor consumed by the memory-reading TGN / JODIE ops."""
        return torch.tensor([self.tables["memory"].data_ptr(), self.tables["mailbox"].data_ptr(),
                             self.owner.data_ptr(), stamp.data_ptr(), node2root.data_ptr(), step_ctr.data_ptr(),
                             mem_new.data_ptr(), self.tables["memory_ts"].data_ptr()], dtype=torch.int64)

    def barrier(self, C) -> None:
        C.peer_barrier(self.tables["flags"], self.rank, self.world, self.epoch, self.budget)
