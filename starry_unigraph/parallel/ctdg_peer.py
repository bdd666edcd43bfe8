"""Multi-GPU CTDG memory over NVLink: node memory, mailbox and their
timestamps live in symmetric allocations; each node's rows are authoritative
on its owner rank (``node_parts``, default ``id % world``).

Per step t (reference semantics: remote memory/mail pushed to owners and
applied before the next step reads them, backends/ctdg/runtime/memory.py:
328-553, runtime.py:243-246):

  1. prep + neighbour sampling (local; overlaps the peers still finishing
     step t-1)
  2. wait C(t-1): every peer finished step t-1's pushes into the tables and its
     reads of this rank's gradient buffer; fused with this step's mailbox
     claims (64-bit atomicMax of (ts, event id) on the owner)
  3. compute, no communication call: the memory updater reads the roots'
     mailbox and memory rows straight from their owners' tables inside the GEMM
     producers and writes the new rows to a local buffer; attention reads
     neighbour rows from the owners (this step's roots from the local buffer);
     backward likewise
  4. barrier A (every rank's gradients are complete and nobody reads the
     tables for step t any more)
  5. on a side stream: memory write-back (memory_ts = max over writers) and the
     claim winners' mailbox slots; on the main stream: reduce-scatter of the
     gradient, Adam on this rank's shard, all-gather of the new parameters
  6. signal C(t), no wait (the wait is step t+1's item 2)

Every wait is a bounded device spin that records a status code and returns.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from starry_unigraph.parallel.symmetric import SymmetricArena

# ~10 s at B200 clocks before a device barrier gives up and records kPeerTimeout: long
# enough to absorb host-side skew between ranks (set-up, logging, a checkpoint on
# one rank), short enough that a rank that never arrives surfaces as an error
DEFAULT_BARRIER_BUDGET = 20_000_000_000


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
            "param": (((int(grad_numel) + 3) // 4 * 4,), torch.float32),
            "flags": ((32,), torch.int64),    # barrier A
            "flags_c": ((32,), torch.int64),  # end-of-step signal / next-step wait
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
        a["param"].zero_()
        a["flags"].zero_()
        a["flags_c"].zero_()
        self.owner = owner.to(self.device, torch.int32).contiguous()
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.epoch_c = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.budget = int(barrier_budget)
        self.tables = {n: a.peer_table(n) for n in ("memory", "memory_ts", "mailbox", "mailbox_ts", "claim", "grad",
                                                    "param", "flags", "flags_c")}
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

    def signal_end(self, C) -> None:
        """First half of the end-of-step barrier (no wait)."""
        C.peer_signal(self.tables["flags_c"], self.rank, self.world, self.epoch_c)

    def drain(self, C) -> None:
        """Wait until every peer finished its last step's pushes (and reads of this
        rank's buffers). Needed before the tables are read on the host and before
        teardown: with the split end-of-step barrier a fast rank may otherwise free
        memory that a slow peer still writes into."""
        C.peer_wait(self.arena["flags_c"], self.rank, self.world, self.epoch_c, self.budget)

    def wait_claim(self, C, roots, n_roots, win, ev_eid, ev_ts) -> None:
        """Second half of the previous step's end-of-step barrier, fused with this
        step's mailbox claims."""
        C.tgn_peer_wait_claim(self.arena["flags_c"], self.rank, self.world, self.epoch_c, self.budget, roots, n_roots,
                              win, ev_eid, ev_ts, self.owner, self.tables["claim"])
