"""Per-node memory with a K-slot mailbox, as plain tensors (reference
runtime/store/MemoryState.py:41-76, where ``MemoryState.update/gather`` are
empty and ``MemoryBank.describe`` reads attributes the class never sets).

* ``MemoryBank``: memory [N, hidden] with its last-update time, a mailbox
  [N, K, 2 * hidden + edge_feat_dim] with per-slot times, and a version counter
  that every update advances. Mail slots fill in a ring per node.
* ``MemoryState``: a dense per-node state (for example an embedding cache) over
  a bank, with the dependence declarations of the chunk that owns it;
  ``update`` writes rows (and, given mail, the bank's mailbox), ``gather`` reads
  them.

The training engines keep their node memory in ``CTDGMemoryBank`` (owner-
partitioned, peer-accessible); these classes are the store-module API for code
written against the unified runtime.
"""
from __future__ import annotations

from typing import Any

import torch

from starry_unigraph.runtime.route.comm_plan import SpatialDeps, StateDeps


class MemoryBank:
    def __init__(self, num_nodes: int, hidden_dim: int, edge_feat_dim: int = 0, mailbox_slots: int = 1,
                 device: str | torch.device = "cpu", async_sync: bool = False) -> None:
        self.num_nodes = int(num_nodes)
        self.num_local_nodes = int(num_nodes)  # one process holds every row here
        self.hidden_dim = int(hidden_dim)
        self.edge_feat_dim = int(edge_feat_dim)
        self.mailbox_slots = max(1, int(mailbox_slots))
        self.device = torch.device(device)
        self._storage_device = self.device
        self.async_sync = bool(async_sync)
        self.memory = torch.zeros(self.num_nodes, self.hidden_dim, device=self.device)
        self.memory_ts = torch.zeros(self.num_nodes, device=self.device)
        self.mailbox = torch.zeros(self.num_nodes, self.mailbox_slots, 2 * self.hidden_dim + self.edge_feat_dim,
                                   device=self.device)
        self.mailbox_ts = torch.zeros(self.num_nodes, self.mailbox_slots, device=self.device)
        self.next_mail_pos = torch.zeros(self.num_nodes, dtype=torch.long, device=self.device)
        self.memory_version = 0

    def update_memory(self, index: torch.Tensor, values: torch.Tensor, ts: torch.Tensor | None = None) -> None:
        index = index.to(self.device).long()
        self.memory[index] = values.to(self.memory)
        if ts is not None:
            self.memory_ts[index] = ts.to(self.memory_ts)
        self.memory_version += 1

    def write_mail(self, index: torch.Tensor, mails: torch.Tensor, ts: torch.Tensor | None = None) -> None:
        """One mail per listed node into its next ring slot (a node listed twice
        takes consecutive slots in list order)."""
        index = index.to(self.device).long()
        if index.numel() == 0:
            return
        order = torch.argsort(index, stable=True)
        idx = index[order]
        first = torch.ones_like(idx, dtype=torch.bool)
        first[1:] = idx[1:] != idx[:-1]
        start = torch.cummax(torch.where(first, torch.arange(idx.numel(), device=self.device),
                                         torch.zeros_like(idx)), 0).values
        rank_in_node = torch.arange(idx.numel(), device=self.device) - start
        slot = (self.next_mail_pos[idx] + rank_in_node) % self.mailbox_slots
        self.mailbox[idx, slot] = mails.to(self.mailbox)[order]
        if ts is not None:
            self.mailbox_ts[idx, slot] = ts.to(self.mailbox_ts)[order]
        counts = torch.bincount(idx, minlength=self.num_nodes)
        self.next_mail_pos = (self.next_mail_pos + counts) % self.mailbox_slots
        self.memory_version += 1

    def describe(self) -> dict[str, Any]:
        return {
            "num_nodes": self.num_nodes,
            "num_local_nodes": self.num_local_nodes,
            "hidden_dim": self.hidden_dim,
            "mailbox_slots": self.mailbox_slots,
            "memory_version": self.memory_version,
            "storage_device": str(self._storage_device),
        }


class MemoryState:
    def __init__(self, node_nums: int, hidden_dim: int, memory_bank: MemoryBank,
                 state_deps: StateDeps | None = None, spatial_deps: SpatialDeps | None = None) -> None:
        self.node_nums = int(node_nums)
        self.memory_bank = memory_bank
        self.state_deps = state_deps
        self.spatial_deps = spatial_deps
        self.memory = torch.zeros(self.node_nums, int(hidden_dim), device=memory_bank.device)

    def update(self, index: torch.Tensor, memory: torch.Tensor, mails: torch.Tensor | None = None,
               state_deps: StateDeps | None = None, mail_ts: torch.Tensor | None = None) -> None:
        """Store `memory` rows at `index`; with `mails`, also append them to the
        bank's mailbox of those nodes. `state_deps` replaces the declared
        dependences (the rows to notify after this update)."""
        index = index.to(self.memory.device).long()
        self.memory[index] = memory.to(self.memory)
        if mails is not None:
            self.memory_bank.write_mail(index, mails, mail_ts)
        if state_deps is not None:
            self.state_deps = state_deps

    def gather(self, index: torch.Tensor, memory: torch.Tensor | None = None, mails: bool = False,
               state_deps: StateDeps | None = None):
        """Rows at `index`, written into `memory` when given; with `mails`, also
        the bank's mailbox of those nodes (returned as a pair)."""
        index = index.to(self.memory.device).long()
        rows = self.memory[index]
        if memory is not None:
            memory.copy_(rows)
            rows = memory
        if mails:
            return rows, self.memory_bank.mailbox[index]
        return rows
