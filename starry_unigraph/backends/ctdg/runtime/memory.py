"""Per-node memory + K-slot mailbox (reference backends/ctdg/runtime/memory.py:44-574).

Storage is indexed by global node id on every rank (180 GB of HBM holds the
largest configured graphs many times over), with ownership given by
``node_parts`` (default ``id % world_size``). Rows of nodes owned elsewhere act
as this rank's view of remote state:

* ``remote_fetch=False`` reproduces the reference exactly: non-owned rows read
  as zeros (they are never written locally except by received syncs of owned
  rows, which cannot happen) and updates for remote nodes are pushed to their
  owners, applied at the start of the next step (``wait_pending_syncs``).
* ``remote_fetch=True`` additionally refreshes the non-owned rows of the next
  batch's roots from their owners before the step (pull), so a node's memory is
  the owner's latest value instead of zeros.

The mailbox write keeps the reference's slot semantics: all messages of one
node in one pass land in the slot ``next_pos`` (the last by (ts, event index)
wins), then ``next_pos += count mod K``; the src pass runs before the dst pass.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from starry_unigraph.types import DistributedContext


@dataclass
class _PendingSync:
    work: list[Any]
    recv_ids: torch.Tensor
    recv_payload: torch.Tensor
    kind: str


@dataclass
class CTDGMemoryBank:
    num_nodes: int
    hidden_dim: int
    device: str
    mailbox_slots: int = 1
    edge_feat_dim: int = 0
    rank: int = 0
    world_size: int = 1
    async_sync: bool = True
    node_parts: torch.Tensor | None = None
    remote_fetch: bool = False
    _pending: list[_PendingSync] = field(default_factory=list, init=False, repr=False)

    def __post_init__(self) -> None:
        D, K = self.hidden_dim, self.mailbox_slots
        self.edge_feat_dim = max(0, int(self.edge_feat_dim))
        self.slot_width = 2 * D + self.edge_feat_dim
        dev = torch.device(self.device)
        self._storage_device = dev
        if self.world_size > 1:
            owner = self.node_parts.long() if self.node_parts is not None else \
                torch.arange(self.num_nodes, dtype=torch.long) % self.world_size
        else:
            owner = torch.zeros(self.num_nodes, dtype=torch.long)
        self.owner = owner.to(dev)
        self.local_ids = torch.nonzero(owner == self.rank).view(-1)
        self.num_local_nodes = int(self.local_ids.numel())
        self.memory = torch.zeros(self.num_nodes, D, dtype=torch.float32, device=dev)
        self.memory_ts = torch.full((self.num_nodes,), -1.0, dtype=torch.float32, device=dev)
        self.mailbox = torch.zeros(self.num_nodes, K, self.slot_width, dtype=torch.float32, device=dev)
        self.mailbox_ts = torch.zeros(self.num_nodes, K, dtype=torch.float32, device=dev)
        self.next_mail_pos = torch.zeros(self.num_nodes, dtype=torch.long, device=dev)
        self.memory_version = 0
        self.mailbox_version = 0
        self.historical_cache = None
        self.last_memory_sync: tuple | None = None
        self.last_mail_sync: tuple | None = None
        self.pulled_rows = 0  # rows refreshed from their owners by pull_remote, cumulative

    # ------------------------------------------------------------------ reads
    @property
    def last_update(self) -> torch.Tensor:
        return self.memory_ts

    def is_owned(self, node_ids: torch.Tensor) -> torch.Tensor:
        return self.owner[node_ids.to(self.owner.device).long()] == self.rank

    def _visible(self, node_ids: torch.Tensor) -> torch.Tensor:
        ids = node_ids.to(self._storage_device).long()
        if self.world_size == 1 or self.remote_fetch:
            return torch.ones_like(ids, dtype=torch.bool)
        return self.owner[ids] == self.rank

    def gather(self, node_ids: torch.Tensor) -> torch.Tensor:
        ids = node_ids.to(self._storage_device).long()
        out = self.memory[ids]
        vis = self._visible(ids)
        if not bool(vis.all()):
            out = out * vis.unsqueeze(1)
        return out

    def read_mailbox(self, node_ids: torch.Tensor) -> torch.Tensor:
        ids = node_ids.to(self._storage_device).long()
        out = self.mailbox[ids]
        vis = self._visible(ids)
        if not bool(vis.all()):
            out = out * vis.view(-1, 1, 1)
        return out

    def gather_mailbox(self, node_ids: torch.Tensor) -> torch.Tensor:
        return self.read_mailbox(node_ids)[:, 0, :]

    def read_mailbox_ts(self, node_ids: torch.Tensor) -> torch.Tensor:
        ids = node_ids.to(self._storage_device).long()
        out = self.mailbox_ts[ids]
        vis = self._visible(ids)
        return out * vis.unsqueeze(1) if not bool(vis.all()) else out

    # ------------------------------------------------------------------ writes
    def write_mailbox(self, src_ids, dst_ids, src_mem, dst_mem, edge_feat, timestamps) -> None:
        E = self.edge_feat_dim
        ef = edge_feat.float().to(self._storage_device)
        if ef.dim() == 1:
            ef = ef.view(-1, 1)
        ef = ef[..., :E] if ef.size(-1) >= E else torch.cat(
            [ef, torch.zeros(*ef.shape[:-1], E - ef.size(-1), device=ef.device)], dim=-1)
        smem = src_mem.float().to(self._storage_device)
        dmem = dst_mem.float().to(self._storage_device)
        ts = timestamps.float().to(self._storage_device)
        self._write_slots(src_ids, torch.cat([smem, dmem, ef], dim=-1), ts)
        self._write_slots(dst_ids, torch.cat([dmem, smem, ef], dim=-1), ts)
        self.mailbox_version += 1

    def _write_slots(self, ids: torch.Tensor, values: torch.Tensor, ts: torch.Tensor) -> None:
        ids = ids.to(self._storage_device).long()
        keep = self._visible(ids) if self.world_size > 1 else torch.ones_like(ids, dtype=torch.bool)
        if self.world_size > 1 and not self.remote_fetch:
            keep = self.owner[ids] == self.rank
        if not bool(keep.any()):
            return
        ids, values, ts = ids[keep], values[keep], ts[keep]
        K = self.mailbox_slots
        # last message per node by (ts, position): stable sort by ts, keep last occurrence
        order = torch.sort(ts, stable=True).indices
        ids_s, vals_s, ts_s = ids[order], values[order], ts[order]
        uniq, inv, counts = torch.unique(ids_s, return_inverse=True, return_counts=True)
        pos_in = torch.arange(ids_s.numel(), device=ids.device)
        last = torch.zeros(uniq.numel(), dtype=torch.long, device=ids.device).scatter_reduce(
            0, inv, pos_in, reduce="amax", include_self=False)
        slot = self.next_mail_pos[uniq]
        self.mailbox[uniq, slot] = vals_s[last]
        self.mailbox_ts[uniq, slot] = ts_s[last]
        self.next_mail_pos[uniq] = (slot + counts) % K

    def _apply_memory_update(self, node_ids: torch.Tensor, values: torch.Tensor, timestamps: torch.Tensor) -> None:
        if node_ids.numel() == 0:
            return
        ids = node_ids.to(self._storage_device).long()
        keep = torch.ones_like(ids, dtype=torch.bool) if (self.world_size == 1 or self.remote_fetch) \
            else self.owner[ids] == self.rank
        if not bool(keep.any()):
            return
        ids, vals, ts = ids[keep], values[keep].float(), timestamps[keep].float().to(ids.device)
        order = torch.sort(ts, stable=True).indices
        self.memory[ids[order]] = vals[order]
        self.memory_ts[ids[order]] = ts[order]
        self.memory_version += 1

    _apply_updates = _apply_memory_update

    def _apply_mail_update(self, node_ids, mail_slots, mail_ts) -> None:
        if node_ids.numel() == 0:
            return
        ids = node_ids.to(self._storage_device).long()
        inc = mail_ts.to(ids.device).max(dim=1).values
        cur = self.mailbox_ts[ids].max(dim=1).values
        newer = inc > cur
        if bool(newer.any()):
            self.mailbox[ids[newer]] = mail_slots.to(ids.device)[newer]
            self.mailbox_ts[ids[newer]] = mail_ts.to(ids.device)[newer]
            self.mailbox_version += 1

    # ------------------------------------------------------------------ distributed sync
    @staticmethod
    def _distributed_ready(ctx: DistributedContext) -> bool:
        if not ctx.is_distributed:
            return False
        import torch.distributed as dist

        return dist.is_initialized()

    def _exchange(self, ctx: DistributedContext, ids: torch.Tensor, payload: torch.Tensor, kind: str) -> None:
        """Owner-routed all-to-all of (ids, payload rows). Every rank always takes part
        (also with nothing to send), so collective participation never diverges."""
        import torch.distributed as dist

        dev = self._storage_device if ctx.backend == "nccl" else torch.device("cpu")
        ids = ids.to(dev).long()
        payload = payload.to(dev).float()
        owner = self.owner.to(dev)[ids] if ids.numel() else ids
        order = torch.argsort(owner, stable=True) if ids.numel() else ids
        ids, payload = ids[order], payload[order]
        send_counts = torch.bincount(owner[order], minlength=ctx.world_size) if ids.numel() else \
            torch.zeros(ctx.world_size, dtype=torch.long, device=dev)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        width = payload.size(1) if payload.dim() == 2 else 1
        recv_ids = torch.empty(sum(rc), dtype=torch.long, device=dev)
        recv_payload = torch.empty(sum(rc), width, dtype=torch.float32, device=dev)
        w1 = dist.all_to_all_single(recv_ids, ids, rc, sc, async_op=True)
        w2 = dist.all_to_all_single(recv_payload.view(-1), payload.reshape(-1).contiguous(),
                                    [c * width for c in rc], [c * width for c in sc], async_op=True)
        self._pending.append(_PendingSync(work=[w1, w2], recv_ids=recv_ids, recv_payload=recv_payload, kind=kind))
        if not self.async_sync:
            self.wait_pending_syncs()

    def submit_async_memory_sync(self, ctx: DistributedContext, node_ids, values, timestamps) -> None:
        if not self._distributed_ready(ctx):
            self._apply_memory_update(node_ids, values.detach(), timestamps.detach())
            return
        ids = node_ids.to(self._storage_device).long()
        remote = self.owner[ids] != ctx.rank
        ids, vals, ts = ids[remote], values.detach().float()[remote], timestamps.detach().float()[remote]
        if self.historical_cache is not None and ids.numel():
            changed = self.historical_cache.historical_check(ids, vals)
            self.historical_cache.update_cache(self.historical_cache.slot_indices(ids[changed]), vals[changed],
                                               ts[changed])
            ids, vals, ts = ids[changed], vals[changed], ts[changed]
        self._exchange(ctx, ids, torch.cat([vals, ts.unsqueeze(1)], dim=1), "memory")

    def submit_async_mail_sync(self, ctx: DistributedContext, node_ids, mail_slots, mail_ts) -> None:
        if not self._distributed_ready(ctx):
            return
        ids = node_ids.to(self._storage_device).long()
        remote = self.owner[ids] != ctx.rank
        ids = ids[remote]
        def rows(t: torch.Tensor) -> torch.Tensor:  # [n, ...] -> [n, width], also for n == 0
            return t.flatten(1) if t.dim() > 1 else t.unsqueeze(1)

        payload = torch.cat([rows(mail_slots.detach().float()[remote]), rows(mail_ts.detach().float()[remote])], dim=1)
        self._exchange(ctx, ids, payload, "mail")

    def wait_pending_syncs(self) -> None:
        K, SW, D = self.mailbox_slots, self.slot_width, self.hidden_dim
        while self._pending:
            p = self._pending.pop(0)
            for w in p.work:
                w.wait()
            n = int(p.recv_ids.numel())
            ids = p.recv_ids.to(self._storage_device)
            pay = p.recv_payload.to(self._storage_device)
            if p.kind == "memory":
                keep = self.owner[ids] == self.rank
                ids_k, pay_k = ids[keep], pay[keep]
                order = torch.sort(pay_k[:, D], stable=True).indices
                self.memory[ids_k[order]] = pay_k[order, :D]
                self.memory_ts[ids_k[order]] = pay_k[order, D]
                self.memory_version += 1
                self.last_memory_sync = (n,)
            else:
                self._apply_mail_update(ids, pay[:, :K * SW].view(n, K, SW), pay[:, K * SW:].view(n, K))
                self.last_mail_sync = (n,)

    def pull_remote(self, ctx: DistributedContext, node_ids: torch.Tensor) -> None:
        """Refresh non-owned rows of ``node_ids`` (memory, memory_ts, mailbox, mailbox_ts,
        next_mail_pos) from their owners: request ids, owners answer with rows."""
        if not self._distributed_ready(ctx) or not self.remote_fetch:
            return
        import torch.distributed as dist

        dev = self._storage_device if ctx.backend == "nccl" else torch.device("cpu")
        ids = torch.unique(node_ids.to(self._storage_device).long())
        ids = ids[self.owner[ids] != ctx.rank].to(dev)
        owner = self.owner.to(dev)[ids]
        order = torch.argsort(owner, stable=True)
        ids = ids[order]
        sc_t = torch.bincount(owner[order], minlength=ctx.world_size) if ids.numel() else \
            torch.zeros(ctx.world_size, dtype=torch.long, device=dev)
        rc_t = torch.empty_like(sc_t)
        dist.all_to_all_single(rc_t, sc_t)
        sc, rc = sc_t.tolist(), rc_t.tolist()
        req = torch.empty(sum(rc), dtype=torch.long, device=dev)
        dist.all_to_all_single(req, ids, rc, sc)
        K, SW, D = self.mailbox_slots, self.slot_width, self.hidden_dim
        rq = req.to(self._storage_device)
        rows = torch.cat([self.memory[rq], self.memory_ts[rq].unsqueeze(1), self.mailbox[rq].flatten(1),
                          self.mailbox_ts[rq], self.next_mail_pos[rq].float().unsqueeze(1)], dim=1).to(dev)
        width = rows.size(1) if rows.dim() == 2 and rows.numel() else D + 1 + K * SW + K + 1
        ans = torch.empty(sum(sc), width, dtype=torch.float32, device=dev)
        dist.all_to_all_single(ans.view(-1), rows.reshape(-1).contiguous(), [c * width for c in sc],
                               [c * width for c in rc])
        self.pulled_rows += int(ids.numel())
        if ids.numel():
            i = ids.to(self._storage_device)
            a = ans.to(self._storage_device)
            self.memory[i] = a[:, :D]
            self.memory_ts[i] = a[:, D]
            self.mailbox[i] = a[:, D + 1:D + 1 + K * SW].view(-1, K, SW)
            self.mailbox_ts[i] = a[:, D + 1 + K * SW:D + 1 + K * SW + K]
            self.next_mail_pos[i] = a[:, -1].long()

    def describe(self) -> dict[str, Any]:
        return {"num_nodes": self.num_nodes, "num_local_nodes": self.num_local_nodes, "hidden_dim": self.hidden_dim,
                "mailbox_slots": self.mailbox_slots, "memory_version": self.memory_version,
                "storage_device": str(self._storage_device), "remote_fetch": self.remote_fetch}
