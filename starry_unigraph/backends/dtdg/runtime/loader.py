"""Snapshot loader (reference backends/dtdg/runtime/loader.py:21-279).

The whole partition is moved to the device once (a B200 holds every configured
partition many times over), so a step never waits on a host->device copy and
needs no per-snapshot barrier; the reference's pinned side-stream prefetch is
kept for CPU-resident partitions (``resident=False``).
"""
from __future__ import annotations

from typing import Any

import torch

from starry_unigraph.data.partition import PartitionData

from .state import RNNStateManager, STGraphBlob


class STGraphLoader:
    def __init__(self, rank: int, size: int, data: PartitionData, device: torch.device, chunk_count: int,
                 chunk_index: torch.Tensor, stream: Any = None) -> None:
        self.rank, self.size, self.data, self.device = rank, size, data, device
        self.chunk_count, self.chunk_index, self.stream = chunk_count, chunk_index, stream

    @classmethod
    def from_partition_data(cls, data: PartitionData, device: str | torch.device, chunk_index: torch.Tensor,
                            rank: int = 0, size: int = 1, resident: bool = True) -> "STGraphLoader":
        dev = torch.device(device)
        stream = None
        if dev.type == "cuda":
            if resident:
                data = data.to(dev)
            else:
                data = data.pin_memory()
                stream = torch.cuda.Stream(dev)
        chunk_index = chunk_index.long().to(dev)
        chunk_count = int(chunk_index.max().item() + 1) if chunk_index.numel() else 0
        return cls(rank, size, data, dev, chunk_count, chunk_index, stream)

    def __len__(self) -> int:
        return len(self.data)

    def __getitem__(self, index: slice) -> "STGraphLoader":
        if not isinstance(index, slice):
            raise TypeError("Only slice access is supported")
        return STGraphLoader(self.rank, self.size, self.data[index], self.device, self.chunk_count, self.chunk_index,
                             self.stream)

    @staticmethod
    def reorder_chunks(order: torch.Tensor, score: torch.Tensor | None = None) -> torch.Tensor:
        order = order.long()
        if score is None:
            return order
        ranked = score[order].argsort(dim=0, descending=True)
        remapped = torch.empty_like(ranked)
        remapped[ranked] = torch.arange(ranked.numel(), dtype=ranked.dtype, device=ranked.device)
        return remapped

    def _get_perm_ends(self, chunk_order=None, chunk_decay=None, num_full_snaps: int = 1):
        if chunk_order is None:
            return None, None
        if int(chunk_order.numel()) != int(self.chunk_count):
            raise ValueError(f"Expected chunk_order size {self.chunk_count}, got {chunk_order.numel()}")
        if not chunk_decay:
            return None, [None] * max(1, num_full_snaps)
        chunk_order = chunk_order.to(self.device)
        ordered = chunk_order[self.chunk_index]
        _, perm = ordered.sort(dim=0, stable=True)
        ends = torch.cumsum(torch.bincount(ordered, minlength=self.chunk_count), 0).tolist()
        ends_list = [ends[max(0, min(self.chunk_count - 1, int(step) - 1))] for step in reversed(chunk_decay)]
        ends_list.extend([None] * max(1, num_full_snaps))
        return perm, ends_list

    def __call__(self, chunk_order=None, chunk_decay=None, num_full_snaps: int = 1, disable_states: bool = True,
                 disable_routes: bool = False, window: int | None = None):
        perm, ends_list = self._get_perm_ends(chunk_order, chunk_decay, num_full_snaps)
        if window is not None:
            # explicit window: `window` slots, older ones truncated like the decay ends (if any)
            ends_list = ([None] * window) if ends_list is None else \
                ([e for e in ends_list if e is not None][:max(0, window - 1)] + [None] * window)[:window]
            ends_list = (ends_list + [None] * window)[:window]
        if ends_list is None:
            for i in range(len(self)):
                states = RNNStateManager(ends_list=[None], mode="pad", disable_routes=disable_routes)
                states.add(self.fetch_graph(i, perm=perm))
                yield states.snapshot()
        else:
            states = RNNStateManager(ends_list=ends_list, mode="pad" if disable_states else "mix",
                                     disable_routes=disable_routes)
            for i in range(len(self)):
                states.add(self.fetch_graph(i, perm=perm))
                yield states.snapshot()  # frozen: the window stays valid after the loader slides on

    def __iter__(self):
        yield from self.__call__()

    def fetch_graph(self, index: int, perm: torch.Tensor | None = None, ends: int | None = None,
                    disable_routes: bool = False, disable_states: bool = True):
        if self.stream is not None:
            with torch.cuda.stream(self.stream):
                snap = self.data[index].to(device=self.device, non_blocking=True)
            torch.cuda.current_stream(self.device).wait_stream(self.stream)
        else:
            snap = self.data[index]
        block = snap.item(node_perm=perm, keep_ids=True)
        if self.size == 1 or disable_routes:
            block.route = None
        block.flare_snapshot_id = index
        block.flare_is_full_snapshot = ends is None
        return block

    def build_snapshot_index(self) -> dict[str, Any]:
        return {"snaps": len(self.data), "partition_rank": self.rank, "partition_size": self.size,
                "chunk_count": self.chunk_count, "index_ready": True}
