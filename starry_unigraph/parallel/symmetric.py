"""Symmetric device allocations: one buffer per rank at the same size, mapped
into every rank's address space (``torch.distributed._symmetric_memory``), and
carved into named tensors at identical offsets. A kernel reaches rank q's copy
of tensor ``name`` at ``peer_table(name)[q]``: plain loads, stores and atomics
over NVLink / NVSwitch, with no collective call.

The reference has no counterpart (all its traffic is NCCL collectives,
reference distributed.py:102-120, backends/ctdg/runtime/memory.py:305-484).
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

_ALIGN = 256


@dataclass
class _Slot:
    offset: int
    shape: tuple[int, ...]
    dtype: torch.dtype


def _nbytes(shape: tuple[int, ...], dtype: torch.dtype) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n * torch.empty((), dtype=dtype).element_size()


class SymmetricArena:
    def __init__(self, specs: dict[str, tuple[tuple[int, ...], torch.dtype]], device: torch.device,
                 group: dist.ProcessGroup | None = None):
        # plain peer mappings only: no NVLink multicast object is bound to these buffers
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem

        self.device = torch.device(device)
        self.group = group or dist.group.WORLD
        self.slots: dict[str, _Slot] = {}
        off = 0
        for name, (shape, dtype) in specs.items():
            self.slots[name] = _Slot(off, tuple(int(s) for s in shape), dtype)
            off += (_nbytes(shape, dtype) + _ALIGN - 1) // _ALIGN * _ALIGN
        self.nbytes = max(off, _ALIGN)
        gname = self.group.group_name
        if hasattr(symm_mem, "is_symm_mem_enabled_for_group") and not symm_mem.is_symm_mem_enabled_for_group(gname):
            symm_mem.enable_symm_mem_for_group(gname)
        self.buffer = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=self.device)
        self.handle = symm_mem.rendezvous(self.buffer, self.group)
        self.rank = int(self.handle.rank)
        self.world_size = int(self.handle.world_size)
        self.base_ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.tensors: dict[str, torch.Tensor] = {}
        for name, sl in self.slots.items():
            nb = _nbytes(sl.shape, sl.dtype)
            self.tensors[name] = self.buffer[sl.offset:sl.offset + nb].view(sl.dtype).view(sl.shape)
        self._tables: dict[str, torch.Tensor] = {}

    def __getitem__(self, name: str) -> torch.Tensor:
        return self.tensors[name]

    def peer_table(self, name: str) -> torch.Tensor:
        """Device int64 [world]: address of every rank's copy of `name`."""
        if name not in self._tables:
            off = self.slots[name].offset
            self._tables[name] = torch.tensor([p + off for p in self.base_ptrs], dtype=torch.int64,
                                              device=self.device)
        return self._tables[name]

    def barrier_host(self) -> None:
        self.handle.barrier()
