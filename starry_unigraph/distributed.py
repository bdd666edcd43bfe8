"""Distributed context: torchrun environment -> config -> process group.

Reference behaviour (distributed.py:66-131): torchrun variables override the
``dist.*`` section, ``runtime.device == "cuda"`` becomes ``cuda:{local_rank}``
under torchrun, the process group is created from ``env://``. Here the process
group also gets a finite timeout so that a rank that stops participating turns
into an error on the others instead of a hang.
"""
from __future__ import annotations

import datetime
import os
from copy import deepcopy
from typing import Any

import torch

from starry_unigraph.types import DistributedContext


class DistRouteIndex:
    """Packed 64-bit route index: bits [0,48) local index, [48,62) partition id,
    bit 62 the "shared" flag (reference distributed.py:10-54, with its missing
    imports fixed)."""

    PART_SHIFT = 48
    SHARED_BIT = 62
    LOC_MASK = 0xFFFFFFFFFFFF
    PART_MASK = 0x3FFF

    def __init__(self, index: torch.Tensor, part_ids: torch.Tensor | None = None) -> None:
        if part_ids is None:
            self._data = index.long()
        else:
            index = index.long()
            part_ids = part_ids.long().to(index.device)
            self._data = (index & self.LOC_MASK) | ((part_ids & self.PART_MASK) << self.PART_SHIFT)

    @property
    def loc(self) -> torch.Tensor:
        return self._data & self.LOC_MASK

    @property
    def part(self) -> torch.Tensor:
        return (self._data >> self.PART_SHIFT) & self.PART_MASK

    def set_shared(self, index: slice | torch.Tensor) -> None:
        self._data[index] |= 1 << self.SHARED_BIT

    @property
    def is_shared(self) -> torch.Tensor:
        return ((self._data >> self.SHARED_BIT) & 1).to(torch.bool)

    @property
    def dist(self) -> torch.Tensor:
        return self._data

    @property
    def device(self) -> torch.device:
        return self._data.device

    @property
    def shape(self) -> torch.Size:
        return self._data.shape

    def to(self, device: Any) -> "DistRouteIndex":
        return DistRouteIndex(self._data.to(device))


def _env_int(name: str, default: int) -> int:
    value = os.environ.get(name)
    if value is None:
        return default
    try:
        return int(value)
    except ValueError:
        return default


def apply_distributed_env(config: dict[str, Any]) -> dict[str, Any]:
    merged = deepcopy(config)
    dist_cfg = merged.setdefault("dist", {})
    torchrun_active = any(k in os.environ for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK"))
    dist_cfg["backend"] = dist_cfg.get("backend", "nccl")
    dist_cfg["world_size"] = _env_int("WORLD_SIZE", int(dist_cfg.get("world_size", 1)))
    dist_cfg["rank"] = _env_int("RANK", int(dist_cfg.get("rank", 0)))
    dist_cfg["local_rank"] = _env_int("LOCAL_RANK", int(dist_cfg.get("local_rank", 0)))
    dist_cfg["local_world_size"] = _env_int("LOCAL_WORLD_SIZE", int(dist_cfg.get("local_world_size", 1)))
    dist_cfg["master_addr"] = os.environ.get("MASTER_ADDR", str(dist_cfg.get("master_addr", "127.0.0.1")))
    dist_cfg["master_port"] = _env_int("MASTER_PORT", int(dist_cfg.get("master_port", 29500)))
    dist_cfg["init_method"] = str(dist_cfg.get("init_method", "env://"))
    dist_cfg["launcher"] = "torchrun" if torchrun_active else str(dist_cfg.get("launcher", "single_process"))
    runtime_cfg = merged.setdefault("runtime", {})
    if runtime_cfg.get("device") == "cuda" and dist_cfg["launcher"] == "torchrun":
        runtime_cfg["device"] = f"cuda:{dist_cfg['local_rank']}"
    return merged


def build_distributed_context(config: dict[str, Any]) -> DistributedContext:
    d = config.get("dist", {})
    return DistributedContext(
        backend=str(d.get("backend", "nccl")),
        world_size=int(d.get("world_size", 1)),
        rank=int(d.get("rank", 0)),
        local_rank=int(d.get("local_rank", 0)),
        local_world_size=int(d.get("local_world_size", 1)),
        master_addr=str(d.get("master_addr", "127.0.0.1")),
        master_port=int(d.get("master_port", 29500)),
        init_method=str(d.get("init_method", "env://")),
        launcher=str(d.get("launcher", "single_process")),
        timeout_s=float(d.get("timeout_s", 600)),
    )


def initialize_distributed(ctx: DistributedContext) -> DistributedContext:
    if not ctx.is_distributed:
        return ctx
    import torch.distributed as dist

    if ctx.backend == "nccl" and torch.cuda.is_available():
        torch.cuda.set_device(ctx.local_rank)
    if not dist.is_initialized():
        kwargs: dict[str, Any] = dict(
            backend=ctx.backend,
            init_method=ctx.init_method,
            rank=ctx.rank,
            world_size=ctx.world_size,
            timeout=datetime.timedelta(seconds=ctx.timeout_s),
        )
        if ctx.backend == "nccl" and torch.cuda.is_available():
            kwargs["device_id"] = torch.device("cuda", ctx.local_rank)
        dist.init_process_group(**kwargs)
    ctx.initialized = True
    return ctx


def finalize_distributed(ctx: DistributedContext) -> None:
    if not ctx.initialized:
        return
    import torch.distributed as dist

    if dist.is_initialized():
        dist.destroy_process_group()
    ctx.initialized = False
