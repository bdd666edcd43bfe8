"""Process topology: torchrun environment -> ``dist`` config section -> process group.

Behaviour kept from the reference (distributed.py:66-131): the torchrun variables
override the ``dist`` section, a CUDA run under torchrun is pinned to
``cuda:{local_rank}``, and the process group comes from ``env://``. In addition the
process group is created with a finite timeout (``dist.timeout_s``), so a rank
that stops taking part in collectives surfaces as an error on the others instead
of a hang.

``DistRouteIndex`` is the reference's packed route index (distributed.py:10-54):
one int64 per entry holding a local row, the owning partition and a "shared"
flag. The reference declares it with missing imports; here it is usable.
"""
from __future__ import annotations

import dataclasses
import datetime
import os
from copy import deepcopy
from typing import Any, Callable

import torch

from starry_unigraph.types import DistributedContext

# ---------------------------------------------------------------------------
# packed route index
# ---------------------------------------------------------------------------
_LOC_BITS = 48      # local row: bits [0, 48)
_PART_BITS = 14     # owning partition: bits [48, 62)
_SHARED_BIT = 62    # entry also held by other partitions


def _field_mask(bits: int) -> int:
    return (1 << bits) - 1


def pack_route_index(local: torch.Tensor, part: torch.Tensor | int) -> torch.Tensor:
    """int64 codes of (local row, partition) pairs (the shared flag clear)."""
    local = local.long()
    part_t = torch.as_tensor(part, dtype=torch.long, device=local.device)
    return (local & _field_mask(_LOC_BITS)) | ((part_t & _field_mask(_PART_BITS)) << _LOC_BITS)


class DistRouteIndex:
    """Packed (local row, partition, shared) codes with the reference's accessors
    (``loc``, ``part``, ``is_shared``, ``dist``, ``set_shared``, ``to``)."""

    PART_SHIFT = _LOC_BITS
    SHARED_BIT = _SHARED_BIT
    LOC_MASK = _field_mask(_LOC_BITS)
    PART_MASK = _field_mask(_PART_BITS)

    def __init__(self, index: torch.Tensor, part_ids: torch.Tensor | None = None) -> None:
        # one argument: already packed codes; two: rows and their partitions
        self._codes = index.long() if part_ids is None else pack_route_index(index, part_ids)

    def _field(self, shift: int, bits: int) -> torch.Tensor:
        return (self._codes >> shift) & _field_mask(bits)

    @property
    def loc(self) -> torch.Tensor:
        return self._field(0, _LOC_BITS)

    @property
    def part(self) -> torch.Tensor:
        return self._field(_LOC_BITS, _PART_BITS)

    @property
    def is_shared(self) -> torch.Tensor:
        return self._field(_SHARED_BIT, 1).bool()

    def set_shared(self, index: slice | torch.Tensor) -> None:
        self._codes[index] |= 1 << _SHARED_BIT

    @property
    def dist(self) -> torch.Tensor:
        return self._codes

    @property
    def device(self) -> torch.device:
        return self._codes.device

    @property
    def shape(self) -> torch.Size:
        return self._codes.shape

    def to(self, device: Any) -> "DistRouteIndex":
        return DistRouteIndex(self._codes.to(device))


# ---------------------------------------------------------------------------
# torchrun environment
# ---------------------------------------------------------------------------
def _as_int(text: str | None) -> int | None:
    try:
        return None if text is None else int(text)
    except ValueError:
        return None


# dist key <- (environment variable, parser); unset or unparsable variables keep the config value
_ENV_OVERRIDES: dict[str, tuple[str, Callable[[str | None], Any]]] = {
    "world_size": ("WORLD_SIZE", _as_int),
    "rank": ("RANK", _as_int),
    "local_rank": ("LOCAL_RANK", _as_int),
    "local_world_size": ("LOCAL_WORLD_SIZE", _as_int),
    "master_addr": ("MASTER_ADDR", lambda t: t),
    "master_port": ("MASTER_PORT", _as_int),
}

# dist key -> (default, type) of every DistributedContext field read from the config
_DIST_DEFAULTS: dict[str, tuple[Any, type]] = {
    "backend": ("nccl", str),
    "world_size": (1, int),
    "rank": (0, int),
    "local_rank": (0, int),
    "local_world_size": (1, int),
    "master_addr": ("127.0.0.1", str),
    "master_port": (29500, int),
    "init_method": ("env://", str),
    "launcher": ("single_process", str),
    "timeout_s": (600, float),
}


def _under_torchrun() -> bool:
    return any(os.environ.get(v) is not None for v in ("WORLD_SIZE", "RANK", "LOCAL_RANK"))


def apply_distributed_env(config: dict[str, Any]) -> dict[str, Any]:
    """Copy of `config` whose ``dist`` section reflects the torchrun variables."""
    out = deepcopy(config)
    section = out.setdefault("dist", {})
    for key, (default, kind) in _DIST_DEFAULTS.items():
        if key != "timeout_s":
            section[key] = kind(section.get(key, default))
    for key, (var, parse) in _ENV_OVERRIDES.items():
        value = parse(os.environ.get(var))
        if value is not None:
            section[key] = value
    if _under_torchrun():
        section["launcher"] = "torchrun"
        runtime = out.setdefault("runtime", {})
        if runtime.get("device") == "cuda":
            runtime["device"] = f"cuda:{section['local_rank']}"
    return out


def build_distributed_context(config: dict[str, Any]) -> DistributedContext:
    section = config.get("dist", {})
    values = {key: kind(section.get(key, default)) for key, (default, kind) in _DIST_DEFAULTS.items()}
    known = {f.name for f in dataclasses.fields(DistributedContext)}
    return DistributedContext(**{k: v for k, v in values.items() if k in known})


# ---------------------------------------------------------------------------
# process group
# ---------------------------------------------------------------------------
def initialize_distributed(ctx: DistributedContext) -> DistributedContext:
    """Create the default process group once (an existing one is adopted)."""
    if not ctx.is_distributed:
        return ctx
    import torch.distributed as dist

    on_gpu = ctx.backend == "nccl" and torch.cuda.is_available()
    if on_gpu:
        torch.cuda.set_device(ctx.local_rank)
        # a collective that fails or outlives dist.timeout_s aborts its communicator and raises in
        # the caller (no process teardown), so the session's own error paths run
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "3")
    if not dist.is_initialized():
        extra = {"device_id": torch.device("cuda", ctx.local_rank)} if on_gpu else {}
        dist.init_process_group(backend=ctx.backend, init_method=ctx.init_method, rank=ctx.rank,
                                world_size=ctx.world_size, timeout=datetime.timedelta(seconds=ctx.timeout_s),
                                **extra)
    ctx.initialized = True
    return ctx


def finalize_distributed(ctx: DistributedContext) -> None:
    if not ctx.initialized:
        return
    import torch.distributed as dist

    if dist.is_initialized():
        dist.destroy_process_group()
    ctx.initialized = False
