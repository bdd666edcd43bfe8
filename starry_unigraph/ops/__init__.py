"""Python handles on the in-tree native extensions.

``cuda_ext()`` returns ``starry_unigraph._C`` (the sm_100a kernels). It raises
when a CUDA device is present but the extension is missing, so a GPU run never
falls back silently to a library path. ``native_ext()`` returns the host C++
module ``starry_unigraph._native`` (temporal sampler, TPPR, time split,
partitioner) or None when it was not built.
"""
from __future__ import annotations

import importlib
from contextlib import contextmanager
from functools import lru_cache

import torch


class ExtensionMissing(RuntimeError):
    pass


@lru_cache(maxsize=1)
def _load(name: str):
    return importlib.import_module(name)


def cuda_ext():
    try:
        return _load("starry_unigraph._C")
    except ImportError as exc:  # pragma: no cover - exercised on GPU boxes without a build
        raise ExtensionMissing(
            "starry_unigraph._C is not built; run `python setup.py build_ext --inplace` "
            "(sm_100a CUDA kernels are required on CUDA devices)"
        ) from exc


def has_cuda_ext() -> bool:
    try:
        cuda_ext()
        return True
    except ExtensionMissing:
        return False


def native_ext():
    try:
        return _load("starry_unigraph._native")
    except ImportError:
        return None


def check_status(clear: bool = True) -> None:
    """Raise if a kernel recorded a bounded-wait timeout or bad index (synchronises)."""
    if not torch.cuda.is_available():
        return
    code = int(cuda_ext().status_read(clear))
    if code != 0:
        names = {1: "operand stage wait timed out", 2: "free stage wait timed out", 3: "accumulator wait timed out",
                 4: "TMEM drain wait timed out", 5: "index out of range", 6: "peer flag wait timed out",
                 7: "size above compiled bound"}
        raise RuntimeError(f"device status {code}: {names.get(code, 'unknown')}")


@contextmanager
def gemm_precision(tf32: bool):
    """Run the enclosed GEMM launches with tf32 (True) or bf16 (False) tensor-core
    operands and restore the previous setting afterwards. The setting is
    process-wide (autograd issues backward kernels from its own threads), so a
    step that selects its precision this way leaves other callers unaffected."""
    C = cuda_ext()
    prev = bool(C.gemm_precision_tf32())
    C.set_gemm_precision(bool(tf32))
    try:
        yield
    finally:
        C.set_gemm_precision(prev)
