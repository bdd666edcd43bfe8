"""starry_unigraph: distributed temporal GNN training (CTDG + DTDG) for B200.

Public entry points: ``SchedulerSession`` (prepare / train / predict), the
``python -m starry_unigraph`` CLI, and the stable re-export surface in
``starry_unigraph.lib_stable``.
"""
from .session import SchedulerSession

__version__ = "0.2.0"

__all__ = ["SchedulerSession", "__version__"]


def __getattr__(name):  # lazy: lib_stable imports the whole framework
    if name == "lib_stable":
        import importlib

        return importlib.import_module("starry_unigraph.lib_stable")
    raise AttributeError(name)
