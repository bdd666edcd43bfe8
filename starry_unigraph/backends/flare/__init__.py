"""Backward-compatible names of the Flare DTDG pipeline (reference backends/flare/__init__.py)."""
from starry_unigraph.backends.dtdg import *  # noqa: F401,F403
from starry_unigraph.backends.dtdg import __all__  # noqa: F401
from starry_unigraph.data.partition import PartitionData, RouteData, TensorData  # noqa: F401
