"""Utilities: tracing/timing, JSONL metrics, host-side fault injection and
peer heartbeats."""
from .faults import FaultInjector, Heartbeat, InjectedFault, PeerFailure
from .metrics import MetricsLogger
from .tracing import DeviceTimer, max_over_ranks, nvtx_range

__all__ = ["FaultInjector", "Heartbeat", "InjectedFault", "PeerFailure", "MetricsLogger", "DeviceTimer",
           "max_over_ranks", "nvtx_range"]
