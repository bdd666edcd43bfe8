from .decay_cache import DecayCache
from .hot_cache import HotCache
from .partition_cache import PartitionCache

__all__ = ["DecayCache", "HotCache", "PartitionCache"]
