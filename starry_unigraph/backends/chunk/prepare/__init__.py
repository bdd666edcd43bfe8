from .adaptive import ChunkGenerator, DependenceRoute, schedule
from .generate_chunk import generate_chunks
from .time_split import adaptive_split

__all__ = ["ChunkGenerator", "DependenceRoute", "schedule", "generate_chunks", "adaptive_split"]
