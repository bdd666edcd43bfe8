from .adaptive import ChunkGenerator
from .generate_chunk import generate_chunks
from .time_split import adaptive_split

__all__ = ["ChunkGenerator", "generate_chunks", "adaptive_split"]
