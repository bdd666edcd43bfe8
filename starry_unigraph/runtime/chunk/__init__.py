from .session_loader import ChunkRuntimeLoader
from .training import run_chunk_eval_step, run_chunk_train_step

__all__ = ["ChunkRuntimeLoader", "run_chunk_train_step", "run_chunk_eval_step"]
