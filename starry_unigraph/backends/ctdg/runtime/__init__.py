from .cache import AdaParameter, CTDGHistoricalCache
from .data import CTDGDataBatch, TGTemporalDataset
from .factory import build_ctdg_runtime
from .memory import CTDGMemoryBank
from .models import (
    CTDG_MODEL_SPECS,
    CTDGLinkPredictor,
    CTDGMemoryUpdater,
    DenseBlock,
    JODIEMemoryUpdater,
    TemporalTransformerConv,
    build_ctdg_model,
    build_memory_updater,
)
from .route import AsyncExchangeHandle, CTDGFeatureRoute
from .runtime import CTDGOnlineRuntime, CTDGPreparedBatch
from .sampler import CTDGSampleOutput, NativeTemporalSampler, TemporalCSR
from .session import CTDGSession

__all__ = [
    "AdaParameter", "CTDGHistoricalCache", "CTDGDataBatch", "TGTemporalDataset", "build_ctdg_runtime",
    "CTDGMemoryBank", "CTDG_MODEL_SPECS", "CTDGLinkPredictor", "CTDGMemoryUpdater", "DenseBlock",
    "JODIEMemoryUpdater", "TemporalTransformerConv", "build_ctdg_model", "build_memory_updater",
    "AsyncExchangeHandle", "CTDGFeatureRoute", "CTDGOnlineRuntime", "CTDGPreparedBatch", "CTDGSampleOutput",
    "NativeTemporalSampler", "TemporalCSR", "CTDGSession",
]
