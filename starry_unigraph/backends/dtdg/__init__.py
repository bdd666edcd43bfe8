from .preprocess import BaseDTDGPreprocessor, FlareDTDGPreprocessor, load_prepared_from_disk, validate_artifacts
from .runtime import *  # noqa: F401,F403
from .runtime import __all__ as _rt_all
from .types import DTDGPartitionBook

__all__ = ["BaseDTDGPreprocessor", "FlareDTDGPreprocessor", "load_prepared_from_disk", "validate_artifacts",
           "DTDGPartitionBook", *_rt_all]
