from .preprocess import CTDGPreprocessor
from .runtime import *  # noqa: F401,F403
from .runtime import __all__ as _rt_all

__all__ = ["CTDGPreprocessor", *_rt_all]
