from .base import Runner, run_units
from .ctdg_runner import CTDGRunner
from .dtdg_runner import DTDGRunner

__all__ = ["Runner", "run_units", "CTDGRunner", "DTDGRunner"]
