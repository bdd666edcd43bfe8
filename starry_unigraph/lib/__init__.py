from .loader import load_adaptive_split_module, load_bts_sampler_module

__all__ = ["load_bts_sampler_module", "load_adaptive_split_module"]
