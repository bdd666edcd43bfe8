from .bts_sampler import BTSNativeSampler, build_temporal_neighbor_block, is_bts_sampler_available

__all__ = ["BTSNativeSampler", "build_temporal_neighbor_block", "is_bts_sampler_available"]
