from .comm_engine import CommEngine, CommHandle
from .spatial_plan import SpatialPlan
from .state_plan import StatePlan

__all__ = ["CommEngine", "CommHandle", "SpatialPlan", "StatePlan"]
