from .comm_plan import plan_from_routes
from .route import Route, RouteExchange, set_route_transport

__all__ = ["Route", "RouteExchange", "set_route_transport", "plan_from_routes"]
