"""Route re-export (the reference keeps a byte-identical copy here)."""
from starry_unigraph.backends.dtdg.runtime.route import Route, RouteExchange, set_route_transport

__all__ = ["Route", "RouteExchange", "set_route_transport"]
