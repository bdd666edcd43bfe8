"""Unified runtime layer: pipeline engine, backend/state protocols, caches,
communication engine, runners, chunk runtime, reusable modules."""
