"""Graph-mode backends: ``ctdg`` (online event streams), ``dtdg`` (Flare snapshots), ``chunk``."""
