"""CTDG preprocessing (reference backends/ctdg/preprocess.py:15-137).

Writes meta/artifacts.json, partitions/manifest.json, routes/manifest.json,
sampling/index.json and, for multi-partition runs, partitions/node_parts.pt,
partitions/edge_parts.pt and sampling/boundaries.json (per-split batch plan).
"""
from __future__ import annotations

from pathlib import Path

import torch

from starry_unigraph.preprocess.base import ArtifactOutput, ArtifactPayload, GraphPreprocessor
from starry_unigraph.types import PreparedArtifacts, SessionContext

ARTIFACT_VERSION = 1


class CTDGPreprocessor(GraphPreprocessor):
    graph_mode = "ctdg"

    def _dataset(self, ctx: SessionContext):
        from .runtime.data import TGTemporalDataset

        cached = ctx.provider_state.get("ctdg_dataset")
        if cached is not None:
            return cached
        root = ctx.dataset_path or Path(ctx.config["data"]["root"]).expanduser().resolve()
        ds = TGTemporalDataset(root, ctx.config["data"]["name"], split_ratio=ctx.config.get("data", {}).get("split_ratio"),
                               config=ctx.config, raw=ctx.provider_state.get("raw_events"))
        ctx.provider_state["ctdg_dataset"] = ds
        return ds

    def prepare_raw(self, ctx: SessionContext) -> None:
        ctx.provider_state["ctdg_dataset_stats"] = self._dataset(ctx).describe()

    def build_partitions(self, ctx: SessionContext) -> None:
        from .preprocess_partition import build_round_robin_node_parts, derive_edge_parts, speed_partition

        ds = self._dataset(ctx)
        stats = ctx.provider_state["ctdg_dataset_stats"]
        algo = str(ctx.config["graph"]["partition"])
        num_parts = int(ctx.config["dist"]["world_size"])
        node_parts = edge_parts = None
        if algo.lower() == "speed":
            try:
                node_parts, edge_parts = speed_partition(ds, num_parts, ctx.config)
            except Exception as exc:  # reference behaviour: fall back to round-robin
                print(f"Warning: SPEED partitioning unavailable ({exc}); falling back to round-robin")
        if node_parts is None and num_parts > 1:
            node_parts = build_round_robin_node_parts(ds.num_nodes, num_parts)
            edge_parts = derive_edge_parts(ds.src, node_parts)
        if node_parts is not None:
            ctx.provider_state["node_parts"] = node_parts
            ctx.provider_state["edge_parts"] = edge_parts
            plan = {}
            bs = int(ctx.config["train"]["batch_size"])
            max_local = 0
            for split in ("train", "val", "test"):
                eids = ds.split_event_ids(split)
                counts = torch.bincount(edge_parts[eids], minlength=num_parts) if eids.numel() else \
                    torch.zeros(num_parts, dtype=torch.long)
                # largest per-rank share of any global window (sizes the static step buffers)
                gbs = bs * num_parts
                for st in range(0, int(eids.numel()), gbs):
                    w = torch.bincount(edge_parts[eids[st:st + gbs]], minlength=num_parts)
                    max_local = max(max_local, int(w.max()))
                plan[split] = {"num_events": int(eids.numel()), "global_batches_per_local_batch": num_parts,
                               "max_local_events_per_part": int(counts.max()) if counts.numel() else 0,
                               "min_local_events_per_part": int(counts.min()) if counts.numel() else 0}
            plan["max_local_batch"] = max_local
            ctx.provider_state["batch_plan"] = plan
            ctx.provider_state["max_local_batch"] = max_local
        ctx.provider_state["partition_manifest"] = {
            "graph_mode": "ctdg", "num_parts": num_parts, "partition_algo": algo, "num_nodes": stats["num_nodes"],
            "num_edges": stats["num_edges"], "has_node_parts": node_parts is not None,
            "has_edge_parts": edge_parts is not None,
            "edge_owner": "src_node_partition" if edge_parts is not None else None}

    def build_runtime_artifacts(self, ctx: SessionContext) -> PreparedArtifacts:
        from .runtime.route import CTDGFeatureRoute

        stats = ctx.provider_state["ctdg_dataset_stats"]
        route = CTDGFeatureRoute(str(ctx.config["graph"]["route"]), int(ctx.config["dist"]["world_size"]))
        meta = {"graph_mode": self.graph_mode, "artifact_version": ARTIFACT_VERSION,
                "num_parts": int(ctx.config["dist"]["world_size"]), "num_nodes": stats["num_nodes"],
                "num_edges": stats["num_edges"], "feature_dim": stats["edge_feat_dim"],
                "node_feat_dim": stats.get("node_feat_dim", 0), "task_type": ctx.config["model"]["task"],
                "feature_route_plan": route.describe(), "partition_algo": str(ctx.config["graph"]["partition"]),
                "edge_owner": "src_node_partition", "batch_alignment": "global_time_window"}
        outputs = [ArtifactOutput("partitions/manifest.json", ctx.provider_state["partition_manifest"]),
                   ArtifactOutput("routes/manifest.json", route.describe()),
                   ArtifactOutput("sampling/index.json", {"dataset": ctx.config["data"]["name"], **stats})]
        if "node_parts" in ctx.provider_state:
            outputs.append(ArtifactOutput("partitions/node_parts.pt", ctx.provider_state["node_parts"], "torch"))
            meta["has_node_parts"] = True
        if ctx.provider_state.get("edge_parts") is not None:
            outputs.append(ArtifactOutput("partitions/edge_parts.pt", ctx.provider_state["edge_parts"], "torch"))
            meta["has_edge_parts"] = True
        if "batch_plan" in ctx.provider_state:
            outputs.append(ArtifactOutput("sampling/boundaries.json", ctx.provider_state["batch_plan"]))
            meta["max_local_batch"] = ctx.provider_state.get("max_local_batch")
        return self.emit_artifacts(ctx, ArtifactPayload(provider_meta=meta, outputs=outputs))
