"""DTDG preprocessing: raw events (or a synthetic snapshot sequence) ->
partitions -> Flare artifacts (reference backends/dtdg/preprocess.py:22-170).

Artifacts: meta/artifacts.json, partitions/manifest.json, routes/manifest.json,
flare/manifest.json and one flare/part_NNN.pth (``PartitionData``) per rank.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any

from starry_unigraph.data import build_snapshot_dataset_from_events, load_raw_temporal_events
from starry_unigraph.preprocess.base import (ArtifactOutput, ArtifactPayload, GraphPreprocessor,
                                             load_prepared_from_disk, read_artifact_meta)
from starry_unigraph.types import PreparedArtifacts, SessionContext

from .dtdg_prepare import build_dtdg_partitions, build_flare_partition_data_list
from .types import DTDGPartitionBook, SnapshotRoutePlan

ARTIFACT_VERSION = 1


def validate_artifacts(prepared: PreparedArtifacts, expected_graph_mode: str, expected_num_parts: int | None = None):
    from starry_unigraph.session import validate_artifacts as _v

    return _v(prepared, expected_graph_mode, expected_num_parts)


def _synthetic_snapshots(config: dict[str, Any]) -> dict[str, Any]:
    from dataclasses import replace

    from starry_unigraph.data.synthetic import DTDG_PRESETS, SnapshotSpec, snapshot_sequence

    spec = dict(config.get("data", {}).get("synthetic") or {})
    preset = spec.pop("preset", None)
    base = DTDG_PRESETS[preset] if preset else SnapshotSpec(num_nodes=1000, num_snapshots=8,
                                                            edges_per_snapshot=5000, churn=0.3, feat_dim=16)
    spec = replace(base, **spec)
    snaps = snapshot_sequence(spec)
    return {"num_nodes": spec.num_nodes, "num_edges": spec.edges_per_snapshot * spec.num_snapshots,
            "num_snapshots": len(snaps), "num_life_edges": spec.edges_per_snapshot * spec.num_snapshots,
            "dataset": snaps, "source": f"synthetic:{preset or 'custom'}", "node_feat_dim": spec.feat_dim,
            "node_feature_source": "synthetic", "label": spec.label}


class BaseDTDGPreprocessor(GraphPreprocessor):
    graph_mode = "dtdg"
    artifact_dirs = ("meta", "partitions", "routes", "snapshots", "flare")

    def prepare_raw(self, ctx: SessionContext) -> None:
        cfg = ctx.config
        if str(cfg.get("data", {}).get("format", "auto")).lower() == "synthetic":
            raw = _synthetic_snapshots(cfg)
        else:
            root = ctx.dataset_path if ctx.dataset_path is not None else Path(cfg["data"]["root"]).expanduser().resolve()
            events = load_raw_temporal_events(root=root, dataset_name=cfg["data"]["name"], config=cfg)
            raw = build_snapshot_dataset_from_events(events=events, snaps=int(cfg["train"]["snaps"]))
        ctx.provider_state["raw_dataset"] = raw
        ctx.provider_state["raw_stats"] = {k: raw.get(k, 0) for k in ("num_nodes", "num_edges", "num_snapshots",
                                                                      "node_feat_dim", "node_feature_source")}

    def build_partitions(self, ctx: SessionContext) -> None:
        raw = ctx.provider_state["raw_dataset"]
        num_parts = int(ctx.config["dist"]["world_size"])
        algo = str(ctx.config["graph"]["partition"])
        result = build_dtdg_partitions(raw, num_parts, algo, ctx.config)
        ctx.provider_state["partition_result"] = result
        ctx.provider_state["partition_manifest"] = {"num_parts": num_parts, "partition_algo": algo,
                                                    "num_nodes": raw["num_nodes"], "num_edges": raw["num_edges"],
                                                    "num_snapshots": raw["num_snapshots"]}

    def _route_plan(self, ctx: SessionContext) -> SnapshotRoutePlan:
        return SnapshotRoutePlan(route_type=ctx.config["graph"]["route"], cache_policy=ctx.config["runtime"]["cache"])

    def _provider_meta(self, ctx: SessionContext, plan: SnapshotRoutePlan) -> dict[str, Any]:
        book = DTDGPartitionBook(num_parts=ctx.config["dist"]["world_size"],
                                 partition_algo=ctx.config["graph"]["partition"],
                                 snapshot_count=int(ctx.provider_state["raw_stats"].get("num_snapshots", 0)))
        raw = ctx.provider_state["raw_dataset"]
        return {"graph_mode": self.graph_mode, **book.describe(),
                "feature_dim": ctx.provider_state["raw_stats"].get("node_feat_dim", 0), "edge_feat_dim": 0,
                "label_dim": 1, "label": raw.get("label", "regression"), "task_type": ctx.config["model"]["task"],
                "artifact_version": ARTIFACT_VERSION, "snapshot_route_plan": plan.describe(),
                "pipeline": "flare_native",
                "node_feature_source": ctx.provider_state["raw_stats"].get("node_feature_source", "unknown")}


class FlareDTDGPreprocessor(BaseDTDGPreprocessor):
    def build_runtime_artifacts(self, ctx: SessionContext) -> PreparedArtifacts:
        raw = ctx.provider_state["raw_dataset"]
        plan = self._route_plan(ctx)
        parts = build_flare_partition_data_list(raw, ctx.provider_state["partition_result"], plan, ctx.config)
        outputs = [ArtifactOutput("partitions/manifest.json", ctx.provider_state["partition_manifest"]),
                   ArtifactOutput("routes/manifest.json", plan.describe()),
                   ArtifactOutput("flare/manifest.json", {"pipeline": "flare_native", "num_parts": len(parts),
                                                          "files": [f"part_{i:03d}.pth" for i in range(len(parts))]})]
        outputs += [ArtifactOutput(f"flare/part_{i:03d}.pth", p, serializer="torch") for i, p in enumerate(parts)]
        # global node -> partition map (the NVLink halo path addresses peer rows with it)
        outputs.append(ArtifactOutput("partitions/node_parts.pt",
                                      ctx.provider_state["partition_result"]["node_parts"].long(), "torch"))
        meta = self._provider_meta(ctx, plan)
        meta["has_node_parts"] = True
        return self.emit_artifacts(ctx, ArtifactPayload(provider_meta=meta, outputs=outputs))


__all__ = ["FlareDTDGPreprocessor", "BaseDTDGPreprocessor", "validate_artifacts", "load_prepared_from_disk",
           "read_artifact_meta", "ARTIFACT_VERSION"]
