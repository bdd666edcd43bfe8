"""Chunk-mode preprocessing (reference preprocess/chunk.py:19-116, which only
wrote manifests): builds time-slice x node-cluster chunks with the native
adaptive split and partitioner, assigns clusters to ranks round-robin, and
writes snapshots/manifest.json, clusters/part_NNN/cluster_manifest.json and
clusters/part_NNN/chunks.pt."""
from __future__ import annotations

from pathlib import Path
from typing import Any

from starry_unigraph.data.chunk_builder import ChunkBuilder
from starry_unigraph.data.chunk_data import ChunkData
from starry_unigraph.preprocess.base import ArtifactOutput, ArtifactPayload, GraphPreprocessor
from starry_unigraph.types import PreparedArtifacts, SessionContext

ARTIFACT_VERSION = 1


class ChunkPreprocessor(GraphPreprocessor):
    graph_mode = "chunk"
    artifact_dirs = ("meta", "partitions", "routes", "snapshots", "clusters")

    def prepare_raw(self, ctx: SessionContext) -> None:
        from starry_unigraph.backends.ctdg.runtime.data import TGTemporalDataset

        root = ctx.dataset_path or Path(ctx.config["data"]["root"]).expanduser().resolve()
        ds = TGTemporalDataset(root, ctx.config["data"]["name"], config=ctx.config,
                               raw=ctx.provider_state.get("raw_events"))
        ctx.provider_state["chunk_dataset"] = ds

    def build_partitions(self, ctx: SessionContext) -> None:
        from starry_unigraph.backends.chunk.prepare.adaptive import ChunkGenerator, schedule

        ds = ctx.provider_state["chunk_dataset"]
        c = ctx.config.get("chunk", {})
        gen = ChunkGenerator(num_clusters=int(c.get("node_clusters", 8)), time_slices=int(c.get("time_slices", 16)),
                             adaptive=bool(c.get("adaptive", False)),
                             info_loss_threshold=float(c.get("info_loss_threshold", 0.3)),
                             edge_share=float(c.get("edge_share", 0.9)))
        out = gen.generate(ds.src, ds.dst, ds.ts, ds.num_nodes, eid=ds.event_ids)
        chunks = out["chunks"]
        W = int(ctx.config["dist"]["world_size"])
        parts = [[ch for ch in chunks if ch.chunk_id[1] % W == p] for p in range(W)]
        ctx.provider_state["chunk_parts"] = parts
        ctx.provider_state["chunk_routes"] = out["routes"]
        ctx.provider_state["chunk_order"] = schedule(out["routes"])
        ctx.provider_state["chunk_builder"] = out["builder"] | {"num_clusters": out["num_clusters"],
                                                                "cross_ratio": out["cross_ratio"]}
        if W > 1:  # a node is owned by the rank that runs its cluster's chunks
            node_parts = out["clusters"].long() % W
            ctx.provider_state["node_parts"] = node_parts
            ctx.provider_state["edge_parts"] = node_parts[ds.src.long()]

    def build_runtime_artifacts(self, ctx: SessionContext) -> PreparedArtifacts:
        parts = ctx.provider_state["chunk_parts"]
        ds = ctx.provider_state["chunk_dataset"]
        W = len(parts)
        node_parts = ctx.provider_state.get("node_parts")
        meta: dict[str, Any] = {"graph_mode": "chunk", "artifact_version": ARTIFACT_VERSION, "num_parts": W,
                                "num_nodes": ds.num_nodes, "num_edges": ds.num_edges,
                                "builder": ctx.provider_state["chunk_builder"], "pipeline": "chunked",
                                "has_node_parts": node_parts is not None, "has_edge_parts": node_parts is not None}
        slices = sorted({ch.chunk_id[0] for p in parts for ch in p})
        routes = ctx.provider_state["chunk_routes"]
        outputs = [ArtifactOutput("partitions/manifest.json", {"num_parts": W, "partition_algo": "cluster_round_robin"}),
                   ArtifactOutput("routes/manifest.json", {"route_type": ctx.config["graph"]["route"],
                                                           "dependence_routes": [r.describe() for r in routes],
                                                           "order": [list(cid) for cid in ctx.provider_state["chunk_order"]]}),
                   ArtifactOutput("snapshots/manifest.json", {"time_slices": slices, "num_chunks": sum(map(len, parts))})]
        if node_parts is not None:
            outputs.append(ArtifactOutput("partitions/node_parts.pt", node_parts, "torch"))
            outputs.append(ArtifactOutput("partitions/edge_parts.pt", ctx.provider_state["edge_parts"], "torch"))
        for p, chunks in enumerate(parts):
            outputs.append(ArtifactOutput(f"clusters/part_{p:03d}/cluster_manifest.json",
                                          {"part": p, "chunks": [list(c.chunk_id) for c in chunks],
                                           "chunk_events": [c.num_events for c in chunks],
                                           "events": sum(c.num_events for c in chunks)}))
            outputs.append(ArtifactOutput(f"clusters/part_{p:03d}/chunks.pt", ChunkData(chunks), serializer="torch"))
        return self.emit_artifacts(ctx, ArtifactPayload(provider_meta=meta, outputs=outputs))
