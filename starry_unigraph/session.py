"""SchedulerSession: the public prepare / train / predict lifecycle
(reference session.py:25-439).

``from_config`` merges the YAML config over the defaults, applies torchrun
variables, validates, resolves the model family and task; ``prepare_data``
runs the mode's preprocessor; ``build_runtime`` loads the artifacts and builds
the CTDG online runtime or the DTDG Flare runtime; ``run_epoch`` returns the
reference's dict (split, steps, local_steps, loss, local_loss, metrics,
elapsed_s = max over ranks, local_elapsed_s, outputs).
"""
from __future__ import annotations

import time
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from starry_unigraph.checkpoint import load_checkpoint, save_checkpoint
from starry_unigraph.config.schema import detect_graph_mode, load_config, validate_config
from starry_unigraph.distributed import apply_distributed_env, build_distributed_context
from starry_unigraph.preprocess.base import load_prepared_from_disk, read_artifact_meta
from starry_unigraph.registry import ModelRegistry, TaskRegistry
from starry_unigraph.types import PredictionResult, PreparedArtifacts, RuntimeBundle, SessionContext

ARTIFACT_VERSION = 1


def validate_artifacts(prepared: PreparedArtifacts, expected_graph_mode: str,
                       expected_num_parts: int | None = None) -> dict[str, Any]:
    """Reference backends/dtdg/preprocess.py:27-53."""
    if not prepared.meta_path.exists():
        raise FileNotFoundError(f"Missing artifacts metadata: {prepared.meta_path}")
    meta = read_artifact_meta(prepared.meta_path)
    if meta.get("artifact_version") != ARTIFACT_VERSION:
        raise RuntimeError(f"Artifact version mismatch: expected {ARTIFACT_VERSION}, got {meta.get('artifact_version')}")
    if meta.get("graph_mode") != expected_graph_mode:
        raise RuntimeError(f"Artifact graph_mode mismatch: expected {expected_graph_mode}, got {meta.get('graph_mode')}")
    if expected_num_parts is not None and meta.get("num_parts") != expected_num_parts:
        raise RuntimeError(f"Artifact num_parts mismatch: expected {expected_num_parts}, got {meta.get('num_parts')}")
    for sub in ("partitions", "routes"):
        path = prepared.directories.get(sub, prepared.meta_path.parent.parent / sub) / "manifest.json"
        if not path.exists():
            raise FileNotFoundError(f"Missing {sub[:-1]} manifest: {path}")
    return meta


class SchedulerSession:
    def __init__(self, session_ctx: SessionContext, model_spec: Any, task_adapter: Any):
        self.ctx = session_ctx
        self.model_spec = model_spec
        self.task_adapter = task_adapter
        self.current_epoch = 0
        self.global_step = 0
        self.runtime = RuntimeBundle()
        self.snapshot_core: Any = None
        self.ctdg_session: Any = None
        self.prepared: PreparedArtifacts | None = None
        self.pipeline_engine: Any = None
        from starry_unigraph.utils import FaultInjector

        self._faults = FaultInjector.from_env()
        self._heartbeat = None
        self._hb_last = 0.0
        self._metrics = None

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_config(cls, config_or_path: str | Path | dict[str, Any], dataset_path: str | Path | None = None,
                    overrides: dict[str, Any] | None = None) -> "SchedulerSession":
        config = apply_distributed_env(load_config(config_or_path, overrides=overrides))
        warnings = validate_config(config)
        model_spec = ModelRegistry.resolve(model_name=config["model"]["name"], family=config["model"]["family"])
        task_cls = TaskRegistry.resolve(config["model"]["task"])
        artifact_root = (Path("artifacts") / config["data"]["name"]).resolve()
        ctx = SessionContext(config=config, project_root=Path.cwd(),
                             dataset_path=Path(dataset_path).expanduser().resolve() if dataset_path else None,
                             artifact_root=artifact_root, dist=build_distributed_context(config), warnings=warnings)
        return cls(session_ctx=ctx, model_spec=model_spec, task_adapter=task_cls())

    @property
    def graph_mode(self) -> str:
        return detect_graph_mode(self.ctx.config)

    def _device(self) -> str:
        base = str(self.ctx.config["runtime"]["device"])
        if base == "cuda" and dist.is_available() and dist.is_initialized():
            return f"cuda:{self.ctx.dist.local_rank}"
        if base.startswith("cuda") and not torch.cuda.is_available():
            return "cpu"
        return base

    # ------------------------------------------------------------------ prepare
    def prepare_data(self) -> PreparedArtifacts:
        mode = self.graph_mode
        if mode == "ctdg":
            from starry_unigraph.backends.ctdg.preprocess import CTDGPreprocessor

            pre = CTDGPreprocessor()
        elif mode == "dtdg":
            from starry_unigraph.backends.dtdg.preprocess import FlareDTDGPreprocessor

            pre = FlareDTDGPreprocessor()
        elif mode == "chunk":
            from starry_unigraph.preprocess.chunk import ChunkPreprocessor

            pre = ChunkPreprocessor()
        else:
            raise ValueError(f"Unknown graph_mode for preprocessing: {mode!r}")
        self.prepared = pre.run(self.ctx)
        self.ctx.prepared_artifacts = self.prepared
        return self.prepared

    # ------------------------------------------------------------------ runtime
    def _load_partition(self):
        flare_dir = self.prepared.directories.get("flare", self.ctx.artifact_root / "flare")
        if not (flare_dir / "manifest.json").exists():
            raise FileNotFoundError(f"Missing flare manifest: {flare_dir / 'manifest.json'}")
        part_id = min(self.ctx.dist.rank, self.ctx.dist.world_size - 1)
        path = flare_dir / f"part_{part_id:03d}.pth"
        if not path.exists():
            raise FileNotFoundError(f"Missing flare partition artifact: {path}")
        return path, torch.load(path, weights_only=False)

    def build_runtime(self) -> RuntimeBundle:
        if self.prepared is None:
            self.prepared = load_prepared_from_disk(self.ctx.artifact_root)
        self.ctx.prepared_artifacts = self.prepared
        mode = self.prepared.provider_meta.get("graph_mode")
        device = self._device()
        if mode == "ctdg":
            from starry_unigraph.backends.ctdg.runtime.session import CTDGSession

            if "max_local_batch" in self.prepared.provider_meta:
                self.ctx.provider_state["max_local_batch"] = self.prepared.provider_meta["max_local_batch"]
            self.ctdg_session = CTDGSession()
            self.ctdg_session.build_runtime(self.ctx)
            self.runtime = self.ctdg_session._runtime
        elif mode == "dtdg":
            from starry_unigraph.backends.dtdg import FlareRuntimeLoader, init_flare_training

            validate_artifacts(self.prepared, "dtdg", self.ctx.dist.world_size)
            path, part = self._load_partition()
            self.snapshot_core = FlareRuntimeLoader.from_partition_data(
                data=part, device=device, rank=self.ctx.dist.rank, world_size=self.ctx.dist.world_size,
                config=self.ctx.config)
            self.runtime = RuntimeBundle(state={"graph_mode": "dtdg"})
            init_flare_training(runtime=self.runtime, session_ctx=self.ctx, partition_data=part, device=device)
            self._maybe_peer_halo(device)
            from starry_unigraph.runtime.route.comm_plan import plan_from_routes

            if getattr(part, "routes", None) is not None:
                self.runtime.state["halo_volume"] = plan_from_routes(part.routes)
            self.runtime.state.update({"flare_partition_path": str(path),
                                       "window_state": self.snapshot_core.describe_window_state(),
                                       "snapshot_state": self.snapshot_core.dump_state(),
                                       "route_cache": self.snapshot_core.describe_route_cache()})
        elif mode == "chunk":
            from starry_unigraph.runtime.chunk import ChunkRuntimeLoader

            validate_artifacts(self.prepared, "chunk", self.ctx.dist.world_size)
            from starry_unigraph.backends.ctdg.runtime.factory import build_ctdg_runtime

            self.snapshot_core = ChunkRuntimeLoader.from_prepared_artifacts(
                prepared_dir=self.ctx.artifact_root, device=device, rank=self.ctx.dist.rank,
                world_size=self.ctx.dist.world_size, config=self.ctx.config)
            online, bundle = build_ctdg_runtime(self.ctx)
            self.snapshot_core.attach_ctdg(online)
            self.runtime = bundle
            self.runtime.state.update({"graph_mode": "chunk", "chunk_manifest": self.snapshot_core.chunk_manifest})
        else:
            raise ValueError(f"Unknown graph_mode: {mode}")
        return self.runtime

    def _maybe_peer_halo(self, device: str) -> None:
        """Multi-GPU DTDG with ``comm.path: p2p``: halo rows are read from peer memory
        inside the aggregation kernel (starry_unigraph.parallel.halo)."""
        from starry_unigraph.parallel.halo import PeerHaloContext, halo_width, set_halo_context

        set_halo_context(None)
        if not (self.ctx.dist.is_distributed and dist.is_initialized() and str(device).startswith("cuda")):
            return
        if str(self.ctx.config.get("comm", {}).get("path", "p2p")) != "p2p":
            return
        path = self.prepared.directories.get("partitions", self.ctx.artifact_root / "partitions") / "node_parts.pt"
        if not path.exists():
            return
        node_parts = torch.load(path, weights_only=True)
        width = halo_width(self.runtime.model, int(self.ctx.config["model"]["hidden_dim"]))
        hc = PeerHaloContext(node_parts, width, torch.device(device))
        set_halo_context(hc)
        self.runtime.state["halo"] = {"transport": "nvlink_p2p", "world": hc.world, "features": hc.F}

    def build_pipeline_engine(self, model: Any = None):
        """The unified engine over this session's backend. Without `model` it drives the
        session's own runtime (``RuntimeStepModel``): its epochs train and evaluate
        exactly as ``run_epoch`` does, unit by unit."""
        from starry_unigraph.runtime.backend_adapters import (ChunkGraphBackend, CTDGGraphBackend,
                                                              DummyStateManager, FlareGraphBackend, RuntimeStepModel)
        from starry_unigraph.runtime.engine import PipelineEngine

        if self.prepared is None:
            self.prepared = load_prepared_from_disk(self.ctx.artifact_root)
        if self.ctdg_session is None and self.snapshot_core is None:
            self.build_runtime()
        mode = self.prepared.provider_meta.get("graph_mode")
        if mode == "ctdg":
            from starry_unigraph.runtime.state import CTDGStateManager

            backend = CTDGGraphBackend(self.ctdg_session, max_batch=int(self.ctx.config["train"]["batch_size"]))
            state_manager = CTDGStateManager(self.ctdg_session.online_runtime.memory)
        elif mode == "dtdg":
            from starry_unigraph.runtime.state import DTDGStateManager

            backend = FlareGraphBackend(self.snapshot_core)
            state_manager = DTDGStateManager()
        else:
            backend = ChunkGraphBackend(self.snapshot_core)
            state_manager = DummyStateManager()
        self.pipeline_engine = PipelineEngine(backend=backend, state_manager=state_manager,
                                              model=model if model is not None else RuntimeStepModel(self),
                                              task_adapter=self.task_adapter, device=self._device(),
                                              optimizer=self.runtime.optimizer)
        return self.pipeline_engine

    def build_runner(self):
        """Runner of the session's mode (``runtime.runner``): build_sequence ->
        prepare_data -> sync_data -> compute -> post_compute per unit of work,
        driven by ``starry_unigraph.runtime.runner.run_units``."""
        from starry_unigraph.runtime.runner import CTDGRunner, DTDGRunner

        if self.ctdg_session is None and self.snapshot_core is None:
            self.build_runtime()
        if self.ctdg_session is not None:
            return CTDGRunner(self.ctdg_session.online_runtime, int(self.ctx.config["train"]["batch_size"]))
        return DTDGRunner(self.snapshot_core, self.runtime)

    # ------------------------------------------------------------------ step hooks
    def _between_steps(self, step: int) -> None:
        """Runs on the host before every step: injected faults (SU_FAULT) and the
        peer heartbeat (dist.heartbeat_s > 0), so a rank learns that a peer is gone
        before it enters the next collective."""
        rank = self.ctx.dist.rank
        if self._faults:
            self._faults.maybe_inject(rank, step)
        hb_s = float(self.ctx.config.get("dist", {}).get("heartbeat_s", 0) or 0)
        if hb_s > 0 and self.ctx.dist.is_distributed and dist.is_initialized():
            now = time.time()
            if self._heartbeat is None:
                from starry_unigraph.utils import Heartbeat

                store = dist.distributed_c10d._get_default_store()
                self._heartbeat = Heartbeat(store, rank, self.ctx.dist.world_size, timeout_s=hb_s)
            if now - self._hb_last >= min(1.0, hb_s / 4):
                self._heartbeat.beat(step)
                self._heartbeat.check()
                self._hb_last = now

    def _log_metrics(self, **record: Any) -> None:
        path = self.ctx.config.get("runtime", {}).get("metrics_path")
        if not path:
            return
        if self._metrics is None:
            from starry_unigraph.utils import MetricsLogger

            self._metrics = MetricsLogger(path, rank=self.ctx.dist.rank)
        self._metrics.log(**record)

    # ------------------------------------------------------------------ epochs
    def _summarise(self, split: str, outputs: list[dict[str, Any]], losses: list[float], elapsed: float):
        res = self._summarise_impl(split, outputs, losses, elapsed)
        self._log_metrics(epoch=self.current_epoch, split=split, steps=res["steps"], loss=res["loss"],
                          global_loss=res["global_loss"], metrics=res["metrics"], elapsed_s=res["elapsed_s"])
        return res

    def _summarise_impl(self, split: str, outputs: list[dict[str, Any]], losses: list[float], elapsed: float):
        metric_acc: dict[str, list[float]] = {}
        for item in outputs:
            for k, v in item.get("meta", {}).get("metrics", {}).items():
                metric_acc.setdefault(k, []).append(float(v))
        loss_sum = float(sum(losses))
        steps = len(losses) if split != "train" else len(outputs)
        tot_loss, tot_steps, max_elapsed = self._distributed_epoch_stats(loss_sum, steps, elapsed)
        loss = tot_loss / tot_steps if tot_steps else 0.0
        # "loss" keeps the reference's figure (sum over ranks / total steps). A DTDG rank's loss
        # is already weighted by its share of the nodes, so that figure is the global mean
        # divided by the world size; "global_loss" is the global mean itself.
        shares = self.ctdg_session is None and self.runtime is not None and \
            "part_loss_scale" in getattr(self.runtime, "state", {})
        world = self.ctx.dist.world_size if self.ctx.dist.is_distributed and dist.is_initialized() else 1
        return {"split": split, "steps": tot_steps, "local_steps": steps,
                "loss": loss, "global_loss": loss * world if shares else loss,
                "local_loss": loss_sum / steps if steps else 0.0,
                "metrics": {k: float(sum(v) / len(v)) for k, v in metric_acc.items() if v},
                "elapsed_s": max_elapsed, "local_elapsed_s": elapsed, "outputs": outputs}

    def run_epoch(self, split: str = "train") -> dict[str, Any]:
        if self.ctx.dist.is_distributed and dist.is_initialized():
            # ranks start the epoch's first step together: its device-side peer barriers then
            # wait only for the GPU work of the step, not for host-side work of a lagging rank
            dist.barrier()
        if self.ctdg_session is not None:
            rt = self.ctdg_session.online_runtime
            train = split == "train"
            start = time.perf_counter()
            if rt.engine is not None:
                base = self.global_step
                res = rt.run_split_device(split, int(self.ctx.config["train"]["batch_size"]), train,
                                          on_step=lambda i: self._between_steps(base + i))
                outputs = [{"loss": l, "meta": {"split": split, "batch_size": n,
                                                "metrics": ({"ap": m[0], "auc": m[1], "mrr": m[2]} if n else {})}}
                           for l, m, n in zip(res["losses"], res["metrics"], res["sizes"])]
            else:
                it = self.ctdg_session.iter_train(self.ctx) if train else self.ctdg_session.iter_eval(self.ctx, split)
                outputs = []
                for i, b in enumerate(it):
                    self._between_steps(self.global_step + i)
                    outputs.append(self.ctdg_session.train_step(b) if train else self.ctdg_session.eval_step(b))
            elapsed = time.perf_counter() - start
            if train:
                self.global_step += len(outputs)
                self.current_epoch += 1
            losses = [float(o["loss"]) for o in outputs if "loss" in o]
            return self._summarise(split, outputs, losses, elapsed)
        assert self.snapshot_core is not None, "Call build_runtime() first"
        if split == "train":
            iterator = self.snapshot_core.iter_train(split=split)
        else:
            self.runtime.state.pop("eval_rnn_state", None)
            iterator = self.snapshot_core.iter_eval(split=split)
        start = time.perf_counter()
        outputs = []
        for i, batch in enumerate(iterator):
            self._between_steps(self.global_step if split == "train" else i)
            if split == "train":
                outputs.append(self.snapshot_core.run_train_step(self.runtime, batch))
                self.global_step += 1
            else:
                outputs.append(self.snapshot_core.run_eval_step(self.runtime, batch))
        elapsed = time.perf_counter() - start
        if split == "train":
            self.current_epoch += 1
        losses = [float(self.task_adapter.compute_loss(o)) for o in outputs if "loss" in o]
        return self._summarise(split, outputs, losses, elapsed)

    def run_task(self) -> dict[str, Any]:
        self.build_runtime()
        train_summary, eval_summary = [], []
        t0 = time.perf_counter()
        for epoch in range(int(self.ctx.config["train"]["epochs"])):
            train_summary.append(self.run_epoch(split="train"))
            if (epoch + 1) % int(self.ctx.config["train"]["eval_interval"]) == 0:
                eval_summary.append(self.run_epoch(split="val"))
        return {"epochs": self.current_epoch, "train": train_summary, "eval": eval_summary,
                "train_total_s": sum(x.get("elapsed_s", 0.0) for x in train_summary),
                "train_total_local_s": sum(x.get("local_elapsed_s", 0.0) for x in train_summary),
                "run_task_total_s": time.perf_counter() - t0, "warnings": self.ctx.warnings}

    def evaluate(self, split: str = "test") -> dict[str, Any]:
        return self.run_epoch(split=split)

    def predict(self, split: str = "test") -> PredictionResult:
        if self.ctdg_session is not None:
            rt = self.ctdg_session.online_runtime
            preds: list[float] = []
            targets: list[int] = []
            if rt.engine is not None:
                res = rt.run_split_device(split, int(self.ctx.config["train"]["batch_size"]), train=False,
                                          collect_predictions=True)
                for p in res["predictions"]:
                    preds.extend(p)
                    targets.extend([1] * len(p))
            else:
                for batch in self.ctdg_session.iter_predict(self.ctx, split=split):
                    out = self.ctdg_session.predict_step(batch)
                    preds.extend(out.get("predictions", []))
                    targets.extend(out.get("targets", []) or [])
            return PredictionResult(predictions=preds, targets=targets or None,
                                    meta={"split": split, "graph_mode": self.model_spec.graph_mode})
        assert self.snapshot_core is not None, "Call build_runtime() first"
        self.runtime.state.pop("eval_rnn_state", None)
        preds, targets = [], []
        for batch in self.snapshot_core.iter_predict(split=split):
            out = self.snapshot_core.run_predict_step(self.runtime, batch)
            preds.extend(out.get("predictions", []))
            if out.get("targets") is not None:
                targets.extend(out["targets"])
        return PredictionResult(predictions=preds, targets=targets or None,
                                meta={"split": split, "graph_mode": self.model_spec.graph_mode})

    def _distributed_epoch_stats(self, loss_sum: float, steps: int, elapsed: float) -> tuple[float, int, float]:
        if not self.ctx.dist.is_distributed or not dist.is_initialized():
            return loss_sum, steps, elapsed
        dev = f"cuda:{self.ctx.dist.local_rank}" if dist.get_backend() == "nccl" else "cpu"
        stats = torch.tensor([loss_sum, float(steps), elapsed], dtype=torch.float64, device=dev)
        dist.all_reduce(stats[0:2], op=dist.ReduceOp.SUM)
        dist.all_reduce(stats[2:3], op=dist.ReduceOp.MAX)
        return float(stats[0]), int(stats[1]), float(stats[2])

    # ------------------------------------------------------------------ checkpoints
    @staticmethod
    def rank_state_path(path: str | Path, rank: int) -> Path:
        """File of one rank's exact-resume state next to checkpoint `path`."""
        path = Path(path)
        return path.with_name(f"{path.name}.rank{rank}")

    def _ctdg_rank_state(self) -> dict[str, Any]:
        """This rank's share of the CTDG training state: the memory-bank rows it
        holds (rows that were ever written: on the NVLink path these are the
        nodes it owns, on the collective path also its view of remote rows), its
        optimizer moments (sharded by rank on the NVLink path), the random
        streams, the fused step's counter and the historical-cache rows."""
        rt = self.ctdg_session.online_runtime
        mb = rt.memory
        rt.memory.wait_pending_syncs()  # pushes submitted after the last step land in the tables first
        touched = (mb.memory_ts >= 0) | (mb.mailbox_ts != 0).any(dim=1) | (mb.next_mail_pos != 0)
        idx = torch.nonzero(touched).view(-1)
        bank = {"index": idx.cpu()}
        for n in ("memory", "memory_ts", "mailbox", "mailbox_ts", "next_mail_pos"):
            bank[n] = getattr(mb, n)[idx].cpu()
        rng: dict[str, Any] = {"torch": torch.get_rng_state(), "negatives": rt._gen.get_state()}
        if torch.cuda.is_available():
            rng["cuda"] = torch.cuda.get_rng_state_all()
        engine = rt.engine
        state: dict[str, Any] = {"rank": self.ctx.dist.rank, "world_size": self.ctx.dist.world_size,
                                 "memory_bank": bank, "optimizer": self.runtime.optimizer.state_dict(), "rng": rng}
        if engine is not None:
            state["engine_step"] = engine.step_ctr.detach().cpu()  # dropout / negative streams are keyed on it
            peer = engine.peer
            if peer is not None and peer.hist_cache is not None:
                state["hist_cache"] = [t.detach().cpu() for t in peer.hist_cache]
        return state

    def _load_ctdg_rank_state(self, state: dict[str, Any]) -> None:
        rt = self.ctdg_session.online_runtime
        if int(state["world_size"]) != self.ctx.dist.world_size:
            raise RuntimeError(f"exact-resume state was written by {state['world_size']} ranks, "
                               f"this run has {self.ctx.dist.world_size}")
        mb = rt.memory
        bank = state["memory_bank"]
        with torch.no_grad():
            mb.memory.zero_()
            mb.memory_ts.fill_(-1.0)
            mb.mailbox.zero_()
            mb.mailbox_ts.zero_()
            mb.next_mail_pos.zero_()
            idx = bank["index"].to(mb.memory.device)
            for n in ("memory", "memory_ts", "mailbox", "mailbox_ts", "next_mail_pos"):
                getattr(mb, n)[idx] = bank[n].to(mb.memory.device)
        self.runtime.optimizer.load_state_dict(state["optimizer"])
        rng = state["rng"]
        torch.set_rng_state(rng["torch"])
        rt._gen.set_state(rng["negatives"])
        if "cuda" in rng and torch.cuda.is_available():
            torch.cuda.set_rng_state_all(rng["cuda"])
        engine = rt.engine
        if engine is not None:
            if "engine_step" in state:
                engine.step_ctr.copy_(state["engine_step"])
            peer = engine.peer
            if peer is not None:
                peer.arena["claim"].zero_()  # claim keys of the abandoned run would outrank resumed mails
                if peer.hist_cache is not None and "hist_cache" in state:
                    for dst, src in zip(peer.hist_cache, state["hist_cache"]):
                        dst.copy_(src)

    def save_checkpoint(self, path: str | Path, *, exact_resume: bool = False) -> Path:
        """Reference keys in `path` (rank 0 writes it: all ranks hold identical
        parameters). With ``exact_resume`` (CTDG) every rank also writes
        ``<path>.rank<r>`` with its own memory-bank rows, optimizer moments and
        random streams. On several ranks this is a collective: every rank calls it,
        and it returns once the files are complete."""
        path = Path(path)
        distributed = self.ctx.dist.is_distributed and dist.is_initialized()
        rank = dist.get_rank() if distributed else 0
        if self.ctdg_session is not None:
            engine = getattr(self.ctdg_session.online_runtime, "engine", None)
            if engine is not None:
                engine.drain()  # multi-GPU: the peers' last pushes have landed in this rank's tables
            if exact_resume:
                path.parent.mkdir(parents=True, exist_ok=True)
                save_checkpoint(self.rank_state_path(path, rank), self._ctdg_rank_state())
            if rank == 0:
                path.parent.mkdir(parents=True, exist_ok=True)
                extra = {"epoch": self.current_epoch, "global_step": self.global_step}
                if exact_resume:
                    extra["exact_resume"] = {"world_size": self.ctx.dist.world_size}
                self.ctdg_session.save_checkpoint(path, extra)
            if distributed:
                dist.barrier()
            return path
        opt = self.runtime.optimizer
        # every rank: on the NVLink path the optimizer moments are sharded and gathered here
        opt_state = opt.state_dict() if opt is not None else None
        if rank == 0:  # one writer (all ranks hold identical parameters)
            path.parent.mkdir(parents=True, exist_ok=True)
            model = self.runtime.model.module if hasattr(self.runtime.model, "module") else self.runtime.model
            payload = {"model_state": {k: v.detach().cpu() for k, v in model.state_dict().items()},
                       "optimizer_state": opt_state,
                       "scheduler_state": self.runtime.scheduler, "config": self.ctx.config,
                       "epoch": self.current_epoch, "global_step": self.global_step}
            save_checkpoint(path, payload)
        if distributed:
            dist.barrier()  # the file is complete before any rank goes on (and may read it)
        return path

    def load_checkpoint(self, path: str | Path) -> dict[str, Any]:
        if self.ctdg_session is None and self.snapshot_core is None:
            self.build_runtime()
        distributed = self.ctx.dist.is_distributed and dist.is_initialized()
        if self.ctdg_session is not None:
            engine = getattr(self.ctdg_session.online_runtime, "engine", None)
            if engine is not None:
                engine.drain()
            ckpt = self.ctdg_session.load_checkpoint(path)
            self.current_epoch = int(ckpt.get("epoch", self.current_epoch))
            self.global_step = int(ckpt.get("global_step", self.global_step))
            if isinstance(ckpt.get("exact_resume"), dict):
                rank_file = self.rank_state_path(path, self.ctx.dist.rank)
                if not rank_file.exists():
                    raise FileNotFoundError(f"exact-resume checkpoint without this rank's state: {rank_file}")
                self._load_ctdg_rank_state(load_checkpoint(rank_file))
            if engine is not None:
                torch.cuda.synchronize(engine.device)
            if distributed:
                dist.barrier()  # no rank steps (and reads peers' tables) before all have loaded
            return ckpt
        payload = load_checkpoint(path)
        state = payload.get("model_state")
        model = self.runtime.model.module if hasattr(self.runtime.model, "module") else self.runtime.model
        if isinstance(state, torch.nn.Module):  # reference payloads pickle the live module
            inner = state.module if hasattr(state, "module") else state
            state = inner.state_dict()
        if state is not None:
            with torch.no_grad():
                for k, v in model.state_dict().items():
                    v.copy_(state[k])
        opt_state = payload.get("optimizer_state")
        if opt_state is not None and self.runtime.optimizer is not None:
            if isinstance(opt_state, dict):  # written by this framework: a mismatch is an error
                self.runtime.optimizer.load_state_dict(opt_state)
            else:
                # the reference pickles its live torch optimizer, whose state layout need not
                # match this framework's flat optimizer: keep fresh moments and say so
                try:
                    self.runtime.optimizer.load_state_dict(opt_state.state_dict())
                except Exception as exc:  # noqa: BLE001
                    import warnings

                    warnings.warn(f"optimizer state of the checkpoint not restored ({exc}); "
                                  "training resumes with fresh Adam moments")
        self.runtime.scheduler = payload.get("scheduler_state")
        self.current_epoch = int(payload.get("epoch", 0))
        self.global_step = int(payload.get("global_step", 0))
        return payload
