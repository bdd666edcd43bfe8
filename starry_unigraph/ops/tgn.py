"""Fused sm_100a TGN training / evaluation step.

One step (reference backends/ctdg/runtime/runtime.py:225-328) is a fixed
sequence of kernel launches over static device buffers, so it can be captured
once per (split, mode) in a CUDA graph and replayed:

  prep -> sample -> GRU memory update (fused scatter) -> mailbox write ->
  Q/KV projections (gather + time encoding fused into the GEMM producers) ->
  attention -> W_out + dropout + ReLU + LayerNorm -> link projections ->
  BCE loss + logits gradient (+ AP/AUC) -> [backward GEMMs -> gradient sync ->
  fused Adam].

Shapes are padded to ``bmax`` events and ``rmax = 2 * bmax`` roots; the real
counts live on the device, so the host never synchronises inside a step.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

import torch

from starry_unigraph.ops import cuda_ext
from starry_unigraph.ops.flat import FlatParams, FusedAdam


class _TracingOps:
    """Proxy of the extension module for one traced step: every op call gets an NVTX
    range and a pair of CUDA events on the stream it runs on."""

    def __init__(self, C: Any) -> None:
        self._C = C
        self.records: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def __getattr__(self, name: str):
        fn = getattr(self._C, name)
        if not callable(fn) or name in ("launch_count", "status_read", "set_gemm_precision", "gemm_precision_tf32"):
            return fn

        def traced(*args, **kwargs):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push(name)
            a.record()
            out = fn(*args, **kwargs)
            b.record()
            torch.cuda.nvtx.range_pop()
            self.records.append((name, a, b))
            return out

        return traced


@dataclass
class TGNShapes:
    bmax: int
    k: int
    D: int
    E: int
    T: int
    Do: int
    H: int
    K: int

    @property
    def rmax(self) -> int:
        return 2 * self.bmax

    @property
    def slot_width(self) -> int:
        return 2 * self.D + self.E


class TGNCudaEngine:
    def __init__(
        self,
        *,
        model: torch.nn.Module,
        updater: torch.nn.Module,
        memory: Any,
        edge_feat: torch.Tensor,
        neg_pool: torch.Tensor,
        csr_provider: Callable[[str], Any],
        bmax: int,
        fanout: int,
        policy: str,
        lr: float,
        dropout: float,
        att_dropout: float,
        num_head: int,
        seed: int = 0,
        use_graphs: bool = True,
        grad_sync: Callable[[torch.Tensor], float] | None = None,
        peer: Any = None,
        precision: str = "tf32",
    ) -> None:
        self.C = cuda_ext()
        if precision not in ("tf32", "bf16"):
            raise ValueError(f"runtime.precision must be tf32 or bf16, got {precision!r}")
        # tensor-core operand precision of every GEMM of the step (fp32 storage and accumulation)
        self.tf32 = precision == "tf32"
        self.model = model
        self.updater = updater
        self.memory = memory
        # multi-GPU write-back overlapped with the next step (reference ctdg.async_sync)
        self.async_sync = bool(getattr(memory, "async_sync", True))
        dev = memory.memory.device
        self.device = dev
        D = memory.hidden_dim
        E = memory.edge_feat_dim
        # "tgn": attention embedding over sampled neighbours + GRU memory updater;
        # "jodie": time-projection embedding of the memory + tanh-RNN updater (no sampling)
        self.kind = "jodie" if not hasattr(model, "conv") else "tgn"
        if self.kind == "jodie":
            if memory.mailbox_slots != 1:
                raise ValueError("the fused JODIE step keeps one mailbox slot per node")
            self.s = TGNShapes(bmax=int(bmax), k=1, D=D, E=E, T=1, Do=D, H=1, K=1)
        else:
            conv = model.conv
            self.s = TGNShapes(bmax=int(bmax), k=int(fanout), D=D, E=E, T=conv.dim_time, Do=conv.dim_out,
                               H=int(num_head), K=memory.mailbox_slots)
            if self.s.T <= 0:
                raise ValueError("the fused TGN step requires dim_time > 0")
        self.policy = 0 if policy == "recent" else 1
        self.dropout = float(dropout)
        self.att_dropout = float(att_dropout)
        self.seed = int(seed)
        self.use_graphs = bool(use_graphs)
        self.csr_provider = csr_provider
        self.grad_sync = grad_sync
        # bf16 edge features stay bf16 on the device (the operand producers, the
        # mailbox kernels and the peer mail write read them as bf16); others are fp32
        ef = edge_feat.to(dev)
        if ef.dtype not in (torch.float32, torch.bfloat16):
            ef = ef.float()
        if ef.dim() == 1:
            ef = ef.view(-1, 1)
        self.efeat = ef.contiguous()
        self.neg_pool = neg_pool.to(dev).long().contiguous()
        # parameters live in one flat buffer (fused Adam, one-buffer gradient sync)
        self.flat = FlatParams([model], dev)
        self.peer = peer
        if peer is not None:
            # gradients and parameters in symmetric buffers: each rank reduces its shard of
            # every rank's gradient and stores the updated shard into every rank's parameters
            self.flat.rebind_grad(peer.arena["grad"])
            self.flat.rebind_data(peer.arena["param"])
        self.opt = FusedAdam(self.flat, lr=lr)
        self._alloc()
        self._pd = None
        if peer is not None:
            self.mem_new = torch.zeros(self.s.rmax, self.s.D, dtype=torch.float32, device=dev)
            self._pd = peer.descriptor(self.stamp, self.node2root, self.step_ctr, self.mem_new)
        self._graphs: dict[tuple[str, bool], torch.cuda.CUDAGraph] = {}
        self._warm: dict[tuple[str, bool], int] = {}
        self._launches: dict[tuple[str, bool], int] = {}  # library kernel launches per step, counted eagerly
        self._side = torch.cuda.Stream(self.device)  # weight-gradient GEMMs overlap the data-gradient chain

    # ------------------------------------------------------------------ buffers
    def _alloc(self) -> None:
        s, dev = self.s, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        i64 = dict(dtype=torch.int64, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        N = self.memory.num_nodes
        B, R, k = s.bmax, s.rmax, s.k
        self.ev_src = torch.zeros(B, **i64)
        self.ev_dst = torch.zeros(B, **i64)
        self.ev_ts = torch.zeros(B, **f32)
        self.ev_eid = torch.zeros(B, **i64)
        self.n_ev = torch.zeros(1, **i32)
        self.stamp = torch.zeros(N, **i32)
        self.node2root = torch.zeros(N, **i32)
        self.step_ctr = torch.zeros(1, **i64)
        self.roots = torch.full((R,), -1, **i64)
        self.n_roots = torch.zeros(1, **i32)
        self.src_idx = torch.zeros(B, **i32)
        self.dst_idx = torch.zeros(B, **i32)
        self.neg = torch.zeros(B, **i64)
        self.neg_idx = torch.zeros(B, **i32)
        self.ts_max = torch.zeros(1, **f32)
        self.root_ts = torch.zeros(1, **i64)
        self.win_key = torch.zeros(2 * R, **i64)
        self.win = torch.zeros(2 * R, **i32)
        self.cnt = torch.zeros(2 * R, **i32)
        self.nbr = torch.zeros(R * k, **i64)
        self.nbr_eid = torch.zeros(R * k, **i64)
        self.nbr_dt = torch.zeros(R * k, **f32)
        self.nbr_cnt = torch.zeros(R, **i32)
        self.edge_total = torch.zeros(1, **i32)
        self.agg_buf = torch.zeros(R, s.D, **f32)
        self.agg_buf2 = torch.zeros(R, s.D, **f32)
        self.mem_prev = torch.zeros(R, s.D, **f32)
        self.Q = torch.zeros(R, s.Do, **f32)
        self.KV = torch.zeros(R * k, 2 * s.Do, **f32)
        self.att_p = torch.zeros(R * k, s.H, **f32)
        self.agg = torch.zeros(R, s.Do, **f32)
        self.out = torch.zeros(R, s.Do, **f32)
        self.xsave = torch.zeros(R, s.Do, **f32)
        self.mean = torch.zeros(R, **f32)
        self.rstd = torch.zeros(R, **f32)
        self.P = torch.zeros(R, 2 * s.D, **f32)
        self.scores = torch.zeros(2 * B, **f32)
        self.loss = torch.zeros(1, **f32)
        self.metrics = torch.zeros(3, **f32)
        self.dP = torch.zeros(R, 2 * s.D, **f32)
        self.dout = torch.zeros(R, s.D, **f32)
        self.dpre = torch.zeros(R, s.Do, **f32)
        self.dagg = torch.zeros(R, s.Do, **f32)
        self.dKV = torch.zeros(R * k, 2 * s.Do, **f32)
        self.dQ = torch.zeros(R, s.Do, **f32)
        self.Mt = torch.zeros(2 * s.Do, s.T, **f32)  # time-encoder products of the W_kv weight gradient
        self.M1 = torch.zeros(2 * s.Do, s.T, **f32)
        if self.kind == "jodie":
            self.prev_ts = torch.zeros(R, **f32)
            self.jdt = torch.zeros(R, **f32)

    # ------------------------------------------------------------------ inputs
    def load_batch(self, src: torch.Tensor, dst: torch.Tensor, ts: torch.Tensor, eid: torch.Tensor) -> None:
        """Copy one batch into the static input buffers (H2D when the inputs are on the host)."""
        n = int(src.numel())
        if n > self.s.bmax:
            raise ValueError(f"batch of {n} events exceeds bmax={self.s.bmax}")
        nb = src.device.type == "cpu" and src.is_pinned()
        self.ev_src[:n].copy_(src, non_blocking=nb)
        self.ev_dst[:n].copy_(dst, non_blocking=nb)
        self.ev_ts[:n].copy_(ts, non_blocking=nb)
        self.ev_eid[:n].copy_(eid, non_blocking=nb)
        self.n_ev.fill_(n)

    def load_packed(self, packed_host: torch.Tensor, n: int) -> None:
        """Single H2D copy of a pinned int64 [4, bmax] pack (src, dst, ts-bits, eid) plus the count."""
        self._packed_dev = getattr(self, "_packed_dev", None)
        if self._packed_dev is None:
            self._packed_dev = torch.zeros(4, self.s.bmax, dtype=torch.int64, device=self.device)
        self._packed_dev.copy_(packed_host, non_blocking=True)
        self.ev_src.copy_(self._packed_dev[0])
        self.ev_dst.copy_(self._packed_dev[1])
        self.ev_ts.copy_(self._packed_dev[2].to(torch.int32).view(torch.float32))
        self.ev_eid.copy_(self._packed_dev[3])
        self.n_ev.fill_(n)

    # ------------------------------------------------------------------ step
    def _params(self):
        m, u = self.model, self.updater
        c = m.conv
        return m, u, c

    def _forward_jodie(self, split: str, train: bool) -> None:
        """JODIE step: memory update (tanh RNN) -> mailbox -> time projection of the
        updated memory -> link scores / BCE -> [projection and link gradients -> Adam]."""
        C, s = self.C, self.s
        m, u = self.model, self.updater
        mem = self.memory
        C.tgn_prep(self.ev_src, self.ev_dst, self.ev_ts, self.n_ev, self.neg_pool, self.stamp, self.node2root,
                   self.step_ctr, self.seed, self.roots, self.n_roots, self.src_idx, self.dst_idx, self.neg,
                   self.neg_idx, self.ts_max, self.root_ts, self.win_key, self.win, self.cnt)
        if self.peer is not None:
            self.peer.wait_claim(C, self.roots, self.n_roots, self.win, self.ev_eid, self.ev_ts)
        cell = u.memory_cell
        C.tgn_rnn_memory_update(self.roots, self.n_roots, mem.mailbox, mem.memory, mem.memory_ts, self.ts_max,
                                cell.weight_ih, cell.weight_hh, cell.bias_ih, cell.bias_hh, self.mem_prev,
                                self.prev_ts, self._pd)
        if self.peer is None:
            C.tgn_mailbox_write(self.roots, self.n_roots, self.win, self.cnt, self.src_idx, self.dst_idx,
                                self.ev_eid, self.ev_ts, self.mem_prev, self.efeat, s.E, mem.mailbox, mem.mailbox_ts,
                                mem.next_mail_pos)
        tp = m.time_proj
        C.jodie_project(self.roots, self.n_roots, mem.memory, self.prev_ts, self.root_ts, float(m.dt_scale),
                        tp.weight, tp.bias, self.out, self.jdt, self._pd)
        C.tgn_link_proj(self.out, self.n_roots, m.src_fc.weight, m.src_fc.bias, m.dst_fc.weight, m.dst_fc.bias,
                        self.P)
        self.loss.zero_()
        if train:
            self.flat.zero_grad()
            self.dP.zero_()
        gw = {n.split(".", 1)[1]: v for n, v in self.flat.grad_views.items()}
        C.tgn_link_loss(self.P, self.src_idx, self.dst_idx, self.neg_idx, self.n_ev, m.dst_fc.bias, m.out_fc.weight,
                        m.out_fc.bias, train, self.scores, self.loss, self.dP, gw["out_fc.weight"], gw["out_fc.bias"],
                        gw["dst_fc.bias"])
        # AP/AUC/MRR only feed reporting: computed on the side stream, overlapping the backward pass
        main = torch.cuda.current_stream(self.device)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            C.tgn_metrics(self.scores, self.n_ev, self.metrics)
        if train:
            C.tgn_link_proj_bwd(self.dP, self.out, self.n_roots, m.src_fc.weight, m.dst_fc.weight,
                                gw["src_fc.weight"], gw["src_fc.bias"], gw["dst_fc.weight"], gw["dst_fc.bias"],
                                self.dout, 0)
            C.jodie_project_bwd(self.roots, self.n_roots, mem.memory, self.jdt, self.dout,
                                gw["time_proj.weight"], gw["time_proj.bias"], self._pd)
            if self.peer is None:
                scale = 1.0
                if self.grad_sync is not None:
                    scale = self.grad_sync(self.flat.grad)
                self.opt.step(grad_scale=scale)
        main.wait_stream(self._side)
        if self.peer is not None:
            self._peer_sync(train)

    def _forward(self, split: str, train: bool) -> None:
        # host-side precision switch: picks the kernels issued (and captured) below, then restored
        prev = bool(self.C.gemm_precision_tf32())
        self.C.set_gemm_precision(self.tf32)
        try:
            if self.kind == "jodie":
                return self._forward_jodie(split, train)
            return self._forward_tgn(split, train)
        finally:
            self.C.set_gemm_precision(prev)

    def _forward_tgn(self, split: str, train: bool) -> None:
        C, s = self.C, self.s
        m, u, c = self._params()
        mem = self.memory
        csr = self.csr_provider(split)
        drop = self.dropout if train else 0.0
        adrop = self.att_dropout if train else 0.0
        C.tgn_prep(self.ev_src, self.ev_dst, self.ev_ts, self.n_ev, self.neg_pool, self.stamp, self.node2root,
                   self.step_ctr, self.seed, self.roots, self.n_roots, self.src_idx, self.dst_idx, self.neg,
                   self.neg_idx, self.ts_max, self.root_ts, self.win_key, self.win, self.cnt)
        C.tgn_sample(self.roots, self.n_roots, self.root_ts, csr.rowptr, csr.nbr, csr.eid, csr.ts, s.k, self.policy,
                     self.seed, self.step_ctr, self.nbr, self.nbr_eid, self.nbr_dt, self.nbr_cnt, self.edge_total)
        if self.peer is not None:  # previous step's pushes complete on every rank; post this step's claims
            self.peer.wait_claim(C, self.roots, self.n_roots, self.win, self.ev_eid, self.ev_ts)
        g = u.mail_aggregator
        cell = u.memory_cell
        C.tgn_memory_update(self.roots, self.n_roots, mem.mailbox, s.K, mem.memory, mem.memory_ts, self.ts_max,
                            g.weight_ih_l0, g.weight_hh_l0, g.bias_ih_l0, g.bias_hh_l0, cell.weight_ih,
                            cell.weight_hh, cell.bias_ih, cell.bias_hh, self.agg_buf, self.agg_buf2, self.mem_prev, self._pd)
        if self.peer is None:  # multi-GPU: the mailbox is written to the owners after the step (_peer_sync)
            C.tgn_mailbox_write(self.roots, self.n_roots, self.win, self.cnt, self.src_idx, self.dst_idx,
                                self.ev_eid, self.ev_ts, self.mem_prev, self.efeat, s.E, mem.mailbox, mem.mailbox_ts,
                                mem.next_mail_pos)
        te = c.time_enc.w
        C.tgn_attn_proj(mem.memory, self.roots, self.n_roots, self.nbr, self.nbr_eid, self.nbr_dt, self.nbr_cnt,
                        self.efeat, s.E, te.weight, te.bias, c.w_q.weight, c.w_q.bias, c.w_k.weight, c.w_k.bias,
                        c.w_v.weight, c.w_v.bias, self.Q, self.KV, self._pd)
        C.tgn_attn_fwd(self.Q, self.KV, self.nbr_cnt, self.n_roots, s.H, adrop, self.seed, self.step_ctr, self.att_p,
                       self.agg)
        C.tgn_out_fwd(self.agg, mem.memory, self.roots, self.n_roots, c.w_out.weight, c.w_out.bias,
                      c.layer_norm.weight, c.layer_norm.bias, drop, self.seed, self.step_ctr, self.edge_total,
                      self.out, self.xsave, self.mean, self.rstd, self._pd)
        C.tgn_link_proj(self.out, self.n_roots, m.src_fc.weight, m.src_fc.bias, m.dst_fc.weight, m.dst_fc.bias,
                        self.P)
        self.loss.zero_()
        if train:
            self.flat.zero_grad()
            self.dP.zero_()
        G = self.flat.grad_views
        gw = {n.split(".", 1)[1]: v for n, v in G.items()}
        C.tgn_link_loss(self.P, self.src_idx, self.dst_idx, self.neg_idx, self.n_ev, m.dst_fc.bias, m.out_fc.weight,
                        m.out_fc.bias, train, self.scores, self.loss, self.dP, gw["out_fc.weight"], gw["out_fc.bias"],
                        gw["dst_fc.bias"])
        # AP/AUC/MRR only feed reporting: computed on the side stream, overlapping the backward pass
        main = torch.cuda.current_stream(self.device)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            C.tgn_metrics(self.scores, self.n_ev, self.metrics)
        if train:
            self._backward(gw)
        main.wait_stream(self._side)
        if self.peer is not None:
            self._peer_sync(train)

    def _peer_sync(self, train: bool) -> None:
        """Multi-GPU end of step over NVLink (see starry_unigraph.parallel.ctdg_peer):
        barrier A, then the memory write-back and the claim winners' mailbox slots on
        the side stream while the main stream runs the reduce-scatter + Adam +
        all-gather of the parameters, then the end-of-step signal, whose wait is
        fused into the next step's claims."""
        C, s, P = self.C, self.s, self.peer
        P.barrier(C)
        main = torch.cuda.current_stream(self.device)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            C.tgn_peer_push(self.roots, self.n_roots, self.mem_new, self.ts_max, P.owner, P.tables["memory"],
                            P.tables["memory_ts"], P.hist_cache, P.hist_thresh, P.rank, self.win, self.src_idx,
                            self.dst_idx, self.ev_eid, self.ev_ts, self.mem_prev, self.efeat, s.E,
                            P.tables["claim"], P.tables["mailbox"], P.tables["mailbox_ts"])
        if train:
            o = self.opt
            C.peer_rs_adam_ag(P.tables["grad"], P.tables["param"], P.world, P.rank, self.flat.data, o.exp_avg,
                              o.exp_avg_sq, o.step_ctr, o.done, float(o.param_groups[0]["lr"]), float(o.betas[0]),
                              float(o.betas[1]), float(o.eps), float(o.weight_decay), 1.0 / P.world)
        main.wait_stream(self._side)
        P.signal_end(C)
        if not self.async_sync:
            # ctdg.async_sync off: the step also waits for every peer's pushes, so the next
            # step starts from fully written-back tables instead of overlapping them
            P.drain(C)

    def _backward(self, gw: dict[str, torch.Tensor]) -> None:
        """Data gradients on the main stream; every weight-gradient GEMM forks onto a
        side stream as soon as its inputs exist, and the two join before Adam (the
        fork/join is captured into the CUDA graph as dependencies)."""
        C, s = self.C, self.s
        m, u, c = self._params()
        mem = self.memory
        main = torch.cuda.current_stream(self.device)
        side = self._side

        def fork():
            side.wait_stream(main)
            return torch.cuda.stream(side)

        with fork():
            C.tgn_link_proj_bwd(self.dP, self.out, self.n_roots, m.src_fc.weight, m.dst_fc.weight,
                                gw["src_fc.weight"], gw["src_fc.bias"], gw["dst_fc.weight"], gw["dst_fc.bias"],
                                self.dout, 1)
        C.tgn_link_proj_bwd(self.dP, self.out, self.n_roots, m.src_fc.weight, m.dst_fc.weight, gw["src_fc.weight"],
                            gw["src_fc.bias"], gw["dst_fc.weight"], gw["dst_fc.bias"], self.dout, 2)
        C.tgn_out_bwd(self.dout, self.xsave, self.mean, self.rstd, c.layer_norm.weight, self.n_roots, self.dropout,
                      self.seed, self.step_ctr, self.edge_total, self.dpre, gw["conv.layer_norm.weight"],
                      gw["conv.layer_norm.bias"])
        with fork():
            C.tgn_out_proj_bwd(self.dpre, self.agg, mem.memory, self.roots, self.n_roots, c.w_out.weight,
                               gw["conv.w_out.weight"], gw["conv.w_out.bias"], self.dagg, self._pd, 1)
        C.tgn_out_proj_bwd(self.dpre, self.agg, mem.memory, self.roots, self.n_roots, c.w_out.weight,
                           gw["conv.w_out.weight"], gw["conv.w_out.bias"], self.dagg, self._pd, 2)
        C.tgn_attn_bwd(self.Q, self.KV, self.att_p, self.dagg, self.nbr_cnt, self.n_roots, s.H, self.att_dropout,
                       self.seed, self.step_ctr, self.dKV, self.dQ)
        te = c.time_enc.w
        args = (mem.memory, self.roots, self.n_roots, self.nbr, self.nbr_eid, self.nbr_dt, self.nbr_cnt, self.efeat,
                s.E, te.weight, te.bias, c.w_q.weight, c.w_k.weight, c.w_v.weight, self.dQ, self.dKV,
                gw["conv.w_q.weight"], gw["conv.w_q.bias"], gw["conv.w_k.weight"], gw["conv.w_k.bias"],
                gw["conv.w_v.weight"], gw["conv.w_v.bias"], gw["conv.time_enc.w.weight"],
                gw["conv.time_enc.w.bias"], self.Mt, self.M1, self._pd)
        with fork():
            C.tgn_attn_proj_bwd(*args, 1)
        C.tgn_attn_proj_bwd(*args, 2)
        main.wait_stream(side)
        C.tgn_attn_proj_bwd(*args, 3)
        if self.peer is not None:
            return  # all-reduce + Adam run fused in _peer_sync
        scale = 1.0
        if self.grad_sync is not None:
            scale = self.grad_sync(self.flat.grad)
        self.opt.step(grad_scale=scale)

    def step(self, split: str, train: bool) -> None:
        """Run one step on the batch in the static buffers (graph replay after warm-up)."""
        key = (split, bool(train))
        if not self.use_graphs:
            n0 = self.C.launch_count()
            self._forward(split, train)
            self._launches[key] = self.C.launch_count() - n0
            return
        g = self._graphs.get(key)
        if g is not None:
            g.replay()
            return
        warm = self._warm.get(key, 0)
        if warm < 2:
            n0 = self.C.launch_count()
            self._forward(split, train)
            self._launches[key] = self.C.launch_count() - n0
            self._warm[key] = warm + 1
            return
        # capture (the capture run itself does not execute the kernels): save and
        # restore the mutable state the step touches, then replay once for real.
        state = self._snapshot_state()
        g = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(self.device)
        with torch.cuda.graph(g):
            self._forward(split, train)
        self._restore_state(state)
        self._graphs[key] = g
        g.replay()

    def _snapshot_state(self):
        return None  # graph capture does not launch work; device state is untouched

    def _restore_state(self, state) -> None:
        return None

    def trace_step(self, split: str, train: bool) -> list[tuple[str, float]]:
        """Run one eager step (no graph replay) with every op bracketed by CUDA events
        and NVTX ranges; returns (op, device ms) in issue order. Ops on the side stream
        overlap the main-stream ones, so the list is a per-op profile, not a sum."""
        self._forward(split, train)  # untraced eager step first: caching-allocator and stream warm-up
        tracer = _TracingOps(self.C)
        real, self.C = self.C, tracer
        try:
            self._forward(split, train)
        finally:
            self.C = real
        torch.cuda.synchronize(self.device)
        return [(n, a.elapsed_time(b)) for n, a, b in tracer.records]

    def launches_per_step(self, train: bool = True) -> int:
        """Framework kernel launches in one step (torch memsets excluded): the count
        measured on an eager warm-up step when there was one, else an estimate."""
        for (split, tr), n in self._launches.items():
            if tr == bool(train):
                return int(n)
        fwd = 10 + self.s.K  # prep, sample, K+1 GRU GEMMs, mailbox, Q, KV, attention, out+LN, link proj, loss, metrics
        bwd = 11             # link-proj (2), LN, out-proj (2), attention, W_q/W_kv/time-encoder (4), Adam
        n = fwd + (bwd if train else 0)
        if self.peer is not None:
            # - local mailbox; + wait/claim, barrier, push, end signal (Adam becomes reduce-scatter + Adam + all-gather)
            n += -1 + 4
        return n

    def drain(self) -> None:
        """Multi-GPU: wait for every peer's end of the last step (its pushes into
        this rank's tables and its reads of this rank's buffers) and synchronise.
        Call before reading node tables on the host and before teardown."""
        if self.peer is not None:
            self.peer.drain(self.C)
        torch.cuda.synchronize(self.device)

    def reset_graphs(self) -> None:
        self.drain()
        self._graphs.clear()
        self._warm.clear()

    # ------------------------------------------------------------------ results
    def read_scalars(self) -> tuple[float, dict[str, float]]:
        vals = torch.cat([self.loss, self.metrics]).tolist()
        return vals[0], {"ap": vals[1], "auc": vals[2], "mrr": vals[3]}

    def pos_probs(self, n: int) -> torch.Tensor:
        return torch.sigmoid(self.scores[:n])
