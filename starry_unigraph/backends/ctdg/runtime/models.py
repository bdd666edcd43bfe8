"""CTDG models: temporal attention, memory updaters, link predictor.

Math follows the reference (backends/ctdg/runtime/models.py:35-386) with DGL
replaced by a dense sampling block: every root has up to ``k`` sampled
neighbours laid out as ``[R, k]`` plus a validity count.

* TemporalTransformerConv: Q = W_q [h_dst || phi(0)], K/V = W_{k,v} [h_nbr || e || phi(dt)],
  score = LeakyReLU_0.2(sum_d Q K) per head (no 1/sqrt(d)), softmax over the
  root's neighbours, attention dropout, agg = sum att V,
  out = LayerNorm(ReLU(Dropout(W_out [agg || h_dst]))). A block with no edges
  at all yields zeros.
* CTDGMemoryUpdater (TGN): GRU over the K mailbox slots (h0 = 0) then
  GRUCell(agg, memory).
* JODIEMemoryUpdater: RNNCell(mail, memory) with the JODIE time projection
  h_proj = (1 + dt * w_p) * memory applied when reading memory.
* CTDGLinkPredictor: logits = out_fc(ReLU(src_fc(z_src) + dst_fc(z_dst))).

On CUDA devices these modules only hold the parameters; the fused sm_100a
kernels (starry_unigraph.ops.tgn) read them in place.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from starry_unigraph.runtime.modules.time_encode import TimeEncode


@dataclass
class DenseBlock:
    """One sampled layer: roots and their up-to-k most recent / uniform neighbours."""

    roots: torch.Tensor        # [R] global node ids
    nbr: torch.Tensor          # [R, k] global node ids (-1 padding)
    eid: torch.Tensor          # [R, k] event ids (-1 padding)
    dt: torch.Tensor           # [R, k] float time deltas
    count: torch.Tensor        # [R] valid neighbours per root

    @property
    def num_edges(self) -> int:
        return int(self.count.sum())

    def mask(self) -> torch.Tensor:
        k = self.nbr.size(1)
        return torch.arange(k, device=self.nbr.device).unsqueeze(0) < self.count.unsqueeze(1)


class TemporalTransformerConv(nn.Module):
    def __init__(self, dim_node: int, dim_edge: int, dim_time: int, num_head: int, dim_out: int,
                 dropout: float = 0.1, att_dropout: float = 0.1) -> None:
        super().__init__()
        self.num_head = num_head
        self.dim_node = dim_node
        self.dim_edge = dim_edge
        self.dim_time = dim_time
        self.dim_out = dim_out
        if dim_time > 0:
            self.time_enc = TimeEncode(dim_time)
        self.w_q = nn.Linear(dim_node + dim_time, dim_out)
        self.w_k = nn.Linear(dim_node + dim_edge + dim_time, dim_out)
        self.w_v = nn.Linear(dim_node + dim_edge + dim_time, dim_out)
        self.w_out = nn.Linear(dim_node + dim_out, dim_out)
        self.dropout = nn.Dropout(dropout)
        self.att_dropout = nn.Dropout(att_dropout)
        self.att_act = nn.LeakyReLU(0.2)
        self.layer_norm = nn.LayerNorm(dim_out)

    def forward_dense(self, h_root: torch.Tensor, h_nbr: torch.Tensor, efeat: torch.Tensor, dt: torch.Tensor,
                      mask: torch.Tensor) -> torch.Tensor:
        """h_root [R, D], h_nbr [R, k, D], efeat [R, k, E], dt [R, k], mask [R, k] -> [R, dim_out]."""
        R, k = mask.shape
        if R == 0 or not bool(mask.any()):
            return h_root.new_zeros(R, self.dim_out)
        if self.dim_time > 0:
            zero_t = self.time_enc(torch.zeros(R, device=h_root.device))
            q_in = torch.cat([h_root, zero_t], dim=1)
            kv_in = torch.cat([h_nbr, efeat, self.time_enc(dt)], dim=2)
        else:
            q_in = h_root
            kv_in = torch.cat([h_nbr, efeat], dim=2)
        H = self.num_head
        dh = self.dim_out // H
        q = self.w_q(q_in).view(R, 1, H, dh)
        kk = self.w_k(kv_in).view(R, k, H, dh)
        vv = self.w_v(kv_in).view(R, k, H, dh)
        score = self.att_act((q * kk).sum(-1))                      # [R, k, H]
        score = score.masked_fill(~mask.unsqueeze(-1), float("-inf"))
        att = torch.softmax(score, dim=1)
        att = torch.nan_to_num(att, nan=0.0) * mask.unsqueeze(-1)
        att = self.att_dropout(att)
        agg = (att.unsqueeze(-1) * vv).sum(1).reshape(R, self.dim_out)
        rst = self.w_out(torch.cat([agg, h_root], dim=1))
        return self.layer_norm(F.relu(self.dropout(rst)))


class CTDGMemoryUpdater(nn.Module):
    """GRU over the K mailbox slots (in slot order) then GRUCell(agg, memory)."""

    def __init__(self, hidden_dim: int, mailbox_slot_dim: int, mailbox_slots: int) -> None:
        super().__init__()
        self.hidden_dim = hidden_dim
        self.mailbox_slots = mailbox_slots
        self.mail_aggregator = nn.GRU(input_size=mailbox_slot_dim, hidden_size=hidden_dim, batch_first=True)
        self.memory_cell = nn.GRUCell(hidden_dim, hidden_dim)

    def forward(self, mailbox_history: torch.Tensor, current_memory: torch.Tensor) -> torch.Tensor:
        if mailbox_history.size(0) == 0:
            return current_memory.clone()
        _, agg = self.mail_aggregator(mailbox_history)
        return self.memory_cell(agg.squeeze(0), current_memory)


class JODIEMemoryUpdater(nn.Module):
    """JODIE: RNNCell(tanh) over the newest mailbox slot; the time projection
    (1 + dt * w_p) * memory is exposed through ``project``."""

    def __init__(self, hidden_dim: int, mailbox_slot_dim: int, mailbox_slots: int) -> None:
        super().__init__()
        self.hidden_dim = hidden_dim
        self.mailbox_slots = mailbox_slots
        self.memory_cell = nn.RNNCell(mailbox_slot_dim, hidden_dim)
        self.time_proj = nn.Linear(1, hidden_dim)
        nn.init.normal_(self.time_proj.weight, 0.0, 1.0 / (hidden_dim ** 0.5))
        nn.init.zeros_(self.time_proj.bias)

    def forward(self, mailbox_history: torch.Tensor, current_memory: torch.Tensor) -> torch.Tensor:
        if mailbox_history.size(0) == 0:
            return current_memory.clone()
        return self.memory_cell(mailbox_history[:, -1, :], current_memory)

    def project(self, memory: torch.Tensor, dt: torch.Tensor) -> torch.Tensor:
        return memory * (1.0 + self.time_proj(dt.float().reshape(-1, 1)))


@dataclass
class CTDGModelOutput:
    pos_logits: torch.Tensor
    neg_logits: torch.Tensor


class CTDGLinkPredictor(nn.Module):
    def __init__(self, num_nodes: int, hidden_dim: int, edge_feat_dim: int, dim_time: int = 100, num_head: int = 2,
                 dropout: float = 0.1, att_dropout: float = 0.1) -> None:
        super().__init__()
        self.hidden_dim = hidden_dim
        self.conv = TemporalTransformerConv(hidden_dim, edge_feat_dim, dim_time, num_head, hidden_dim, dropout,
                                            att_dropout)
        self.src_fc = nn.Linear(hidden_dim, hidden_dim)
        self.dst_fc = nn.Linear(hidden_dim, hidden_dim)
        self.out_fc = nn.Linear(hidden_dim, 1)

    def forward(self, src_conv: torch.Tensor, dst_conv: torch.Tensor, neg_conv: torch.Tensor) -> CTDGModelOutput:
        h_src = self.src_fc(src_conv)
        pos = self.out_fc(F.relu(h_src + self.dst_fc(dst_conv))).squeeze(-1)
        neg = self.out_fc(F.relu(h_src + self.dst_fc(neg_conv))).squeeze(-1)
        return CTDGModelOutput(pos_logits=pos, neg_logits=neg)


class CTDGJodiePredictor(nn.Module):
    """JODIE embedding + the link predictor (Kumar et al., KDD'19; a flagged
    variant: the reference maps every CTDG family to the attention model,
    backends/ctdg/runtime/models.py:332-342). A node's embedding is its memory
    projected to the query time, z = memory * (1 + w_p * dt + b_p), with dt the
    time since the node's previous memory update; no neighbour sampling."""

    def __init__(self, num_nodes: int, hidden_dim: int, edge_feat_dim: int, dim_time: int = 100, num_head: int = 2,
                 dropout: float = 0.1, att_dropout: float = 0.1) -> None:
        super().__init__()
        self.hidden_dim = hidden_dim
        self.time_proj = nn.Linear(1, hidden_dim)
        nn.init.normal_(self.time_proj.weight, 0.0, 1.0 / (hidden_dim ** 0.5))
        nn.init.zeros_(self.time_proj.bias)
        self.src_fc = nn.Linear(hidden_dim, hidden_dim)
        self.dst_fc = nn.Linear(hidden_dim, hidden_dim)
        self.out_fc = nn.Linear(hidden_dim, 1)
        # time deltas enter the projection in units of the stream's time span (JODIE normalises
        # deltas; raw seconds would scale embeddings by ~1e5)
        self.dt_scale = 1.0

    def embed(self, memory: torch.Tensor, dt: torch.Tensor) -> torch.Tensor:
        return memory * (1.0 + self.time_proj((dt.float() * self.dt_scale).reshape(-1, 1)))

    def forward(self, src_conv: torch.Tensor, dst_conv: torch.Tensor, neg_conv: torch.Tensor) -> CTDGModelOutput:
        h_src = self.src_fc(src_conv)
        pos = self.out_fc(F.relu(h_src + self.dst_fc(dst_conv))).squeeze(-1)
        neg = self.out_fc(F.relu(h_src + self.dst_fc(neg_conv))).squeeze(-1)
        return CTDGModelOutput(pos_logits=pos, neg_logits=neg)


@dataclass(frozen=True)
class CTDGModelSpec:
    model_cls: type[nn.Module]
    updater_cls: type[nn.Module]


CTDG_MODEL_SPECS: dict[str, CTDGModelSpec] = {
    "tgn": CTDGModelSpec(CTDGLinkPredictor, CTDGMemoryUpdater),
    "jodie": CTDGModelSpec(CTDGLinkPredictor, CTDGMemoryUpdater),
    "dyrep": CTDGModelSpec(CTDGLinkPredictor, CTDGMemoryUpdater),
    "tgat": CTDGModelSpec(CTDGLinkPredictor, CTDGMemoryUpdater),
    "apan": CTDGModelSpec(CTDGLinkPredictor, CTDGMemoryUpdater),
}


def build_ctdg_model(model_family: str, *, num_nodes: int, hidden_dim: int, edge_feat_dim: int, dim_time: int = 100,
                     num_head: int = 2, dropout: float = 0.1, att_dropout: float = 0.1,
                     embedding: str = "attention") -> nn.Module:
    spec = CTDG_MODEL_SPECS.get(model_family.lower())
    if spec is None:
        raise KeyError(f"Unsupported CTDG model family: {model_family}")
    if str(embedding) == "time_projection":
        return CTDGJodiePredictor(num_nodes=num_nodes, hidden_dim=hidden_dim, edge_feat_dim=edge_feat_dim)
    return spec.model_cls(num_nodes=num_nodes, hidden_dim=hidden_dim, edge_feat_dim=edge_feat_dim, dim_time=dim_time,
                          num_head=num_head, dropout=dropout, att_dropout=att_dropout)


def build_memory_updater(memory_type: str, *, hidden_dim: int, mailbox_slot_dim: int, mailbox_slots: int) -> nn.Module:
    if str(memory_type).lower() == "rnn":
        return JODIEMemoryUpdater(hidden_dim, mailbox_slot_dim, mailbox_slots)
    return CTDGMemoryUpdater(hidden_dim, mailbox_slot_dim, mailbox_slots)
