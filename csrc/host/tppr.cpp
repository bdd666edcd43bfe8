// Temporal personalised PageRank (TPPR) top-k neighbourhoods, after the
// streaming TPPR formulation used by the reference (vendor/bts_sampler/
// sampler/include/tppr.h:77-375):
//   * streaming update for an event (s1 -> s2 at time t, edge e):
//       norm' = beta * norm + beta
//       PPR'(s1) = PPR(s1) * norm/norm' * beta  +  (PPR(s2) + {(e, s2, t): alpha}) * beta/norm' * (1 - alpha)
//     (first event of s1: PPR'(s1) = {(e, s2, t): (1 - alpha) * alpha}), truncated to the top-k entries;
//   * streaming_topk: for each event first read the current top-k of src, dst
//     (and the negative "fake" node), then apply the update for both endpoints;
//   * get_pruned_topk: depth-limited temporal random walk from a node with
//     geometric decay beta over its most recent neighbours.
// alpha/beta are kept as floats (the reference truncates them to integers in
// several places); the event count is derived from the node list length.
#include <algorithm>
#include <cmath>

#include "native.h"

namespace sun {

ParallelTppRComputer::ParallelTppRComputer(TemporalNeighborBlock& t, NodeId n, EdgeId e, int th, int f, int nl, int nt,
                                           std::vector<float>& a, std::vector<float>& b)
    : tnb(t), num_nodes(n), num_edges(e), threads(th), fanout(f), num_layers(nl), num_tpprs(nt), alpha_list(a),
      beta_list(b) {
  ret.assign(num_tpprs, {});
  reset_tppr();
}

void ParallelTppRComputer::reset_ret() {
  for (auto& r : ret) r.clear();
}
void ParallelTppRComputer::reset_tppr() {
  ppr.assign(num_tpprs, std::vector<PPRDict>(num_nodes));
  norm.assign(num_tpprs, std::vector<double>(num_nodes, 0.0));
}
void ParallelTppRComputer::reset_val_tppr() {
  val_ppr.assign(num_tpprs, std::vector<PPRDict>(num_nodes));
  val_norm.assign(num_tpprs, std::vector<double>(num_nodes, 0.0));
}
void ParallelTppRComputer::backup_to_val() {
  val_ppr = ppr;
  val_norm = norm;
}
void ParallelTppRComputer::restore_from_val() {
  ppr = val_ppr;
  norm = val_norm;
}

static PPRDict topk(const PPRDict& d, int k) {
  if (static_cast<int>(d.size()) <= k) return d;
  std::vector<std::pair<PPRKey, double>> v(d.begin(), d.end());
  std::partial_sort(v.begin(), v.begin() + k, v.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
  PPRDict out;
  for (int i = 0; i < k; ++i) out.emplace(v[i].first, v[i].second);
  return out;
}

PPRDict ParallelTppRComputer::update_pair(NodeId s1, NodeId s2, int id, EdgeId eid, Ts ts) const {
  const double alpha = alpha_list[id], beta = beta_list[id];
  const double last = norm[id][s1];
  PPRDict out;
  double s2_scale;
  if (last == 0.0) {
    s2_scale = 1.0 - alpha;
  } else {
    const double nn = last * beta + beta;
    const double s1_scale = last / nn * beta;
    s2_scale = beta / nn * (1.0 - alpha);
    for (const auto& kv : ppr[id][s1]) out[kv.first] = kv.second * s1_scale;
    for (const auto& kv : ppr[id][s2]) out[kv.first] += kv.second * s2_scale;
  }
  out[PPRKey(eid, s2, ts)] = alpha != 0.0 ? s2_scale * alpha : s2_scale;
  return topk(out, fanout);
}

void ParallelTppRComputer::extract(const PPRDict& d, Ts now, int id, int64_t pos) {
  TemporalGraphBlock b;
  for (const auto& kv : d) {
    b.eid.push_back(std::get<0>(kv.first));
    b.sample_nodes.push_back(std::get<1>(kv.first));
    b.sample_nodes_ts.push_back(std::get<2>(kv.first));
    b.e_weights.push_back(static_cast<float>(kv.second));
    b.delta_ts.push_back(now - std::get<2>(kv.first));
  }
  ret[id][pos] = std::move(b);
}

void ParallelTppRComputer::streaming_topk(torch::Tensor nodes, torch::Tensor root_ts, torch::Tensor eids,
                                          bool with_fake) {
  auto nd = nodes.to(torch::kInt64).contiguous();
  auto tt = root_ts.to(torch::kInt64).contiguous();
  auto ee = eids.to(torch::kInt64).contiguous();
  const int64_t* n = nd.data_ptr<int64_t>();
  const int64_t* t = tt.data_ptr<int64_t>();
  const int64_t* e = ee.data_ptr<int64_t>();
  const int parts = with_fake ? 3 : 2;
  const int64_t m = nd.numel() / parts;
  reset_ret();
  for (int id = 0; id < num_tpprs; ++id) {
    ret[id].assign(nd.numel(), TemporalGraphBlock());
    for (int64_t i = 0; i < m; ++i) {
      const NodeId s = n[i], d = n[i + m];
      extract(ppr[id][s], t[i], id, i);
      extract(ppr[id][d], t[i], id, i + m);
      if (with_fake) extract(ppr[id][n[i + 2 * m]], t[i], id, i + 2 * m);
      PPRDict ns = update_pair(s, d, id, e[i], t[i]);
      const double beta = beta_list[id];
      if (s != d) {
        PPRDict nd2 = update_pair(d, s, id, e[i], t[i]);
        ppr[id][d] = std::move(nd2);
        norm[id][d] = norm[id][d] * beta + beta;
      }
      ppr[id][s] = std::move(ns);
      norm[id][s] = norm[id][s] * beta + beta;
    }
  }
}

void ParallelTppRComputer::single_streaming_topk(torch::Tensor nodes, torch::Tensor root_ts, torch::Tensor eids,
                                                 int tppr_id) {
  const int saved = num_tpprs;
  std::vector<float> a = alpha_list, b = beta_list;
  // run the streaming update for one TPPR instance only
  auto nd = nodes.to(torch::kInt64).contiguous();
  auto tt = root_ts.to(torch::kInt64).contiguous();
  auto ee = eids.to(torch::kInt64).contiguous();
  const int64_t* n = nd.data_ptr<int64_t>();
  const int64_t* t = tt.data_ptr<int64_t>();
  const int64_t* e = ee.data_ptr<int64_t>();
  const int64_t m = nd.numel() / 3;
  ret[tppr_id].assign(nd.numel(), TemporalGraphBlock());
  for (int64_t i = 0; i < m; ++i) {
    const NodeId s = n[i], d = n[i + m];
    extract(ppr[tppr_id][s], t[i], tppr_id, i);
    extract(ppr[tppr_id][d], t[i], tppr_id, i + m);
    extract(ppr[tppr_id][n[i + 2 * m]], t[i], tppr_id, i + 2 * m);
    PPRDict ns = update_pair(s, d, tppr_id, e[i], t[i]);
    const double beta = beta_list[tppr_id];
    if (s != d) {
      ppr[tppr_id][d] = update_pair(d, s, tppr_id, e[i], t[i]);
      norm[tppr_id][d] = norm[tppr_id][d] * beta + beta;
    }
    ppr[tppr_id][s] = std::move(ns);
    norm[tppr_id][s] = norm[tppr_id][s] * beta + beta;
  }
  (void)saved;
}

void ParallelTppRComputer::compute_val_tppr(torch::Tensor src, torch::Tensor dst, torch::Tensor root_ts,
                                            torch::Tensor eids) {
  auto s_ = src.to(torch::kInt64).contiguous();
  auto d_ = dst.to(torch::kInt64).contiguous();
  auto t_ = root_ts.to(torch::kInt64).contiguous();
  auto e_ = eids.to(torch::kInt64).contiguous();
  for (int id = 0; id < num_tpprs; ++id) {
    const double beta = beta_list[id];
    for (int64_t i = 0; i < s_.numel(); ++i) {
      const NodeId s = s_.data_ptr<int64_t>()[i], d = d_.data_ptr<int64_t>()[i];
      const Ts t = t_.data_ptr<int64_t>()[i];
      const EdgeId e = e_.data_ptr<int64_t>()[i];
      PPRDict ns = update_pair(s, d, id, e, t);
      if (s != d) {
        ppr[id][d] = update_pair(d, s, id, e, t);
        norm[id][d] = norm[id][d] * beta + beta;
      }
      ppr[id][s] = std::move(ns);
      norm[id][s] = norm[id][s] * beta + beta;
    }
  }
  backup_to_val();
}

void ParallelTppRComputer::get_pruned_topk(torch::Tensor src_nodes, torch::Tensor root_ts, int tppr_id) {
  auto nd = src_nodes.to(torch::kInt64).contiguous();
  auto tt = root_ts.to(torch::kInt64).contiguous();
  const int64_t n = nd.numel();
  const double alpha = alpha_list[tppr_id], beta = beta_list[tppr_id];
  ret[tppr_id].assign(n, TemporalGraphBlock());
#pragma omp parallel for num_threads(std::max(1, threads)) schedule(dynamic, 16)
  for (int64_t i = 0; i < n; ++i) {
    PPRDict dict;
    std::vector<std::tuple<NodeId, Ts, double>> frontier{{nd.data_ptr<int64_t>()[i], tt.data_ptr<int64_t>()[i], 1.0}};
    for (int depth = 0; depth < num_layers && !frontier.empty(); ++depth) {
      std::vector<std::tuple<NodeId, Ts, double>> next;
      for (const auto& [q, qt, qw] : frontier) {
        if (q < 0 || q >= static_cast<NodeId>(tnb.timestamp.size())) continue;
        const auto& tsv = tnb.timestamp[q];
        const int64_t end = std::lower_bound(tsv.begin(), tsv.end(), qt) - tsv.begin();
        if (end == 0) continue;
        const double nrm = beta / (1.0 - beta) * (1.0 - std::pow(beta, static_cast<double>(end)));
        double w = (alpha != 0.0 && depth == 0) ? qw * (1.0 - alpha) * beta / nrm * alpha : qw * (1.0 - alpha) * beta / nrm;
        for (int64_t z = 0; z < std::min<int64_t>(fanout, end); ++z) {
          const int64_t c = end - z - 1;
          const PPRKey key(tnb.eid[q][c], tnb.neighbors[q][c], tsv[c]);
          dict[key] += w;
          next.emplace_back(tnb.neighbors[q][c], tsv[c], w);
          w *= beta;
        }
      }
      frontier.swap(next);
    }
    if (!dict.empty()) {
      PPRDict top = topk(dict, fanout);
      TemporalGraphBlock b;
      for (const auto& kv : top) {
        b.eid.push_back(std::get<0>(kv.first));
        b.sample_nodes.push_back(std::get<1>(kv.first));
        b.sample_nodes_ts.push_back(std::get<2>(kv.first));
        b.e_weights.push_back(static_cast<float>(kv.second));
        b.delta_ts.push_back(tt.data_ptr<int64_t>()[i] - std::get<2>(kv.first));
      }
      ret[tppr_id][i] = std::move(b);
    }
  }
}

}  // namespace sun
