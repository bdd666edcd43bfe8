// OpenMP temporal neighbour sampler (host oracle / CPU path). Policies and their
// semantics follow vendor/bts_sampler/sampler/include/sampler.h:213-399 of the
// reference:
//   end = lower_bound(ts[node], root_ts)  (strictly earlier events)
//   recent  (or any non-boundary policy with end <= k): the last min(k, end) entries
//   uniform : k draws with replacement over [0, end)
//   weighted / boundery_uniform : k draws proportional to edge weight over [0, end)
//     (the reference draws over the whole list, future events included; restricted here)
//   boundery_recent_uniform : the k most recent candidates, remote ones
//     (edge or neighbour outside local_part) kept with probability p
//   boundery_recent_decay   : remote candidates kept with probability
//     p * exp((ts - root_ts) / delta) / sum * n_remote, local ones always
// Randomness is a counter-based splitmix64 stream per (call, root), so results do
// not depend on the thread count.
#include <omp.h>

#include <chrono>
#include <cmath>
#include <random>

#include "native.h"

namespace sun {

static inline uint64_t splitmix64(uint64_t& x) {
  uint64_t z = (x += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline double unif01(uint64_t& s) { return (splitmix64(s) >> 11) * (1.0 / 9007199254740992.0); }

ParallelSampler::ParallelSampler(TemporalNeighborBlock& t, NodeId n, EdgeId e, int th, std::vector<int>& f, int nl,
                                 std::string pol, int lp, torch::Tensor edge_part, torch::Tensor npart, double p)
    : tnb(t), num_nodes(n), num_edges(e), threads(std::max(1, th)), fanouts(f), num_layers(nl), policy(pol),
      local_part(lp), boundary_p(p) {
  static const char* known[] = {"recent", "uniform", "weighted", "boundery_recent_uniform", "boundery_recent_decay",
                                "boundery_uniform"};
  bool ok = false;
  for (auto* k : known) ok = ok || policy == k;
  TORCH_CHECK(ok, "The policy \"" + policy + "\" does not exist");
  if (local_part != -1) {
    auto ep = edge_part.to(torch::kInt32).contiguous();
    auto np = npart.to(torch::kInt32).contiguous();
    part.assign(ep.data_ptr<int>(), ep.data_ptr<int>() + ep.numel());
    node_part.assign(np.data_ptr<int>(), np.data_ptr<int>() + np.numel());
  }
  ret.resize(num_layers);
}

void ParallelSampler::reset() {
  ret.clear();
  ret.resize(num_layers);
}

namespace {
struct RootOut {
  std::vector<NodeId> nodes;
  std::vector<Ts> nts, dts;
  std::vector<EdgeId> eids;
  std::vector<float> w;
};
}  // namespace

void ParallelSampler::sample_layer_temporal(const std::vector<NodeId>& roots, const std::vector<Ts>& rts, int layer) {
  const auto t0 = std::chrono::steady_clock::now();
  const int k = fanouts[std::min<int>(layer, static_cast<int>(fanouts.size()) - 1)];
  const int64_t R = static_cast<int64_t>(roots.size());
  std::vector<RootOut> outs(R);
  const bool boundary = policy.rfind("boundery", 0) == 0;
  const uint64_t call = static_cast<uint64_t>(calls);
#pragma omp parallel for num_threads(threads) schedule(dynamic, 64)
  for (int64_t i = 0; i < R; ++i) {
    const NodeId node = roots[i];
    const Ts rt = rts[i];
    RootOut& o = outs[i];
    if (node < 0 || node >= static_cast<NodeId>(tnb.neighbors.size())) continue;
    const auto& tsv = tnb.timestamp[node];
    const int64_t end = std::lower_bound(tsv.begin(), tsv.end(), rt) - tsv.begin();
    uint64_t rng = seed ^ (call * 0xD1B54A32D192ED03ull) ^ (static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull);
    auto push = [&](int64_t c, float w) {
      o.nodes.push_back(tnb.neighbors[node][c]);
      o.nts.push_back(tsv[c]);
      o.dts.push_back(rt - tsv[c]);
      o.eids.push_back(tnb.with_eid ? tnb.eid[node][c] : c);
      o.w.push_back(w);
    };
    auto remote = [&](int64_t c) {
      const EdgeId e = tnb.with_eid ? tnb.eid[node][c] : c;
      const NodeId nb = tnb.neighbors[node][c];
      return (e < static_cast<EdgeId>(part.size()) && part[e] != local_part) ||
             (nb < static_cast<NodeId>(node_part.size()) && node_part[nb] != local_part);
    };
    if (policy == "recent" || (end <= k && !boundary)) {
      const int64_t start = std::max<int64_t>(0, end - k);
      for (int64_t c = start; c < end; ++c) push(c, static_cast<float>(c - start));
    } else if (policy == "boundery_recent_uniform") {
      int cnt = 0, considered = 0;
      for (int64_t c = end - 1; c >= 0; --c) {
        if (++considered > k) break;
        if (remote(c) && unif01(rng) > boundary_p) continue;
        push(c, 1.0f);
        if (++cnt > k) break;
      }
    } else if (policy == "boundery_recent_decay") {
      const double delta = end - 1 >= 0 ? static_cast<double>(rt - tsv[end - 1]) * k : 0.0;
      std::vector<double> pr(2 * static_cast<size_t>(k) + 2, 0.0);
      double sum_p = 0.0;
      int n_remote = 0, considered = 0;
      for (int64_t c = end - 1; c >= 0; --c) {
        if (++considered > k) break;
        if (remote(c)) {
          const double ep = std::exp(static_cast<double>(tsv[c] - rt) / delta);
          sum_p += ep;
          pr[considered - 1] = ep;
          ++n_remote;
        }
      }
      if (sum_p < 1e-6) sum_p = 1.0;
      int cnt = 0;
      considered = 0;
      for (int64_t c = end - 1; c >= 0; --c) {
        ++considered;
        if (remote(c)) {
          if (considered > k) continue;
          const double keep = boundary_p * pr[considered - 1] / sum_p * n_remote;
          if (unif01(rng) > keep) continue;
        }
        push(c, 1.0f);
        if (++cnt > k) break;
      }
    } else if (end > 0) {
      if (policy == "uniform") {
        for (int j = 0; j < k; ++j) push(static_cast<int64_t>(splitmix64(rng) % static_cast<uint64_t>(end)), 1.0f);
      } else {  // weighted / boundery_uniform
        const auto& wv = tnb.edge_weight[node];
        double tot = 0.0;
        for (int64_t c = 0; c < end; ++c) tot += wv[c];
        for (int j = 0; j < k; ++j) {
          double u = unif01(rng) * tot, acc = 0.0;
          int64_t c = 0;
          for (; c < end - 1; ++c) {
            acc += wv[c];
            if (u < acc) break;
          }
          push(c, wv[c]);
        }
      }
    }
  }
  TemporalGraphBlock b;
  for (int64_t i = 0; i < R; ++i) {
    const auto& o = outs[i];
    b.src_index.insert(b.src_index.end(), o.nodes.size(), i);
    b.sample_nodes.insert(b.sample_nodes.end(), o.nodes.begin(), o.nodes.end());
    b.sample_nodes_ts.insert(b.sample_nodes_ts.end(), o.nts.begin(), o.nts.end());
    b.delta_ts.insert(b.delta_ts.end(), o.dts.begin(), o.dts.end());
    b.eid.insert(b.eid.end(), o.eids.begin(), o.eids.end());
    b.sample_weight.insert(b.sample_weight.end(), o.w.begin(), o.w.end());
  }
  b.row = b.sample_nodes;
  b.col.resize(b.src_index.size());
  for (size_t j = 0; j < b.src_index.size(); ++j) b.col[j] = roots[b.src_index[j]];
  const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  b.sample_edge_num = static_cast<int64_t>(b.eid.size());
  b.sample_time = dt;
  ret[layer] = std::move(b);
  ret[0].tot_time += dt;
}

void ParallelSampler::sample_layer_static(const std::vector<NodeId>& roots, int layer) {
  const int k = fanouts[std::min<int>(layer, static_cast<int>(fanouts.size()) - 1)];
  const int64_t R = static_cast<int64_t>(roots.size());
  std::vector<RootOut> outs(R);
  const uint64_t call = static_cast<uint64_t>(calls);
#pragma omp parallel for num_threads(threads) schedule(dynamic, 64)
  for (int64_t i = 0; i < R; ++i) {
    const NodeId node = roots[i];
    if (node < 0 || node >= static_cast<NodeId>(tnb.neighbors.size())) continue;
    const int64_t deg = static_cast<int64_t>(tnb.neighbors[node].size());
    uint64_t rng = seed ^ (call * 0xD1B54A32D192ED03ull) ^ (static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull);
    RootOut& o = outs[i];
    auto push = [&](int64_t c) {
      o.nodes.push_back(tnb.neighbors[node][c]);
      o.eids.push_back(tnb.with_eid ? tnb.eid[node][c] : c);
    };
    if (deg <= k) {
      for (int64_t c = 0; c < deg; ++c) push(c);
    } else {
      for (int j = 0; j < k; ++j) push(static_cast<int64_t>(splitmix64(rng) % static_cast<uint64_t>(deg)));
    }
  }
  TemporalGraphBlock b;
  for (int64_t i = 0; i < R; ++i) {
    b.src_index.insert(b.src_index.end(), outs[i].nodes.size(), i);
    b.sample_nodes.insert(b.sample_nodes.end(), outs[i].nodes.begin(), outs[i].nodes.end());
    b.eid.insert(b.eid.end(), outs[i].eids.begin(), outs[i].eids.end());
  }
  b.row = b.sample_nodes;
  b.col.resize(b.src_index.size());
  for (size_t j = 0; j < b.src_index.size(); ++j) b.col[j] = roots[b.src_index[j]];
  b.sample_edge_num = static_cast<int64_t>(b.eid.size());
  ret[layer] = std::move(b);
}

void ParallelSampler::neighbor_sample_from_nodes(torch::Tensor nodes, c10::optional<torch::Tensor> root_ts,
                                                 c10::optional<bool> /*part_unique*/) {
  if (policy == "weighted") TORCH_CHECK(tnb.weighted, "Tnb has no weight information!");
  if (policy == "recent") TORCH_CHECK(tnb.with_timestamp, "Tnb has no timestamp information!");
  auto nd = nodes.to(torch::kInt64).contiguous();
  std::vector<NodeId> roots(nd.data_ptr<int64_t>(), nd.data_ptr<int64_t>() + nd.numel());
  ret.assign(num_layers, TemporalGraphBlock());
  pybind11::gil_scoped_release release;
  if (tnb.with_timestamp) {
    TORCH_CHECK(root_ts.has_value(), "Parameter mismatch: root timestamps are required");
    auto t = root_ts->to(torch::kInt64).contiguous();
    std::vector<Ts> rts(t.data_ptr<int64_t>(), t.data_ptr<int64_t>() + t.numel());
    for (int l = 0; l < num_layers; ++l) {
      sample_layer_temporal(roots, rts, l);
      roots = ret[l].sample_nodes;
      rts = ret[l].sample_nodes_ts;
    }
  } else {
    for (int l = 0; l < num_layers; ++l) {
      sample_layer_static(roots, l);
      roots = ret[l].sample_nodes;
    }
  }
  ++calls;
}

}  // namespace sun
