// Graph partitioner used when pymetis is not installed: a streaming Linear
// Deterministic Greedy pass (Stanton & Kliot, KDD'12) over the symmetrised graph
// in BFS order, followed by balanced label-propagation refinement sweeps.
// Objective: few cut edges under a capacity of (1 + eps) / k of the total vertex
// weight per part. A vertex weighs (1 - s) / N + s * degree / D (N vertices, D
// edge endpoints): `edge_share` s is the fraction of the per-step work that
// scales with edges rather than rows, independent of how many snapshots the
// lifetime graph merges; s = 0 is node balance. On power-law graphs node balance
// alone puts the dense core into one part, whose aggregation work then sets
// every step, while the dense per-row work (GEMMs, recurrent cells) wants rows
// balanced.
#include <omp.h>

#include <algorithm>
#include <numeric>
#include <queue>
#include <random>

#include "native.h"

namespace sun {

torch::Tensor partition_graph(torch::Tensor src, torch::Tensor dst, int64_t num_nodes, int64_t num_parts,
                              double imbalance, int64_t refine_iters, int64_t seed, double edge_share) {
  TORCH_CHECK(num_parts >= 1, "num_parts must be >= 1");
  auto out = torch::zeros({num_nodes}, torch::kInt64);
  if (num_parts == 1 || num_nodes == 0) return out;
  auto s = src.to(torch::kInt64).contiguous(), d = dst.to(torch::kInt64).contiguous();
  const int64_t m = s.numel();
  const int64_t* sp = s.data_ptr<int64_t>();
  const int64_t* dp = d.data_ptr<int64_t>();
  // symmetric CSR with int32 columns
  std::vector<int64_t> ptr(num_nodes + 1, 0);
  for (int64_t i = 0; i < m; ++i) {
    if (sp[i] == dp[i]) continue;
    ptr[sp[i] + 1]++;
    ptr[dp[i] + 1]++;
  }
  for (int64_t v = 0; v < num_nodes; ++v) ptr[v + 1] += ptr[v];
  std::vector<int32_t> adj(ptr[num_nodes]);
  std::vector<int64_t> fill(ptr.begin(), ptr.end() - 1);
  for (int64_t i = 0; i < m; ++i) {
    if (sp[i] == dp[i]) continue;
    adj[fill[sp[i]]++] = static_cast<int32_t>(dp[i]);
    adj[fill[dp[i]]++] = static_cast<int32_t>(sp[i]);
  }
  // BFS order from a random start (restarting in unvisited components)
  std::mt19937_64 rng(static_cast<uint64_t>(seed) * 0x9E3779B97F4A7C15ull + 1);
  std::vector<int64_t> perm(num_nodes);
  std::iota(perm.begin(), perm.end(), 0);
  std::shuffle(perm.begin(), perm.end(), rng);
  std::vector<int64_t> order;
  order.reserve(num_nodes);
  std::vector<char> seen(num_nodes, 0);
  for (int64_t root : perm) {
    if (seen[root]) continue;
    std::queue<int64_t> q;
    q.push(root);
    seen[root] = 1;
    while (!q.empty()) {
      const int64_t v = q.front();
      q.pop();
      order.push_back(v);
      for (int64_t e = ptr[v]; e < ptr[v + 1]; ++e) {
        const int64_t u = adj[e];
        if (!seen[u]) {
          seen[u] = 1;
          q.push(u);
        }
      }
    }
  }
  const int64_t k = num_parts;
  const double share = std::min(1.0, std::max(0.0, edge_share));
  const double endpoints = static_cast<double>(std::max<int64_t>(1, ptr[num_nodes]));
  const double w_node = (1.0 - share) / static_cast<double>(num_nodes), w_end = share / endpoints;
  auto wt = [&](int64_t v) { return w_node + w_end * static_cast<double>(ptr[v + 1] - ptr[v]); };
  const double cap = (1.0 + std::max(0.0, imbalance - 1.0)) / static_cast<double>(k);  // total weight is 1
  std::vector<int64_t> part(num_nodes, -1);
  std::vector<double> load(k, 0.0);
  std::vector<int64_t> cnt(k, 0);
  for (int64_t v : order) {
    std::fill(cnt.begin(), cnt.end(), 0);
    for (int64_t e = ptr[v]; e < ptr[v + 1]; ++e) {
      const int64_t p = part[adj[e]];
      if (p >= 0) cnt[p]++;
    }
    const double w = wt(v);
    int64_t best = -1;
    double best_score = -1.0;
    for (int64_t p = 0; p < k; ++p) {
      if (load[p] + w > cap && load[p] > 0.0) continue;
      const double sc = (cnt[p] + 1e-9) * (1.0 - load[p] / cap);
      if (sc > best_score || (sc == best_score && best >= 0 && load[p] < load[best])) {
        best_score = sc;
        best = p;
      }
    }
    if (best < 0) best = std::min_element(load.begin(), load.end()) - load.begin();
    part[v] = best;
    load[best] += w;
  }
  // balanced label-propagation refinement
  for (int64_t it = 0; it < refine_iters; ++it) {
    int64_t moved = 0;
    for (int64_t v : order) {
      std::fill(cnt.begin(), cnt.end(), 0);
      for (int64_t e = ptr[v]; e < ptr[v + 1]; ++e) cnt[part[adj[e]]]++;
      const int64_t cur = part[v];
      const double w = wt(v);
      int64_t best = cur;
      for (int64_t p = 0; p < k; ++p)
        if (p != cur && cnt[p] > cnt[best] && load[p] + w <= cap) best = p;
      if (best != cur) {
        part[v] = best;
        load[cur] -= w;
        load[best] += w;
        ++moved;
      }
    }
    if (moved == 0) break;
  }
  std::copy(part.begin(), part.end(), out.data_ptr<int64_t>());
  return out;
}

}  // namespace sun
