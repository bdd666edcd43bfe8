// Temporal adjacency keyed by destination (sources of events into each node,
// kept in stream order so per-node lists are time-sorted when the input is).
// Semantics follow vendor/bts_sampler/sampler/include/neighbors.h:243-409 of the
// reference (cache by graph name, optional eid / weight / timestamp columns,
// incremental updates); storage and code are this project's own.
#include <mutex>
#include <sstream>

#include "native.h"

namespace sun {

template <class T>
static const T* ptr_of(const torch::Tensor& t) {
  TORCH_CHECK(t.is_contiguous() && t.dim() == 1, "expected a contiguous 1-D tensor");
  return t.data_ptr<T>();
}

TemporalNeighborBlock& get_neighbors(const std::string& graph_name, torch::Tensor row, torch::Tensor col,
                                     int64_t num_nodes, int is_distinct, c10::optional<torch::Tensor> eid,
                                     c10::optional<torch::Tensor> dist_eid, c10::optional<torch::Tensor> edge_weight,
                                     c10::optional<torch::Tensor> time) {
  static std::map<std::string, TemporalNeighborBlock> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(graph_name);
  if (it != cache.end()) return it->second;
  TemporalNeighborBlock& t = cache[graph_name];
  const NodeId* src = ptr_of<int64_t>(row);
  const NodeId* dst = ptr_of<int64_t>(col);
  const int64_t m = row.numel();
  t.with_eid = eid.has_value();
  t.with_dist_eid = dist_eid.has_value();
  t.weighted = edge_weight.has_value();
  t.with_timestamp = time.has_value();
  std::vector<int64_t> cnt(num_nodes, 0);
  for (int64_t i = 0; i < m; ++i) cnt[dst[i]]++;
  t.neighbors.resize(num_nodes);
  for (int64_t v = 0; v < num_nodes; ++v) t.neighbors[v].reserve(cnt[v]);
  if (t.with_eid) t.eid.resize(num_nodes);
  if (t.with_timestamp) t.timestamp.resize(num_nodes);
  if (t.weighted) {
    t.edge_weight.resize(num_nodes);
    t.inverted_index.resize(num_nodes);
  }
  const EdgeId* e = t.with_eid ? ptr_of<int64_t>(*eid) : nullptr;
  const Ts* ts = t.with_timestamp ? ptr_of<int64_t>(*time) : nullptr;
  const float* w = t.weighted ? ptr_of<float>(*edge_weight) : nullptr;
  for (int64_t i = 0; i < m; ++i) {
    const NodeId d = dst[i];
    t.neighbors[d].push_back(src[i]);
    if (e) t.eid[d].push_back(e[i]);
    if (ts) t.timestamp[d].push_back(ts[i]);
    if (w) {
      t.edge_weight[d].push_back(w[i]);
      t.inverted_index[d][e ? e[i] : src[i]] = static_cast<int64_t>(t.neighbors[d].size()) - 1;
    }
  }
  t.deg.assign(num_nodes, 0);
  for (int64_t v = 0; v < num_nodes; ++v) t.deg[v] = static_cast<int64_t>(t.neighbors[v].size());
  if (is_distinct) {
    t.neighbors_set.resize(num_nodes);
    for (int64_t v = 0; v < num_nodes; ++v) {
      std::vector<NodeId> s = t.neighbors[v];
      std::sort(s.begin(), s.end());
      s.erase(std::unique(s.begin(), s.end()), s.end());
      t.neighbors_set[v] = std::move(s);
    }
  }
  return t;
}

void TemporalNeighborBlock::update_neighbors_with_time(torch::Tensor row, torch::Tensor col, torch::Tensor time,
                                                       torch::Tensor eids, int is_distinct,
                                                       c10::optional<torch::Tensor> ew) {
  const NodeId* src = ptr_of<int64_t>(row);
  const NodeId* dst = ptr_of<int64_t>(col);
  const Ts* ts = ptr_of<int64_t>(time);
  const EdgeId* e = ptr_of<int64_t>(eids);
  const float* w = ew.has_value() ? ptr_of<float>(*ew) : nullptr;
  for (int64_t i = 0; i < row.numel(); ++i) {
    const NodeId d = dst[i];
    if (d >= static_cast<NodeId>(neighbors.size())) {
      neighbors.resize(d + 1);
      deg.resize(d + 1, 0);
      if (with_eid) eid.resize(d + 1);
      if (with_timestamp) timestamp.resize(d + 1);
      if (weighted) {
        edge_weight.resize(d + 1);
        inverted_index.resize(d + 1);
      }
    }
    neighbors[d].push_back(src[i]);
    if (with_eid) eid[d].push_back(e[i]);
    if (with_timestamp) timestamp[d].push_back(ts[i]);
    if (weighted) {
      edge_weight[d].push_back(w ? w[i] : 1.0f);
      inverted_index[d][with_eid ? e[i] : src[i]] = static_cast<int64_t>(neighbors[d].size()) - 1;
    }
    deg[d] = static_cast<int64_t>(neighbors[d].size());
    if (is_distinct && d < static_cast<NodeId>(neighbors_set.size())) {
      auto& s = neighbors_set[d];
      auto pos = std::lower_bound(s.begin(), s.end(), src[i]);
      if (pos == s.end() || *pos != src[i]) s.insert(pos, src[i]);
    }
  }
}

void TemporalNeighborBlock::update_edge_weight(torch::Tensor row_or_eid, torch::Tensor col, torch::Tensor w) {
  TORCH_CHECK(weighted, "This graph has no edge weight information");
  const int64_t* key = ptr_of<int64_t>(row_or_eid);
  const NodeId* dst = ptr_of<int64_t>(col);
  const float* wv = ptr_of<float>(w);
  for (int64_t i = 0; i < col.numel(); ++i) {
    auto it = inverted_index[dst[i]].find(key[i]);
    TORCH_CHECK(it != inverted_index[dst[i]].end(), "edge not present");
    edge_weight[dst[i]][it->second] = wv[i];
  }
}

void TemporalNeighborBlock::update_node_weight(torch::Tensor nid, torch::Tensor node_weight) {
  TORCH_CHECK(weighted, "This graph has no edge weight information");
  const NodeId* n = ptr_of<int64_t>(nid);
  const float* w = ptr_of<float>(node_weight);
  // an edge's weight becomes the weight of its source node
  for (int64_t i = 0; i < nid.numel(); ++i)
    for (size_t d = 0; d < neighbors.size(); ++d)
      for (size_t j = 0; j < neighbors[d].size(); ++j)
        if (neighbors[d][j] == n[i]) edge_weight[d][j] = w[i];
}

void TemporalNeighborBlock::update_all_node_weight(torch::Tensor node_weight) {
  TORCH_CHECK(weighted, "This graph has no edge weight information");
  const float* w = ptr_of<float>(node_weight);
  const int64_t n = node_weight.numel();
#pragma omp parallel for schedule(dynamic, 64)
  for (int64_t d = 0; d < static_cast<int64_t>(neighbors.size()); ++d)
    for (size_t j = 0; j < neighbors[d].size(); ++j)
      if (neighbors[d][j] < n) edge_weight[d][j] = w[neighbors[d][j]];
}

template <class T>
static void put_vv(std::ostringstream& os, const std::vector<std::vector<T>>& v) {
  const uint64_t n = v.size();
  os.write(reinterpret_cast<const char*>(&n), sizeof(n));
  for (const auto& x : v) {
    const uint64_t m = x.size();
    os.write(reinterpret_cast<const char*>(&m), sizeof(m));
    if (m) os.write(reinterpret_cast<const char*>(x.data()), sizeof(T) * m);
  }
}
template <class T>
static void get_vv(std::istringstream& is, std::vector<std::vector<T>>& v) {
  uint64_t n = 0;
  is.read(reinterpret_cast<char*>(&n), sizeof(n));
  v.assign(n, {});
  for (auto& x : v) {
    uint64_t m = 0;
    is.read(reinterpret_cast<char*>(&m), sizeof(m));
    x.resize(m);
    if (m) is.read(reinterpret_cast<char*>(x.data()), sizeof(T) * m);
  }
}

std::string TemporalNeighborBlock::serialize() const {
  std::ostringstream os;
  const uint8_t flags = (with_eid ? 1 : 0) | (weighted ? 2 : 0) | (with_timestamp ? 4 : 0) | (with_dist_eid ? 8 : 0);
  os.write(reinterpret_cast<const char*>(&flags), 1);
  put_vv(os, neighbors);
  put_vv(os, eid);
  put_vv(os, timestamp);
  put_vv(os, edge_weight);
  put_vv(os, neighbors_set);
  return os.str();
}

TemporalNeighborBlock TemporalNeighborBlock::deserialize(const std::string& s) {
  TemporalNeighborBlock t;
  std::istringstream is(s);
  uint8_t flags = 0;
  is.read(reinterpret_cast<char*>(&flags), 1);
  t.with_eid = flags & 1;
  t.weighted = flags & 2;
  t.with_timestamp = flags & 4;
  t.with_dist_eid = flags & 8;
  get_vv(is, t.neighbors);
  get_vv(is, t.eid);
  get_vv(is, t.timestamp);
  get_vv(is, t.edge_weight);
  get_vv(is, t.neighbors_set);
  t.deg.resize(t.neighbors.size());
  for (size_t v = 0; v < t.neighbors.size(); ++v) t.deg[v] = static_cast<int64_t>(t.neighbors[v].size());
  if (t.weighted) {
    t.inverted_index.resize(t.neighbors.size());
    for (size_t d = 0; d < t.neighbors.size(); ++d)
      for (size_t j = 0; j < t.neighbors[d].size(); ++j)
        t.inverted_index[d][t.with_eid ? t.eid[d][j] : t.neighbors[d][j]] = static_cast<int64_t>(j);
  }
  return t;
}

}  // namespace sun
