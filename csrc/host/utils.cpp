// Small host utilities exported by the reference's sampler module
// (vendor/bts_sampler/sampler/include/head.h:99-206, temporal_utils.h:13-91):
//   heads_unique         : unique ids keeping the given heads first, in order
//   divide_nodes_to_part : split ids by contiguous partition ranges part_ptr
//   sparse_get_index     : position of each id inside map_key (-1 if absent)
//   get_norm_temporal    : mean / std of inter-event times of each node (averaged)
#include <cmath>
#include <unordered_map>

#include "native.h"

namespace sun {

torch::Tensor heads_unique(torch::Tensor array, torch::Tensor heads, int /*threads*/) {
  auto a = array.to(torch::kInt64).contiguous(), h = heads.to(torch::kInt64).contiguous();
  std::unordered_map<int64_t, char> seen;
  std::vector<int64_t> out;
  out.reserve(a.numel() + h.numel());
  for (int64_t i = 0; i < h.numel(); ++i)
    if (seen.emplace(h.data_ptr<int64_t>()[i], 1).second) out.push_back(h.data_ptr<int64_t>()[i]);
  for (int64_t i = 0; i < a.numel(); ++i)
    if (seen.emplace(a.data_ptr<int64_t>()[i], 1).second) out.push_back(a.data_ptr<int64_t>()[i]);
  return torch::tensor(out, torch::kInt64);
}

std::vector<torch::Tensor> divide_nodes_to_part(torch::Tensor nodes, const std::vector<NodeId>& part_ptr,
                                                int /*threads*/) {
  auto n = nodes.to(torch::kInt64).contiguous();
  const int64_t parts = static_cast<int64_t>(part_ptr.size()) - 1;
  std::vector<std::vector<int64_t>> buckets(std::max<int64_t>(parts, 0));
  for (int64_t i = 0; i < n.numel(); ++i) {
    const int64_t v = n.data_ptr<int64_t>()[i];
    const int64_t p = std::upper_bound(part_ptr.begin(), part_ptr.end(), v) - part_ptr.begin() - 1;
    if (p >= 0 && p < parts) buckets[p].push_back(v);
  }
  std::vector<torch::Tensor> out;
  for (auto& b : buckets) out.push_back(torch::tensor(b, torch::kInt64));
  return out;
}

torch::Tensor sparse_get_index(torch::Tensor in, torch::Tensor map_key) {
  auto a = in.to(torch::kInt64).contiguous(), k = map_key.to(torch::kInt64).contiguous();
  std::unordered_map<int64_t, int64_t> pos;
  pos.reserve(k.numel() * 2);
  for (int64_t i = 0; i < k.numel(); ++i) pos.emplace(k.data_ptr<int64_t>()[i], i);
  auto out = torch::empty({a.numel()}, torch::kInt64);
  for (int64_t i = 0; i < a.numel(); ++i) {
    auto it = pos.find(a.data_ptr<int64_t>()[i]);
    out.data_ptr<int64_t>()[i] = it == pos.end() ? -1 : it->second;
  }
  return out;
}

std::vector<double> get_norm_temporal(torch::Tensor row, torch::Tensor col, torch::Tensor ts, int64_t num_nodes) {
  auto r = row.to(torch::kInt64).contiguous(), c = col.to(torch::kInt64).contiguous();
  auto t = ts.to(torch::kFloat64).contiguous();
  std::vector<double> last(num_nodes, -1.0), sum(num_nodes, 0.0), sq(num_nodes, 0.0);
  std::vector<int64_t> n(num_nodes, 0);
  auto touch = [&](int64_t v, double tt) {
    if (last[v] >= 0) {
      const double d = tt - last[v];
      sum[v] += d;
      sq[v] += d * d;
      n[v]++;
    }
    last[v] = tt;
  };
  for (int64_t i = 0; i < r.numel(); ++i) {
    touch(r.data_ptr<int64_t>()[i], t.data_ptr<double>()[i]);
    touch(c.data_ptr<int64_t>()[i], t.data_ptr<double>()[i]);
  }
  double m_acc = 0.0, s_acc = 0.0;
  int64_t k = 0;
  for (int64_t v = 0; v < num_nodes; ++v) {
    if (n[v] == 0) continue;
    const double mean = sum[v] / n[v];
    m_acc += mean;
    s_acc += std::sqrt(std::max(0.0, sq[v] / n[v] - mean * mean));
    ++k;
  }
  return {k ? m_acc / k : 0.0, k ? s_acc / k : 0.0};
}

}  // namespace sun
