// Host (CPU) native components of starry_unigraph, module starry_unigraph._native.
//
//  * TemporalNeighborBlock : per-destination temporal adjacency (sources of the
//    events into each node, in stream order) with event ids, timestamps and
//    optional weights; incremental appends and weight edits; serialisation.
//  * ParallelSampler       : OpenMP temporal / static neighbour sampler with the
//    policies recent, uniform, weighted and the partition-aware boundery_*.
//  * ParallelTppRComputer  : temporal personalised PageRank top-k (streaming and
//    pruned random-walk variants).
//  * adaptive_split        : staleness-driven adaptive time splitting of a stream.
//  * partition_graph       : streaming LDG partitioner + label-propagation refinement.
//  * utilities             : heads_unique, divide_nodes_to_part, sparse_get_index,
//                            get_norm_temporal.
#pragma once

#include <torch/extension.h>

#include <cstdint>
#include <map>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

namespace sun {

using NodeId = int64_t;
using EdgeId = int64_t;
using Ts = int64_t;
using Weight = float;

struct TemporalNeighborBlock {
  std::vector<std::vector<NodeId>> neighbors;
  std::vector<std::vector<EdgeId>> eid;
  std::vector<std::vector<Ts>> timestamp;
  std::vector<std::vector<Weight>> edge_weight;
  std::vector<std::unordered_map<int64_t, int64_t>> inverted_index;  // eid (or src) -> position
  std::vector<int64_t> deg;
  std::vector<std::vector<NodeId>> neighbors_set;  // distinct neighbours (optional)
  bool with_eid = false, weighted = false, with_timestamp = false, with_dist_eid = false;

  TemporalNeighborBlock() = default;
  TemporalNeighborBlock(std::vector<std::vector<NodeId>>& n, std::vector<int64_t>& d) : neighbors(n), deg(d) {}

  void update_neighbors_with_time(torch::Tensor row, torch::Tensor col, torch::Tensor time, torch::Tensor eid,
                                  int is_distinct, c10::optional<torch::Tensor> edge_weight);
  void update_edge_weight(torch::Tensor row_or_eid, torch::Tensor col, torch::Tensor edge_weight);
  void update_node_weight(torch::Tensor nid, torch::Tensor node_weight);
  void update_all_node_weight(torch::Tensor node_weight);
  std::string serialize() const;
  static TemporalNeighborBlock deserialize(const std::string& s);
};

TemporalNeighborBlock& get_neighbors(const std::string& graph_name, torch::Tensor row, torch::Tensor col,
                                     int64_t num_nodes, int is_distinct, c10::optional<torch::Tensor> eid,
                                     c10::optional<torch::Tensor> dist_eid, c10::optional<torch::Tensor> edge_weight,
                                     c10::optional<torch::Tensor> time);

struct TemporalGraphBlock {
  std::vector<NodeId> row, col;
  std::vector<EdgeId> eid;
  std::vector<Ts> delta_ts;
  std::vector<int64_t> src_index;
  std::vector<NodeId> sample_nodes;
  std::vector<Ts> sample_nodes_ts;
  std::vector<float> sample_weight;
  std::vector<Weight> e_weights;
  double sample_time = 0, tot_time = 0;
  int64_t sample_edge_num = 0;
};

struct ParallelSampler {
  TemporalNeighborBlock& tnb;
  NodeId num_nodes;
  EdgeId num_edges;
  int threads;
  std::vector<int> fanouts;
  int num_layers;
  std::string policy;
  int local_part;
  std::vector<int> part, node_part;
  double boundary_p;
  std::vector<TemporalGraphBlock> ret;
  uint64_t seed = 8;
  int64_t calls = 0;

  ParallelSampler(TemporalNeighborBlock& t, NodeId n, EdgeId e, int threads, std::vector<int>& fanouts,
                  int num_layers, std::string policy, int local_part, torch::Tensor edge_part,
                  torch::Tensor node_part, double p);
  void reset();
  void neighbor_sample_from_nodes(torch::Tensor nodes, c10::optional<torch::Tensor> root_ts,
                                  c10::optional<bool> part_unique);
  void sample_layer_temporal(const std::vector<NodeId>& nodes, const std::vector<Ts>& ts, int layer);
  void sample_layer_static(const std::vector<NodeId>& nodes, int layer);
};

using PPRKey = std::tuple<EdgeId, NodeId, Ts>;
struct PPRKeyHash {
  size_t operator()(const PPRKey& k) const {
    uint64_t h = static_cast<uint64_t>(std::get<0>(k)) * 0x9E3779B97F4A7C15ull;
    h ^= static_cast<uint64_t>(std::get<1>(k)) + 0x7F4A7C15ull + (h << 6) + (h >> 2);
    h ^= static_cast<uint64_t>(std::get<2>(k)) + 0x94D049BBull + (h << 6) + (h >> 2);
    return static_cast<size_t>(h);
  }
};
using PPRDict = std::unordered_map<PPRKey, double, PPRKeyHash>;

struct ParallelTppRComputer {
  TemporalNeighborBlock& tnb;
  NodeId num_nodes;
  EdgeId num_edges;
  int threads, fanout, num_layers, num_tpprs;
  std::vector<float> alpha_list, beta_list;
  std::vector<std::vector<PPRDict>> ppr, val_ppr;
  std::vector<std::vector<double>> norm, val_norm;
  std::vector<std::vector<TemporalGraphBlock>> ret;

  ParallelTppRComputer(TemporalNeighborBlock& t, NodeId n, EdgeId e, int threads, int fanout, int num_layers,
                       int num_tpprs, std::vector<float>& alpha, std::vector<float>& beta);
  void reset_ret();
  void reset_tppr();
  void reset_val_tppr();
  void backup_to_val();
  void restore_from_val();
  PPRDict update_pair(NodeId s1, NodeId s2, int id, EdgeId eid, Ts ts) const;
  void extract(const PPRDict& d, Ts now, int id, int64_t pos);
  void get_pruned_topk(torch::Tensor src_nodes, torch::Tensor root_ts, int tppr_id);
  void streaming_topk(torch::Tensor nodes, torch::Tensor root_ts, torch::Tensor eids, bool with_fake);
  void single_streaming_topk(torch::Tensor nodes, torch::Tensor root_ts, torch::Tensor eids, int tppr_id);
  void compute_val_tppr(torch::Tensor src, torch::Tensor dst, torch::Tensor root_ts, torch::Tensor eids);
};

struct SplitResult {
  torch::Tensor group_index;
  torch::Tensor keep_indices;
  double drop_proportion = 0.0;
};

SplitResult adaptive_split(torch::Tensor src, torch::Tensor dst, torch::Tensor ts, int64_t base_batch_size,
                           double graph_feature, double alpha, double beta, double aggl, bool enable_drop,
                           double drop_rate, int64_t window_size);

torch::Tensor partition_graph(torch::Tensor src, torch::Tensor dst, int64_t num_nodes, int64_t num_parts,
                              double imbalance, int64_t refine_iters, int64_t seed, double edge_share);

torch::Tensor heads_unique(torch::Tensor array, torch::Tensor heads, int threads);
std::vector<torch::Tensor> divide_nodes_to_part(torch::Tensor nodes, const std::vector<NodeId>& part_ptr,
                                                int threads);
torch::Tensor sparse_get_index(torch::Tensor in, torch::Tensor map_key);
std::vector<double> get_norm_temporal(torch::Tensor row, torch::Tensor col, torch::Tensor ts, int64_t num_nodes);

}  // namespace sun
