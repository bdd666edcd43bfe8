// pybind11 surface of starry_unigraph._native. Names and call signatures follow
// the reference's libstarrygl_sampler / adaptive_split_cpp modules
// (vendor/bts_sampler/sampler/export.cpp:10-106, split/time_split.cpp:414-430) so
// wrappers written against those keep working.
#include <pybind11/stl.h>

#include "native.h"

namespace py = pybind11;
using namespace sun;

template <class T>
static torch::Tensor vec_tensor(const std::vector<T>& v, torch::ScalarType t) {
  return torch::from_blob(const_cast<T*>(v.data()), {static_cast<int64_t>(v.size())}, t).clone();
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "starry_unigraph host natives: temporal sampler, TPPR, time split, partitioner";
  m.def("get_neighbors", &get_neighbors, py::return_value_policy::reference, py::arg("graph_name"), py::arg("row"),
        py::arg("col"), py::arg("num_nodes"), py::arg("is_distinct") = 0, py::arg("eid") = py::none(),
        py::arg("dist_eid") = py::none(), py::arg("edge_weight") = py::none(), py::arg("time") = py::none());
  m.def("heads_unique", &heads_unique);
  m.def("divide_nodes_to_part", &divide_nodes_to_part);
  m.def("sparse_get_index", &sparse_get_index);
  m.def("get_norm_temporal", &get_norm_temporal);
  m.def("partition_graph", &partition_graph, py::arg("src"), py::arg("dst"), py::arg("num_nodes"),
        py::arg("num_parts"), py::arg("imbalance") = 1.03, py::arg("refine_iters") = 3, py::arg("seed") = 0,
        py::arg("edge_share") = 0.0);

  py::class_<TemporalGraphBlock>(m, "TemporalGraphBlock")
      .def(py::init<>())
      .def("row", [](const TemporalGraphBlock& b) { return vec_tensor(b.row, torch::kInt64); })
      .def("col", [](const TemporalGraphBlock& b) { return vec_tensor(b.col, torch::kInt64); })
      .def("eid", [](const TemporalGraphBlock& b) { return vec_tensor(b.eid, torch::kInt64); })
      .def("delta_ts", [](const TemporalGraphBlock& b) { return vec_tensor(b.delta_ts, torch::kInt64); })
      .def("src_index", [](const TemporalGraphBlock& b) { return vec_tensor(b.src_index, torch::kInt64); })
      .def("sample_nodes", [](const TemporalGraphBlock& b) { return vec_tensor(b.sample_nodes, torch::kInt64); })
      .def("sample_nodes_ts", [](const TemporalGraphBlock& b) { return vec_tensor(b.sample_nodes_ts, torch::kInt64); })
      .def("sample_weight", [](const TemporalGraphBlock& b) { return vec_tensor(b.sample_weight, torch::kFloat32); })
      .def("e_weights", [](const TemporalGraphBlock& b) { return vec_tensor(b.e_weights, torch::kFloat32); })
      .def_readonly("sample_time", &TemporalGraphBlock::sample_time)
      .def_readonly("tot_time", &TemporalGraphBlock::tot_time)
      .def_readonly("sample_edge_num", &TemporalGraphBlock::sample_edge_num);

  py::class_<TemporalNeighborBlock>(m, "TemporalNeighborBlock")
      .def(py::init<std::vector<std::vector<NodeId>>&, std::vector<int64_t>&>())
      .def(py::pickle([](const TemporalNeighborBlock& t) { return py::bytes(t.serialize()); },
                      [](const py::bytes& s) { return TemporalNeighborBlock::deserialize(std::string(s)); }))
      .def("update_neighbors_with_time", &TemporalNeighborBlock::update_neighbors_with_time)
      .def("update_edge_weight", &TemporalNeighborBlock::update_edge_weight)
      .def("update_node_weight", &TemporalNeighborBlock::update_node_weight)
      .def("update_all_node_weight", &TemporalNeighborBlock::update_all_node_weight)
      .def_readonly("neighbors", &TemporalNeighborBlock::neighbors)
      .def_readonly("timestamp", &TemporalNeighborBlock::timestamp)
      .def_readonly("edge_weight", &TemporalNeighborBlock::edge_weight)
      .def_readonly("eid", &TemporalNeighborBlock::eid)
      .def_readonly("deg", &TemporalNeighborBlock::deg)
      .def_readonly("with_eid", &TemporalNeighborBlock::with_eid)
      .def_readonly("with_timestamp", &TemporalNeighborBlock::with_timestamp)
      .def_readonly("weighted", &TemporalNeighborBlock::weighted);

  py::class_<ParallelSampler>(m, "ParallelSampler")
      .def(py::init<TemporalNeighborBlock&, NodeId, EdgeId, int, std::vector<int>&, int, std::string, int,
                    torch::Tensor, torch::Tensor, double>(),
           py::keep_alive<1, 2>())
      .def_readonly("ret", &ParallelSampler::ret)
      .def("neighbor_sample_from_nodes", &ParallelSampler::neighbor_sample_from_nodes, py::arg("nodes"),
           py::arg("root_ts") = py::none(), py::arg("part_unique") = py::none())
      .def("reset", &ParallelSampler::reset)
      .def("get_ret", [](const ParallelSampler& s) { return s.ret; });

  py::class_<ParallelTppRComputer>(m, "ParallelTppRComputer")
      .def(py::init<TemporalNeighborBlock&, NodeId, EdgeId, int, int, int, int, std::vector<float>&,
                    std::vector<float>&>(),
           py::keep_alive<1, 2>())
      .def_readonly("ret", &ParallelTppRComputer::ret)
      .def("reset_ret", &ParallelTppRComputer::reset_ret)
      .def("reset_tppr", &ParallelTppRComputer::reset_tppr)
      .def("reset_val_tppr", &ParallelTppRComputer::reset_val_tppr)
      .def("backup_tppr", &ParallelTppRComputer::backup_to_val)
      .def("restore_tppr", &ParallelTppRComputer::restore_from_val)
      .def("restore_val_tppr", &ParallelTppRComputer::restore_from_val)
      .def("get_pruned_topk", &ParallelTppRComputer::get_pruned_topk)
      .def("streaming_topk",
           [](ParallelTppRComputer& c, torch::Tensor n, torch::Tensor t, torch::Tensor e) {
             c.streaming_topk(n, t, e, true);
           })
      .def("streaming_topk_no_fake",
           [](ParallelTppRComputer& c, torch::Tensor n, torch::Tensor t, torch::Tensor e) {
             c.streaming_topk(n, t, e, false);
           })
      .def("single_streaming_topk", &ParallelTppRComputer::single_streaming_topk)
      .def("compute_val_tppr", &ParallelTppRComputer::compute_val_tppr)
      .def("get_ret", [](const ParallelTppRComputer& c) { return c.ret; });

  py::class_<SplitResult>(m, "SplitResult")
      .def_readwrite("group_index", &SplitResult::group_index)
      .def_readwrite("keep_indices", &SplitResult::keep_indices)
      .def_readwrite("drop_proportion", &SplitResult::drop_proportion);
  m.def("adaptive_split", &adaptive_split, py::arg("src"), py::arg("dst"), py::arg("ts"), py::arg("base_batch_size"),
        py::arg("graph_feature"), py::arg("alpha") = 1.0, py::arg("beta") = 0.5, py::arg("aggl") = 0.0,
        py::arg("enable_drop") = false, py::arg("drop_rate") = 0.8, py::arg("window_size") = 1000);
}
