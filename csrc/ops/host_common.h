// Host-side helpers shared by the CUDA extension translation units.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "kernels.h"

#define SU_CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define SU_CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define SU_CHECK_F32(x) TORCH_CHECK((x).scalar_type() == at::kFloat, #x " must be float32")
#define SU_CHECK_I64(x) TORCH_CHECK((x).scalar_type() == at::kLong, #x " must be int64")
#define SU_CHECK_I32(x) TORCH_CHECK((x).scalar_type() == at::kInt, #x " must be int32")
#define SU_LAUNCH_CHECK() C10_CUDA_KERNEL_LAUNCH_CHECK()

namespace su {

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

template <class T>
inline const T* opt_ptr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr<T>() : nullptr;
}

inline int pad8(int x) { return (x + 7) / 8 * 8; }

// Split-K factor of a weight-gradient GEMM (K = the data rows): with many
// k-chunks every split accumulates at least 12 of them (768 rows) in TMEM
// before its one atomic flush (the flush atomics, not the copies, bound these
// small-output GEMMs); with few (K = one row per root, ~20 chunks) a single CTA
// walking them all is latency-bound (~20 us measured for 19 chunks), so splits
// of 4 chunks run side by side. The splits x output tiles fill the SMs at most once.
inline int wgrad_ksplit(int nchunks, int tiles) {
  const int sms = num_sms(at::cuda::current_device());
  const int by_work = std::max(1, nchunks / (nchunks >= 96 ? 12 : 4));
  const int by_sms = std::max(1, sms / std::max(1, tiles));
  return std::max(1, std::min(by_work, by_sms));
}

// 16-byte alignment of a device pointer (nullptr counts as aligned)
inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// vector flag of the GRU / tanh-RNN epilogue: row strides multiples of 4 floats and
// every local pointer 16-byte aligned (peer tables are symmetric-memory
// allocations, whose bases are page aligned)
inline int gru_vec(const EpiGRU& e) {
  const bool ld = (e.D % 4 == 0) && (e.hprev == nullptr || e.hprev_ld % 4 == 0) &&
                  (e.hout == nullptr || e.hout_ld % 4 == 0) && (e.scatter == nullptr || e.scatter_ld % 4 == 0);
  return (ld && a16(e.hprev) && a16(e.hout) && a16(e.save_prev) && a16(e.scatter) && a16(e.b_ih) &&
          a16(e.b_hh) && e.DP % 16 == 0) ? 1 : 0;
}

// fp32 matrix segment (row-major, gathered through `index` if given)
inline ASeg seg_f32(const at::Tensor& m, int width, int kpad, const int64_t* index = nullptr, int col0 = 0) {
  ASeg s;
  s.kind = kSegF32;
  s.ptr = m.data_ptr<float>();
  s.ld = static_cast<int>(m.stride(0));
  s.col0 = col0;
  s.width = width;
  s.kpad = kpad;
  s.index = index;
  s.vec = ((s.ld % 4) == 0 && (col0 % 4) == 0 && (reinterpret_cast<uintptr_t>(s.ptr) % 16) == 0) ? 1 : 0;
  return s;
}
// bf16 matrix segment (row-major)
inline ASeg seg_bf16(const at::Tensor& m, int width, int kpad, const int64_t* index = nullptr) {
  ASeg s;
  s.kind = kSegBF16;
  s.ptr = m.data_ptr();
  s.ld = static_cast<int>(m.stride(0));
  s.width = width;
  s.kpad = kpad;
  s.index = index;
  s.vec = ((s.ld % 8) == 0 && (reinterpret_cast<uintptr_t>(s.ptr) % 16) == 0) ? 1 : 0;
  return s;
}
// edge-feature rows (fp32 or bf16 storage), gathered through `index`
inline ASeg seg_feat(const at::Tensor& m, int width, int kpad, const int64_t* index) {
  TORCH_CHECK(m.scalar_type() == at::kFloat || m.scalar_type() == at::kBFloat16,
              "edge features must be float32 or bfloat16");
  return m.scalar_type() == at::kBFloat16 ? seg_bf16(m, width, kpad, index) : seg_f32(m, width, kpad, index);
}
inline ASeg seg_time(const float* dt, const at::Tensor& w, const at::Tensor& b, int kpad) {
  ASeg s;
  s.kind = kSegTime;
  s.tdt = dt;
  s.tw = w.data_ptr<float>();
  s.tb = b.data_ptr<float>();
  s.width = static_cast<int>(b.numel());
  s.kpad = kpad;
  return s;
}
inline ASeg seg_ones() {
  ASeg s;
  s.kind = kSegOnes;
  s.width = 1;
  s.kpad = 8;
  return s;
}
inline WCell wcell(const at::Tensor& w, int row0, int col0, int width) {
  WCell c;
  c.ptr = w.data_ptr<float>();
  c.ld = static_cast<int>(w.stride(0));
  c.row0 = row0;
  c.col0 = col0;
  c.width = width;
  c.vec = ((c.ld % 4) == 0 && (col0 % 4) == 0 && (reinterpret_cast<uintptr_t>(c.ptr) % 16) == 0) ? 1 : 0;
  return c;
}

// Multi-GPU view of the CTDG node tables: rows live in the owner rank's table
// (peer pointers of symmetric allocations); rows of this step's roots are read
// from the local `mem_new` buffer once the memory updater has produced them.
// Passed from Python as a CPU int64 tensor of device addresses:
//   [mem_peers, mail_peers, owner, stamp, node2root, step_ctr, mem_new, ts_peers]
struct PeerDesc {
  bool on = false;
  const float* const* mem_peers = nullptr;
  const float* const* mail_peers = nullptr;
  const int* owner = nullptr;
  const int* stamp = nullptr;
  const int* node2root = nullptr;
  const int64_t* step_ctr = nullptr;
  float* mem_new = nullptr;
  const float* const* ts_peers = nullptr;
};

// (items [3 * n_items] int32, warp offsets [warps + 1] int32, split rows int32): the
// item-based SpMM plan of one CSR; nullopt or an empty list keeps the edge-stream kernel
inline SpmmPlan spmm_plan_from(const c10::optional<std::vector<at::Tensor>>& p, SpmmPlan* out) {
  SpmmPlan plan;
  if (!p.has_value() || p->empty()) return plan;
  TORCH_CHECK(p->size() == 3, "SpMM plan: (items, warp_off, split_rows)");
  const at::Tensor& items = (*p)[0];
  const at::Tensor& woff = (*p)[1];
  const at::Tensor& split = (*p)[2];
  SU_CHECK_I32(items); SU_CHECK_I32(woff); SU_CHECK_I32(split);
  TORCH_CHECK(items.numel() % 3 == 0 && woff.numel() >= 2, "malformed SpMM plan");
  plan.items = items.data_ptr<int>();
  plan.n_items = static_cast<int>(items.numel() / 3);
  plan.warp_off = woff.data_ptr<int>();
  plan.warps = static_cast<int>(woff.numel() - 1);
  plan.split_rows = split.numel() ? split.data_ptr<int>() : nullptr;
  plan.n_split = static_cast<int>(split.numel());
  *out = plan;
  return plan;
}

inline PeerDesc peer_desc(const c10::optional<at::Tensor>& t) {
  PeerDesc d;
  if (!t.has_value() || !t->defined()) return d;
  TORCH_CHECK(t->device().is_cpu() && t->scalar_type() == at::kLong && t->numel() >= 7, "bad peer descriptor");
  const int64_t* v = t->data_ptr<int64_t>();
  d.on = true;
  d.mem_peers = reinterpret_cast<const float* const*>(v[0]);
  d.mail_peers = reinterpret_cast<const float* const*>(v[1]);
  d.owner = reinterpret_cast<const int*>(v[2]);
  d.stamp = reinterpret_cast<const int*>(v[3]);
  d.node2root = reinterpret_cast<const int*>(v[4]);
  d.step_ctr = reinterpret_cast<const int64_t*>(v[5]);
  d.mem_new = reinterpret_cast<float*>(v[6]);
  if (t->numel() >= 8) d.ts_peers = reinterpret_cast<const float* const*>(v[7]);
  return d;
}

// memory rows gathered through `index`: the local table, or (multi-GPU) the
// owners' tables with this step's roots taken from mem_new when `fresh`
inline ASeg seg_memory(const at::Tensor& memory, int D, const int64_t* index, const PeerDesc& pd, bool fresh) {
  if (!pd.on) return seg_f32(memory, D, pad8(D), index);
  ASeg s;
  s.kind = kSegSharded;
  s.peers = pd.mem_peers;
  s.owner = pd.owner;
  s.ld = D;
  s.width = D;
  s.kpad = pad8(D);
  s.index = index;
  s.vec = (D % 4) == 0 ? 1 : 0;
  if (fresh) {
    s.stamp = pd.stamp;
    s.node2root = pd.node2root;
    s.step_ctr = pd.step_ctr;
    s.fresh = pd.mem_new;
    s.fresh_ld = D;
  }
  return s;
}

using WeightMN = MNView<WeightSource>;
using SegMN = MNView<SegSource>;

inline WeightMN weight_mn(const WeightLayout& L, int out_rows) {
  WeightMN v;
  v.inner.L = L;
  v.inner_rows = out_rows;
  return v;
}
inline SegMN seg_mn(const SegSource& s, int rows) {
  SegMN v;
  v.inner = s;
  v.inner_rows = rows;
  return v;
}

}  // namespace su
