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
