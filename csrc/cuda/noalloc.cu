// Allocation-free fused LSTM-cell backward (declared in noalloc.h, which states
// the caller rules). Same kernels as the `lstm_bwd` op of the Python extension;
// the gate-gradient temporary (and, when in_dim is not a multiple of 8, the
// padded input-gradient tile) lives in the static scratch array below.
#include <cstdint>

#include "kernels.h"
#include "noalloc.h"

namespace su {
namespace {

constexpr size_t kScratchFloats = SU_NOALLOC_SCRATCH_BYTES / sizeof(float);

// One scratch array and one status word per device (each device gets its own
// copy of a module's __device__ variables).
__device__ __align__(256) float g_scratch[kScratchFloats];
__device__ __align__(16) int g_status[4];

float* g_scratch_addr[64] = {nullptr};
int* g_status_addr[64] = {nullptr};

inline int pad8i(int x) { return (x + 7) / 8 * 8; }
inline size_t round_up64(size_t n) { return (n + 63) / 64 * 64; }

// dxh[r, 0:in) = tmp[r, 0:in); dxh[r, in:in+H) = tmp[r, pad8(in):pad8(in)+H)
__global__ void compact_dxh_kernel(const float* __restrict__ tmp, int ld_tmp, int in_dim, int in_pad, int H,
                                   int64_t rows, float* __restrict__ dxh) {
  const int width = in_dim + H;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * width) return;
  const int64_t r = idx / width;
  const int c = static_cast<int>(idx % width);
  const int src = c < in_dim ? c : (in_pad + (c - in_dim));
  dxh[idx] = tmp[r * ld_tmp + src];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

WCell cell(const float* w, int ld, int col0, int width) {
  WCell c;
  c.ptr = w;
  c.ld = ld;
  c.row0 = 0;
  c.col0 = col0;
  c.width = width;
  c.vec = ((ld % 4) == 0 && (col0 % 4) == 0 && aligned16(w)) ? 1 : 0;
  return c;
}

ASeg f32_seg(const float* p, int ld, int width, int kpad) {
  ASeg s;
  s.kind = kSegF32;
  s.ptr = p;
  s.ld = ld;
  s.width = width;
  s.kpad = kpad;
  s.vec = ((ld % 4) == 0 && aligned16(p)) ? 1 : 0;
  return s;
}

WeightLayout gate_layout(const float* const w[4], int in_dim, int H) {
  WeightLayout L;
  L.nblk = 4;
  L.nseg = 2;
  L.seg_kpad[0] = pad8i(in_dim);
  L.seg_kpad[1] = pad8i(H);
  for (int i = 0; i < 4; ++i) {
    L.blk_rows[i] = H;
    L.blk_pad[i] = H;
    L.cell[i][0] = cell(w[i], in_dim + H, 0, in_dim);
    L.cell[i][1] = cell(w[i], in_dim + H, in_dim, H);
  }
  return L;
}

// Looks up this device's scratch and status addresses once (no allocation).
int device_symbols(float** scratch, int** status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SU_NOALLOC_ERR_CUDA;
  if (g_scratch_addr[dev] == nullptr) {
    void* s = nullptr;
    void* st = nullptr;
    if (cudaGetSymbolAddress(&s, g_scratch) != cudaSuccess) return SU_NOALLOC_ERR_CUDA;
    if (cudaGetSymbolAddress(&st, g_status) != cudaSuccess) return SU_NOALLOC_ERR_CUDA;
    g_scratch_addr[dev] = static_cast<float*>(s);
    g_status_addr[dev] = static_cast<int*>(st);
  }
  *scratch = g_scratch_addr[dev];
  *status = g_status_addr[dev];
  return SU_NOALLOC_OK;
}

}  // namespace
}  // namespace su

using namespace su;

#define SU_EXPORT __attribute__((visibility("default")))

extern "C" SU_EXPORT size_t su_noalloc_scratch_required(int rows, int in_dim, int hidden) {
  if (rows <= 0 || in_dim <= 0 || hidden <= 0) return 0;
  size_t floats = round_up64(static_cast<size_t>(rows) * 4 * hidden);
  if (pad8i(in_dim) != in_dim) floats += static_cast<size_t>(rows) * (pad8i(in_dim) + pad8i(hidden));
  return floats * sizeof(float);
}

extern "C" SU_EXPORT size_t su_noalloc_scratch_capacity(void) { return SU_NOALLOC_SCRATCH_BYTES; }

extern "C" SU_EXPORT const char* su_noalloc_strerror(int code) {
  switch (code) {
    case SU_NOALLOC_OK:
      return "ok";
    case SU_NOALLOC_ERR_ARGUMENT:
      return "invalid argument: a required pointer is NULL or not 16-byte aligned, or a size is not positive";
    case SU_NOALLOC_ERR_SCRATCH:
      return "the call needs more scratch than the static array holds (see su_noalloc_scratch_required and "
             "su_noalloc_scratch_capacity); split the rows into several calls";
    case SU_NOALLOC_ERR_CUDA:
      return "a CUDA runtime call or kernel launch failed (cudaGetLastError has the cause)";
    default:
      return "unknown code";
  }
}

extern "C" SU_EXPORT int su_noalloc_status(int* out4) {
  float* scratch = nullptr;
  int* status = nullptr;
  if (out4 == nullptr) return SU_NOALLOC_ERR_ARGUMENT;
  if (device_symbols(&scratch, &status) != SU_NOALLOC_OK) return SU_NOALLOC_ERR_CUDA;
  // every stream of the device, non-blocking ones included, finishes first: the copy
  // below runs on the legacy default stream, which is not ordered with those
  if (cudaDeviceSynchronize() != cudaSuccess) return SU_NOALLOC_ERR_CUDA;
  if (cudaMemcpyFromSymbol(out4, g_status, sizeof(int) * 4) != cudaSuccess) return SU_NOALLOC_ERR_CUDA;
  return SU_NOALLOC_OK;
}

extern "C" SU_EXPORT int su_noalloc_status_reset(void) {
  float* scratch = nullptr;
  int* status = nullptr;
  if (device_symbols(&scratch, &status) != SU_NOALLOC_OK) return SU_NOALLOC_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return SU_NOALLOC_ERR_CUDA;
  if (cudaMemset(status, 0, sizeof(int) * 4) != cudaSuccess) return SU_NOALLOC_ERR_CUDA;
  return SU_NOALLOC_OK;
}

extern "C" SU_EXPORT int su_lstm_cell_backward_noalloc(
    const float* x, const float* h_prev, const float* c_prev, const float* c_new, const float* gates,
    const float* dh, const float* dc, const float* w_i, const float* w_f, const float* w_g, const float* w_o,
    float* gw_i, float* gb_i, float* gw_f, float* gb_f, float* gw_g, float* gb_g, float* gw_o, float* gb_o,
    float* dxh, float* dc_prev, int rows, int in_dim, int hidden, void* stream) {
  if (rows <= 0 || in_dim <= 0 || hidden <= 0) return SU_NOALLOC_ERR_ARGUMENT;
  const void* required[] = {x, c_new, gates, w_i, w_f, w_g, w_o, gw_i, gb_i, gw_f, gb_f, gw_g, gb_g, gw_o, gb_o,
                            dxh, dc_prev};
  for (const void* p : required)
    if (p == nullptr || !aligned16(p)) return SU_NOALLOC_ERR_ARGUMENT;
  const void* optional[] = {h_prev, c_prev, dh, dc};
  for (const void* p : optional)
    if (p != nullptr && !aligned16(p)) return SU_NOALLOC_ERR_ARGUMENT;
  if (su_noalloc_scratch_required(rows, in_dim, hidden) > SU_NOALLOC_SCRATCH_BYTES) return SU_NOALLOC_ERR_SCRATCH;

  float* scratch = nullptr;
  int* status = nullptr;
  if (device_symbols(&scratch, &status) != SU_NOALLOC_OK) return SU_NOALLOC_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int H = hidden;
  const int DP4 = 4 * H;
  const int in_pad = pad8i(in_dim), h_pad = pad8i(H);
  float* dpre = scratch;
  float* tmp = scratch + round_up64(static_cast<size_t>(rows) * DP4);

  // 1. gate pre-activation gradients (scratch) and d c_prev
  launch_lstm_bwd(st, gates, c_prev, c_new, dh, H, dc, H, rows, H, dpre, dc_prev);

  // 2. d[x || h] = dpre [W_i; W_f; W_g; W_o]
  {
    SegSource a;
    a.nseg = 1;
    a.seg[0] = f32_seg(dpre, DP4, DP4, pad8i(DP4));
    const float* w[4] = {w_i, w_f, w_g, w_o};
    MNView<WeightSource> b;
    b.inner.L = gate_layout(w, in_dim, H);
    b.inner.L.blk_pad[3] = pad8i(DP4) - 3 * H;
    b.inner_rows = pad8i(DP4);
    EpiLinear e;
    GemmShape sh;
    sh.M = rows;
    sh.N = in_pad + h_pad;
    sh.K = pad8i(DP4);
    if (in_pad != in_dim) {  // padded K space: write the padded tile, then compact
      e.out = tmp;
      e.ldo = in_pad + h_pad;
      e.ncols = in_pad + h_pad;
      gemm_with_status(a, b, e, sh, st, status);
      const int64_t n = static_cast<int64_t>(rows) * (in_dim + H);
      compact_dxh_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(tmp, in_pad + h_pad, in_dim, in_pad,
                                                                                H, rows, dxh);
    } else {
      e.out = dxh;
      e.ldo = in_dim + H;
      e.ncols = in_dim + H;
      gemm_with_status(a, b, e, sh, st, status);
    }
  }

  // 3. dW_gate += dpre_gate^T [x || h || 1]  (the ones column gives the bias gradient)
  {
    SegSource dy;
    dy.nseg = 1;
    dy.seg[0] = f32_seg(dpre, DP4, DP4, pad8i(DP4));
    SegSource xs;
    xs.nseg = 3;
    xs.seg[0] = f32_seg(x, in_dim, in_dim, in_pad);
    if (h_prev != nullptr) {
      xs.seg[1] = f32_seg(h_prev, H, H, h_pad);
    } else {
      xs.seg[1].kind = kSegZero;
      xs.seg[1].kpad = h_pad;
    }
    xs.seg[2].kind = kSegOnes;
    xs.seg[2].width = 1;
    xs.seg[2].kpad = 8;
    MNView<SegSource> ta;
    ta.inner = dy;
    ta.inner_rows = rows;
    MNView<SegSource> tb;
    tb.inner = xs;
    tb.inner_rows = rows;
    float* gw[4] = {gw_i, gw_f, gw_g, gw_o};
    EpiWeightGrad e;
    e.L = gate_layout(gw, in_dim, H);
    e.L.nseg = 3;
    e.L.seg_kpad[2] = 8;
    float* gb[4] = {gb_i, gb_f, gb_g, gb_o};
    for (int i = 0; i < 4; ++i) e.bias_grad[i] = gb[i];
    e.bias_seg = 2;
    e.ncols = in_pad + h_pad + 8;
    GemmShape sh;
    sh.M = DP4;
    sh.N = e.ncols;
    sh.K = rows;
    int dev = 0;
    cudaGetDevice(&dev);
    const int nchunks = (rows + kBK - 1) / kBK;
    const int tiles = ((DP4 + kBM - 1) / kBM) * ((sh.N + 255) / 256);
    int want = (2 * num_sms(dev)) / (tiles > 0 ? tiles : 1);
    if (want < 1) want = 1;
    sh.ksplit = want < nchunks ? want : nchunks;
    gemm_with_status(ta, tb, e, sh, st, status);
  }
  return cudaGetLastError() == cudaSuccess ? SU_NOALLOC_OK : SU_NOALLOC_ERR_CUDA;
}
