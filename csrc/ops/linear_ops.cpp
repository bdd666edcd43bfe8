// nn.Linear forward / data-gradient / weight-gradient on the tcgen05 GEMM.
//
//   linear_fwd     : Y = act(X W^T + b)
//   linear_dgrad   : dX = dY W              (B operand = W^T evaluated on the fly)
//   linear_wgrad   : dW += dY^T X, db += sum_rows dY   (split-K, atomic epilogue;
//   (both take dY with any row stride, and an optional mask: dY is read as
//   dY * (mask > 0), the ReLU derivative from the forward output)
//                    the bias gradient comes from a constant-1 column appended
//                    to X inside the producer)
#include "host_common.h"

using namespace su;

// Reads (and optionally clears) the device status word. Synchronises the stream.
int64_t status_read(bool clear) {
  const int dev = at::cuda::current_device();
  int h = 0;
  int* p = device_status_ptr(dev);
  C10_CUDA_CHECK(cudaMemcpyAsync(&h, p, sizeof(int), cudaMemcpyDeviceToHost, cur_stream()));
  C10_CUDA_CHECK(cudaStreamSynchronize(cur_stream()));
  if (clear) C10_CUDA_CHECK(cudaMemsetAsync(p, 0, sizeof(int), cur_stream()));
  return h;
}

static WeightLayout single_weight_layout(const at::Tensor& w) {
  const int N = static_cast<int>(w.size(0)), K = static_cast<int>(w.size(1));
  WeightLayout L;
  L.nblk = 1;
  L.nseg = 1;
  L.blk_rows[0] = N;
  L.blk_pad[0] = N;
  L.seg_kpad[0] = pad8(K);
  L.cell[0][0] = wcell(w, 0, 0, K);
  return L;
}

static void linear_fwd_impl(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                            int64_t act, at::Tensor& y) {
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(w.size(0));
  if (M == 0) return;
  SegSource a;
  a.nseg = 1;
  a.seg[0] = seg_f32(x, K, pad8(K));
  WeightSource b;
  b.L = single_weight_layout(w);
  EpiLinear e;
  e.out = y.data_ptr<float>();
  e.ldo = static_cast<int>(y.stride(0));
  e.ncols = N;
  e.bias = opt_ptr<float>(bias);
  e.act = static_cast<int>(act);
  GemmShape sh;
  sh.M = M;
  sh.N = N;
  sh.K = pad8(K);
  gemm(a, b, e, sh, cur_stream());
  SU_LAUNCH_CHECK();
}

// dY as an operand segment: unit column stride, any row stride, optionally masked
// by the forward output (ReLU derivative, mask[r, c] > 0) while it is packed
static ASeg grad_seg(const at::Tensor& dy, int N, const c10::optional<at::Tensor>& mask) {
  TORCH_CHECK(dy.dim() == 2 && dy.stride(1) == 1, "dy must be a row-major matrix (any row stride)");
  ASeg s = seg_f32(dy, N, pad8(N));
  if (mask.has_value() && mask->defined()) {
    SU_CHECK_F32(*mask);
    TORCH_CHECK(mask->dim() == 2 && mask->size(0) == dy.size(0) && mask->size(1) == dy.size(1) &&
                    mask->stride(1) == 1,
                "mask must be a row-major matrix of dy's shape");
    s.mask = mask->data_ptr<float>();
    s.mask_ld = static_cast<int>(mask->stride(0));
    if ((s.mask_ld % 4) != 0 || (reinterpret_cast<uintptr_t>(s.mask) % 16) != 0) s.vec = 0;
  }
  return s;
}

at::Tensor linear_fwd(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, int64_t act) {
  SU_CHECK_CUDA(x); SU_CHECK_F32(x); SU_CHECK_F32(w); SU_CHECK_CONTIG(w);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be a row-major matrix");
  TORCH_CHECK(w.size(1) == x.size(1), "shape mismatch");
  auto y = at::empty({x.size(0), w.size(0)}, x.options());
  linear_fwd_impl(x, w, bias, act, y);
  return y;
}

// The same into `out` ([M, N], unit column stride, any row stride): e.g. the rows of a
// symmetric staging buffer that peer GPUs read.
void linear_fwd_into(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, int64_t act,
                     at::Tensor& out) {
  SU_CHECK_CUDA(x); SU_CHECK_F32(x); SU_CHECK_F32(w); SU_CHECK_CONTIG(w); SU_CHECK_F32(out);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be a row-major matrix");
  TORCH_CHECK(w.size(1) == x.size(1), "shape mismatch");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == x.size(0) && out.size(1) == w.size(0) && out.stride(1) == 1 &&
                  out.stride(0) >= out.size(1),
              "out must be an [M, N] row-major view");
  linear_fwd_impl(x, w, bias, act, out);
}

at::Tensor linear_dgrad(const at::Tensor& dy, const at::Tensor& w, const c10::optional<at::Tensor>& mask) {
  SU_CHECK_CUDA(dy); SU_CHECK_F32(dy); SU_CHECK_F32(w); SU_CHECK_CONTIG(w);
  const int M = static_cast<int>(dy.size(0)), N = static_cast<int>(w.size(0)), K = static_cast<int>(w.size(1));
  auto dx = at::empty({M, K}, dy.options());
  if (M == 0) return dx;
  SegSource a;
  a.nseg = 1;
  a.seg[0] = grad_seg(dy, N, mask);
  WeightLayout L = single_weight_layout(w);
  L.blk_pad[0] = pad8(N);
  WeightMN b = weight_mn(L, pad8(N));
  EpiLinear e;
  e.out = dx.data_ptr<float>();
  e.ldo = K;
  e.ncols = K;
  GemmShape sh;
  sh.M = M;
  sh.N = K;
  sh.K = pad8(N);
  gemm(a, b, e, sh, cur_stream());
  SU_LAUNCH_CHECK();
  return dx;
}

void linear_wgrad(const at::Tensor& dy, const at::Tensor& x, at::Tensor& dw, const c10::optional<at::Tensor>& db,
                  const c10::optional<at::Tensor>& mask) {
  SU_CHECK_CUDA(dy); SU_CHECK_F32(dy); SU_CHECK_F32(x); SU_CHECK_F32(dw); SU_CHECK_CONTIG(dw);
  const int M = static_cast<int>(dy.size(0)), N = static_cast<int>(dy.size(1)), K = static_cast<int>(x.size(1));
  if (M == 0) return;
  SegSource dys;  // A[n, m] = dY[m, n] (MN-major view)
  dys.nseg = 1;
  dys.seg[0] = grad_seg(dy, N, mask);
  SegSource xs;  // B[k, m] = X[m, k] (+ ones column for the bias gradient)
  xs.nseg = 2;
  xs.seg[0] = seg_f32(x, K, pad8(K));
  xs.seg[1] = seg_ones();
  SegMN a = seg_mn(dys, M);
  SegMN b = seg_mn(xs, M);
  EpiWeightGrad e;
  e.L.nblk = 1;
  e.L.nseg = 2;
  e.L.blk_rows[0] = N;
  e.L.blk_pad[0] = N;
  e.L.seg_kpad[0] = pad8(K);
  e.L.seg_kpad[1] = 8;
  e.L.cell[0][0] = wcell(dw, 0, 0, K);
  e.bias_grad[0] = (db.has_value() && db->defined()) ? db->data_ptr<float>() : nullptr;
  e.bias_seg = 1;
  e.ncols = pad8(K) + 8;
  GemmShape sh;
  sh.M = N;
  sh.N = pad8(K) + 8;
  sh.K = M;
  const int nchunks = (M + kBK - 1) / kBK;
  const int tiles = ((N + kBM - 1) / kBM) * ((sh.N + 255) / 256);
  sh.ksplit = wgrad_ksplit(nchunks, tiles);
  gemm(a, b, e, sh, cur_stream());
  SU_LAUNCH_CHECK();
}
