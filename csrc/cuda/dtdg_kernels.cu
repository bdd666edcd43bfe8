// DTDG (Flare) kernels for sm_100a:
//   * CSR SpMM for GCN aggregation: out[d] = sum_{e in row d} val[e] * x[col[e]]
//     (warp per destination row, 16-byte vectors over features). The backward
//     pass runs the same kernel over the source-sorted (transposed) CSR, so no
//     atomics are needed and results are deterministic.
//   * LSTM cell backward (elementwise over the saved gates).
#include "kernels.h"

namespace su {

template <int VEC>
__global__ void spmm_csr_kernel(const int64_t* __restrict__ rowptr, const int* __restrict__ col,
                                const float* __restrict__ val, const float* __restrict__ x, int64_t n_rows, int F,
                                float* __restrict__ out, int accumulate) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const int64_t lo = rowptr[row], hi = rowptr[row + 1];
  // every lane takes part in every shuffle; lanes beyond F only skip their loads
  for (int fbase = 0; fbase < F; fbase += 32 * VEC) {
    const int f0 = fbase + lane * VEC;
    const bool active = f0 < F;
    float acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
    for (int64_t e0 = lo; e0 < hi; e0 += 32) {
      const int64_t my = e0 + lane;
      const int mc = my < hi ? col[my] : 0;
      const float mv = my < hi ? val[my] : 0.f;
      const int cnt = static_cast<int>((hi - e0) < 32 ? (hi - e0) : 32);
      for (int j = 0; j < cnt; ++j) {
        const int c = __shfl_sync(0xffffffffu, mc, j);
        const float w = __shfl_sync(0xffffffffu, mv, j);
        if (!active) continue;
        const float* xr = x + static_cast<int64_t>(c) * F + f0;
        if (VEC == 4) {
          const float4 t = *reinterpret_cast<const float4*>(xr);
          acc[0] = fmaf(w, t.x, acc[0]);
          acc[1] = fmaf(w, t.y, acc[1]);
          acc[2] = fmaf(w, t.z, acc[2]);
          acc[3] = fmaf(w, t.w, acc[3]);
        } else if (VEC == 2) {
          const float2 t = *reinterpret_cast<const float2*>(xr);
          acc[0] = fmaf(w, t.x, acc[0]);
          acc[1] = fmaf(w, t.y, acc[1]);
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[v] = fmaf(w, xr[v], acc[v]);
        }
      }
    }
    if (active) {
      float* o = out + row * F + f0;
#pragma unroll
      for (int v = 0; v < VEC; ++v) o[v] = accumulate ? o[v] + acc[v] : acc[v];
    }
  }
}

void launch_spmm_csr(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val, const float* x,
                     int64_t n_rows, int F, float* out, int accumulate) {
  const int threads = 256;
  const int64_t blocks = (n_rows * 32 + threads - 1) / threads;
  if (blocks == 0) return;
  if (F % 128 == 0) spmm_csr_kernel<4><<<blocks, threads, 0, st>>>(rowptr, col, val, x, n_rows, F, out, accumulate);
  else if (F % 64 == 0) spmm_csr_kernel<2><<<blocks, threads, 0, st>>>(rowptr, col, val, x, n_rows, F, out, accumulate);
  else spmm_csr_kernel<1><<<blocks, threads, 0, st>>>(rowptr, col, val, x, n_rows, F, out, accumulate);
}

// d(pre-activation) of the four gates and dc_prev from dh', dc' and the saved gates.
__global__ void lstm_bwd_kernel(const float* __restrict__ gates, const float* __restrict__ c_prev,
                                const float* __restrict__ c_new, const float* __restrict__ dh,
                                const float* __restrict__ dc, int64_t rows, int H, float* __restrict__ dpre,
                                float* __restrict__ dc_prev) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * H) return;
  const int64_t r = idx / H;
  const int c = static_cast<int>(idx % H);
  const float* g = gates + r * 4 * H;
  const float i = g[c], f = g[H + c], gg = g[2 * H + c], o = g[3 * H + c];
  const float cn = c_new[idx];
  const float tc = tanhf(cn);
  const float dhv = dh ? dh[idx] : 0.f;
  const float dct = (dc ? dc[idx] : 0.f) + dhv * o * (1.f - tc * tc);
  const float cp = c_prev ? c_prev[idx] : 0.f;
  float* d = dpre + r * 4 * H;
  d[c] = dct * gg * i * (1.f - i);
  d[H + c] = dct * cp * f * (1.f - f);
  d[2 * H + c] = dct * i * (1.f - gg * gg);
  d[3 * H + c] = dhv * tc * o * (1.f - o);
  if (dc_prev) dc_prev[idx] = dct * f;
}

void launch_lstm_bwd(cudaStream_t st, const float* gates, const float* c_prev, const float* c_new, const float* dh,
                     const float* dc, int64_t rows, int H, float* dpre, float* dc_prev) {
  const int64_t n = rows * H;
  if (n == 0) return;
  lstm_bwd_kernel<<<(n + 255) / 256, 256, 0, st>>>(gates, c_prev, c_new, dh, dc, rows, H, dpre, dc_prev);
}

}  // namespace su
