// DTDG (Flare) kernels for sm_100a:
//   * CSR SpMM for GCN aggregation: out[d] = sum_{e in row d} val[e] * x[col[e]]
//     (warps over fixed-size edge chunks, vectors over features). The backward
//     pass runs the same kernel over the source-sorted (transposed) CSR. Rows
//     inside one chunk are written directly; rows longer than a chunk (hubs)
//     are combined with atomic adds.
//   * LSTM cell backward (elementwise over the saved gates).
#include "kernels.h"

namespace su {

// Work-balanced CSR SpMM. Power-law snapshots have hub rows with ~10^5 edges,
// so a warp per row leaves one warp walking a hub while the rest of the GPU
// idles. Instead every warp takes a fixed chunk of kChunk consecutive edges of
// the CSR: it finds the row holding its first edge (binary search in rowptr),
// accumulates row segment by row segment, and flushes each segment with a plain
// store when the whole row lies inside the chunk, or an atomic add when the
// row is shared with a neighbouring chunk (the output was zeroed first, or
// holds the value to accumulate onto).
constexpr int kSpmmChunk = 256;

// where a source row lives: one local matrix, or any rank's copy of a symmetric
// staging buffer (owner / row per source row, for the NVLink halo path)
struct LocalRows {
  const float* x;
  int F;
  __device__ __forceinline__ const float* row(int c) const { return x + static_cast<int64_t>(c) * F; }
};
struct PeerRows {
  const float* const* peers;
  const int* owner;
  const int* lrow;
  int F;
  __device__ __forceinline__ const float* row(int c) const {
    return peers[owner[c]] + static_cast<int64_t>(lrow[c]) * F;
  }
};
// where a finished row segment goes: this rank's output (plain store for rows
// inside the chunk, atomic add for rows shared with another chunk), or pushed
// into the owner rank's buffer with a remote atomic add
struct LocalOut {
  float* out;
  int F;
  int accumulate;
  __device__ __forceinline__ void put(int64_t row, int f, float v, bool whole) const {
    float* o = out + row * F + f;
    if (whole) *o = accumulate ? *o + v : v;
    else atomicAdd(o, v);
  }
};
struct PeerPush {
  float* const* peers;
  const int* owner;
  const int* lrow;
  int F;
  __device__ __forceinline__ void put(int64_t row, int f, float v, bool /*whole*/) const {
    atomicAdd(peers[owner[row]] + static_cast<int64_t>(lrow[row]) * F + f, v);
  }
};

template <int VEC, class Rows, class Out>
__global__ void spmm_chunked_kernel(const int64_t* __restrict__ rowptr, const int* __restrict__ col,
                                    const float* __restrict__ val, const Rows rows, int64_t n_rows, int F,
                                    const Out out) {
  const int lane = threadIdx.x & 31;
  const int64_t nnz = rowptr[n_rows];
  const int64_t nchunks = (nnz + kSpmmChunk - 1) / kSpmmChunk;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t ch = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; ch < nchunks;
       ch += warps) {
    const int64_t cb = ch * kSpmmChunk;
    const int64_t ce = (cb + kSpmmChunk < nnz) ? cb + kSpmmChunk : nnz;
    // row holding edge cb: last r with rowptr[r] <= cb
    int64_t lo = 0, hi = n_rows;
    while (hi - lo > 1) {
      const int64_t mid = (lo + hi) >> 1;
      if (rowptr[mid] <= cb) lo = mid;
      else hi = mid;
    }
    int64_t row = lo;
    int64_t e = cb;
    while (e < ce) {
      const int64_t rs = rowptr[row], re = rowptr[row + 1];
      const int64_t se = re < ce ? re : ce;
      const bool whole = rs >= cb && re <= ce;
      // every lane takes part in every shuffle; lanes beyond F only skip their loads
      for (int fbase = 0; fbase < F; fbase += 32 * VEC) {
        const int f0 = fbase + lane * VEC;
        const bool active = f0 < F;
        float acc[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
        for (int64_t e0 = e; e0 < se; e0 += 32) {
          const int64_t my = e0 + lane;
          const int mc = my < se ? col[my] : 0;
          const float mv = my < se ? val[my] : 0.f;
          const int cnt = static_cast<int>((se - e0) < 32 ? (se - e0) : 32);
          for (int j = 0; j < cnt; ++j) {
            const int c = __shfl_sync(0xffffffffu, mc, j);
            const float w = __shfl_sync(0xffffffffu, mv, j);
            if (!active) continue;
            const float* xr = rows.row(c) + f0;
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
#pragma unroll
          for (int v = 0; v < VEC; ++v) out.put(row, f0 + v, acc[v], whole);
        }
      }
      e = se;
      ++row;
    }
  }
}

template <class Rows, class Out>
static void launch_chunked(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val, const Rows& rows,
                           int64_t n_rows, int F, const Out& out) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int threads = 256;
  const int blocks = num_sms(dev) * 8;  // grid-stride over edge chunks (nnz is on the device)
  count_launch();
  if (F % 128 == 0) spmm_chunked_kernel<4><<<blocks, threads, 0, st>>>(rowptr, col, val, rows, n_rows, F, out);
  else if (F % 64 == 0) spmm_chunked_kernel<2><<<blocks, threads, 0, st>>>(rowptr, col, val, rows, n_rows, F, out);
  else spmm_chunked_kernel<1><<<blocks, threads, 0, st>>>(rowptr, col, val, rows, n_rows, F, out);
}

void launch_spmm_csr(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val, const float* x,
                     int64_t n_rows, int F, float* out, int accumulate) {
  if (n_rows == 0) return;
  // rows without edges and rows shared between chunks start from zero
  if (!accumulate) cudaMemsetAsync(out, 0, static_cast<size_t>(n_rows) * F * sizeof(float), st);
  launch_chunked(st, rowptr, col, val, LocalRows{x, F}, n_rows, F, LocalOut{out, F, accumulate});
}

// Halo-fused aggregation: source rows are read from the owners' staging
// buffers over NVLink (local rows from this rank's own buffer).
void launch_spmm_peer_gather(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val,
                             const float* const* peers, const int* src_owner, const int* src_row, int64_t n_rows,
                             int F, float* out) {
  if (n_rows == 0) return;
  cudaMemsetAsync(out, 0, static_cast<size_t>(n_rows) * F * sizeof(float), st);
  launch_chunked(st, rowptr, col, val, PeerRows{peers, src_owner, src_row, F}, n_rows, F, LocalOut{out, F, 0});
}

// Its backward over the transposed CSR (rows = source rows): each source row's
// gradient is pushed into the owner's gradient buffer with remote atomic adds.
void launch_spmm_peer_push(cudaStream_t st, const int64_t* rowptr_t, const int* col_t, const float* val_t,
                           const float* grad_dst, int64_t n_src, int F, float* const* peers, const int* src_owner,
                           const int* src_row) {
  if (n_src == 0) return;
  launch_chunked(st, rowptr_t, col_t, val_t, LocalRows{grad_dst, F}, n_src, F,
                 PeerPush{peers, src_owner, src_row, F});
}

// d(pre-activation) of the four gates and dc_prev from dh', dc' and the saved gates.
__global__ void lstm_bwd_kernel(const float* __restrict__ gates, const float* __restrict__ c_prev,
                                const float* __restrict__ c_new, const float* __restrict__ dh, int dh_ld,
                                const float* __restrict__ dc, int dc_ld, int64_t rows, int H,
                                float* __restrict__ dpre, float* __restrict__ dc_prev) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * H) return;
  const int64_t r = idx / H;
  const int c = static_cast<int>(idx % H);
  const float* g = gates + r * 4 * H;
  const float i = g[c], f = g[H + c], gg = g[2 * H + c], o = g[3 * H + c];
  const float cn = c_new[idx];
  const float tc = tanhf(cn);
  const float dhv = dh ? dh[r * dh_ld + c] : 0.f;
  const float dct = (dc ? dc[r * dc_ld + c] : 0.f) + dhv * o * (1.f - tc * tc);
  const float cp = c_prev ? c_prev[idx] : 0.f;
  float* d = dpre + r * 4 * H;
  d[c] = dct * gg * i * (1.f - i);
  d[H + c] = dct * cp * f * (1.f - f);
  d[2 * H + c] = dct * i * (1.f - gg * gg);
  d[3 * H + c] = dhv * tc * o * (1.f - o);
  if (dc_prev) dc_prev[idx] = dct * f;
}

void launch_lstm_bwd(cudaStream_t st, const float* gates, const float* c_prev, const float* c_new, const float* dh,
                     int dh_ld, const float* dc, int dc_ld, int64_t rows, int H, float* dpre, float* dc_prev) {
  const int64_t n = rows * H;
  if (n == 0) return;
  count_launch();
  lstm_bwd_kernel<<<(n + 255) / 256, 256, 0, st>>>(gates, c_prev, c_new, dh, dh_ld, dc, dc_ld, rows, H, dpre,
                                                   dc_prev);
}

}  // namespace su
