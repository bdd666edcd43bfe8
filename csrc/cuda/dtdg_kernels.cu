// DTDG (Flare) kernels for sm_100a:
//   * CSR SpMM for GCN aggregation: out[d] = sum_{e in row d} val[e] * x[col[e]]
//     (warps over fixed-size edge chunks, vectors over features). The backward
//     pass runs the same kernel over the source-sorted (transposed) CSR. Rows
//     inside one chunk are written directly; rows longer than a chunk (hubs)
//     are combined with atomic adds.
//   * LSTM cell backward (elementwise over the saved gates, in the forward
//     epilogue's grouped order: lstm_gate_index).
#include <algorithm>

#include "kernels.h"

namespace su {

// Work-balanced CSR SpMM. Power-law snapshots have hub rows with ~10^5 edges,
// so a warp per row leaves one warp walking a hub while the rest of the GPU
// idles. Instead the edges are cut into one contiguous range per warp of a
// persistent grid (equal edge counts): the warp finds the row holding its first
// edge (a 33-ary search over rowptr, one probe per lane), then walks its range
// as a flat stream, gathering the source rows of several edges at a time
// whatever rows they belong to, and closes a row segment whenever the stream
// crosses a row end. A segment is flushed with a plain store when the whole row
// lies inside the range, with an atomic add when the row is shared with a
// neighbouring warp's range (the output was zeroed first, or holds the value to
// accumulate onto). Columns and weights are staged in shared memory in
// sub-chunks of kSpmmChunk edges.
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
// this rank's rows (columns below n_split, the layer input) and the halo rows
// pulled from the owners (columns from n_split on, in pull order)
struct TwoTables {
  const float* x;
  const float* halo;
  int n_split;
  int F;
  int ld;  // row stride of x (>= F: rows of a wider staging buffer)
  __device__ __forceinline__ const float* row(int c) const {
    return c < n_split ? x + static_cast<int64_t>(c) * ld : halo + static_cast<int64_t>(c - n_split) * F;
  }
};
// where a finished row segment goes: this rank's output (plain store for rows
// inside the chunk, atomic add for rows shared with another chunk), or pushed
// into the owner rank's buffer with a remote atomic add
// add v[0..VEC) to p[0..VEC) (16- or 8-byte aligned for VEC 4 / 2) with one vector reduction
template <int VEC>
__device__ __forceinline__ void red_add_vec(float* p, const float (&v)[VEC]) {
  if constexpr (VEC == 4) {
    asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3])
                 : "memory");
  } else if constexpr (VEC == 2) {
    asm volatile("red.global.add.v2.f32 [%0], {%1,%2};" ::"l"(p), "f"(v[0]), "f"(v[1]) : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) atomicAdd(p + i, v[i]);
  }
}

struct LocalOut {
  float* out;
  int F;
  int accumulate;
  __device__ __forceinline__ void put(int64_t row, int f, float v, bool whole) const {
    float* o = out + row * F + f;
    if (whole) *o = accumulate ? *o + v : v;
    else atomicAdd(o, v);
  }
  // VEC consecutive features at f (f a multiple of VEC; rows VEC-aligned since F % VEC == 0)
  template <int VEC>
  __device__ __forceinline__ void put_vec(int64_t row, int f, const float (&v)[VEC], bool whole) const {
    float* o = out + row * F + f;
    if (!whole) {
      red_add_vec<VEC>(o, v);
      return;
    }
    float w[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) w[i] = v[i];
    if (accumulate) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) w[i] += o[i];
    }
    if constexpr (VEC == 4) *reinterpret_cast<float4*>(o) = make_float4(w[0], w[1], w[2], w[3]);
    else if constexpr (VEC == 2) *reinterpret_cast<float2*>(o) = make_float2(w[0], w[1]);
    else
#pragma unroll
      for (int i = 0; i < VEC; ++i) o[i] = w[i];
  }
};
struct PeerPush {
  float* const* peers;
  const int* owner;
  const int* lrow;
  int ld;  // row stride of the owners' gradient buffers (>= the layer width)
  __device__ __forceinline__ void put(int64_t row, int f, float v, bool /*whole*/) const {
    atomicAdd(peers[owner[row]] + static_cast<int64_t>(lrow[row]) * ld + f, v);
  }
  template <int VEC>
  __device__ __forceinline__ void put_vec(int64_t row, int f, const float (&v)[VEC], bool /*whole*/) const {
    red_add_vec<VEC>(peers[owner[row]] + static_cast<int64_t>(lrow[row]) * ld + f, v);
  }
};

template <int VEC>
__device__ __forceinline__ void load_vec(const float* p, float (&t)[VEC]) {
  if constexpr (VEC == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    t[0] = a.x; t[1] = a.y; t[2] = a.z; t[3] = a.w;
  } else if constexpr (VEC == 2) {
    const float2 a = *reinterpret_cast<const float2*>(p);
    t[0] = a.x; t[1] = a.y;
  } else {
#pragma unroll
    for (int v = 0; v < VEC; ++v) t[v] = p[v];
  }
}

template <int VEC, class Rows, class Out>
__global__ void __launch_bounds__(256, 3) spmm_chunked_kernel(const int64_t* __restrict__ rowptr,
                                                              const int* __restrict__ col,
                                                              const float* __restrict__ val, const Rows rows,
                                                              int64_t n_rows, int F, const Out out) {
  constexpr int kUnroll = VEC == 4 ? 8 : 16;  // source rows in flight per lane
  constexpr int kPer = kSpmmChunk / 32;
  __shared__ int s_col[8][kSpmmChunk];
  __shared__ float s_val[8][kSpmmChunk];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  int* scol = s_col[wib];
  float* sval = s_val[wib];
  const int64_t nnz = rowptr[n_rows];
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  // this warp's edges [E0, E1): equal shares, rounded up to whole 32-edge rows of loads
  const int64_t per = (((nnz + warps - 1) / warps) + 31) & ~int64_t(31);
  const int64_t E0 = gw * per;
  if (E0 >= nnz) return;  // warp-uniform
  const int64_t E1 = (E0 + per < nnz) ? E0 + per : nnz;
  // row holding edge E0: last r with rowptr[r] <= E0. 33-ary search, one probe per
  // lane per round: about 4 dependent loads for 10^5..10^6 rows instead of the
  // 17-20 of a binary search (invariant rowptr[lo] <= E0 < rowptr[hi])
  int64_t lo = 0, hi = n_rows;
  while (hi - lo > 1) {
    const int64_t p = lo + (static_cast<int64_t>(lane + 1) * (hi - lo)) / 33;
    const bool le = p <= lo ? true : (p >= hi ? false : rowptr[p] <= E0);
    const unsigned m = __ballot_sync(0xffffffffu, le);
    const int k = __popc(m);  // probes are nondecreasing in the lane, so `le` holds for lanes [0, k)
    const int64_t plo = __shfl_sync(0xffffffffu, p, k > 0 ? k - 1 : 0);
    const int64_t phi = __shfl_sync(0xffffffffu, p, k < 32 ? k : 31);
    if (k > 0 && plo > lo) lo = plo;
    if (k < 32 && phi < hi) hi = phi;
  }
  for (int fbase = 0; fbase < F; fbase += 32 * VEC) {
    const int f0 = fbase + lane * VEC;
    // every lane takes part in the control flow; with VEC >= 2 the dispatch
    // guarantees F % (32 * VEC) == 0, so every lane has features in every pass
    const bool active = VEC >= 2 || f0 < F;
    int64_t row = lo;
    int64_t rs = rowptr[row];
    // lane l holds the end of row `wrow + l`
    int64_t wrow = row;
    int64_t rend = (wrow + lane < n_rows) ? rowptr[wrow + lane + 1] : INT64_MAX;
    int64_t re = __shfl_sync(0xffffffffu, rend, 0);
    float acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
    bool have = false;
    for (int64_t sb = E0; sb < E1; sb += kSpmmChunk) {
      const int n = static_cast<int>((E1 - sb) < kSpmmChunk ? (E1 - sb) : kSpmmChunk);
      // stage the sub-chunk: all loads of a lane in flight together
      int cv[kPer];
      float vv[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int k = lane + 32 * i;
        cv[i] = k < n ? col[sb + k] : 0;
        vv[i] = k < n ? val[sb + k] : 0.f;
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        scol[lane + 32 * i] = cv[i];
        sval[lane + 32 * i] = vv[i];
      }
      __syncwarp();
      for (int e0 = 0; e0 < n; e0 += kUnroll) {
        float t[kUnroll][VEC];
        if (e0 + kUnroll <= n) {
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            if (active) load_vec<VEC>(rows.row(scol[e0 + u]) + f0, t[u]);
          }
        } else {
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            if (active && e0 + u < n) load_vec<VEC>(rows.row(scol[e0 + u]) + f0, t[u]);
          }
        }
        const int cnt = (n - e0) < kUnroll ? (n - e0) : kUnroll;
        const int64_t s0 = sb + e0;  // first edge of the batch
        // the current row must hold edge s0 (after a slow-path batch it may end just before)
        while (s0 >= re) {
          if (have && active) {
            const bool whole = rs >= E0 && re <= E1;
            out.template put_vec<VEC>(row, f0, acc, whole);
          }
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
          have = false;
          rs = re;
          ++row;
          if (row - wrow == 32) {
            wrow = row;
            rend = (wrow + lane < n_rows) ? rowptr[wrow + lane + 1] : INT64_MAX;
          }
          re = __shfl_sync(0xffffffffu, rend, static_cast<int>(row - wrow));
        }
        // Fast path: the 32-row window holds every row that ends inside the batch
        // and the row of the edge after it. The positions where rows end come
        // as one bit mask, so an edge costs its FMAs and a bit test.
        if (__shfl_sync(0xffffffffu, rend, 31) <= s0 + cnt && wrow != row) {
          wrow = row;
          rend = (wrow + lane < n_rows) ? rowptr[wrow + lane + 1] : INT64_MAX;
        }
        if (__shfl_sync(0xffffffffu, rend, 31) > s0 + cnt) {
          const int64_t pe = rend - 1 - s0;  // this lane's row ends at batch edge pe
          unsigned ends = (pe >= 0 && pe < cnt) ? (1u << static_cast<int>(pe)) : 0u;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ends |= __shfl_xor_sync(0xffffffffu, ends, o);
          if (ends == 0u && cnt == kUnroll) {  // the whole batch continues row `row`
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
              const float w = sval[e0 + u];
#pragma unroll
              for (int v = 0; v < VEC; ++v) acc[v] = fmaf(w, t[u][v], acc[v]);
            }
            have = true;
            continue;
          }
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            if (u >= cnt) continue;
            const float w = sval[e0 + u];
#pragma unroll
            for (int v = 0; v < VEC; ++v) acc[v] = fmaf(w, t[u][v], acc[v]);
            have = true;
            if ((ends >> u) & 1u) {  // row `row` ends at this edge (warp-uniform)
              if (active) {
                const bool whole = rs >= E0;  // its end s0 + u + 1 is inside the range
                out.template put_vec<VEC>(row, f0, acc, whole);
              }
#pragma unroll
              for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
              have = false;
              // next: the row holding edge s0 + u + 1 (empty rows in between end at s0 + u + 1)
              const int l = __ffs(__ballot_sync(0xffffffffu, rend > s0 + u + 1)) - 1;
              row = wrow + l;
              rs = s0 + u + 1;
              re = __shfl_sync(0xffffffffu, rend, l);
            }
          }
          continue;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          if (e0 + u >= n) continue;  // (no break: the loop must unroll to keep t[] in registers)
          const int64_t e = sb + e0 + u;
          while (e >= re) {  // the stream left row `row` (warp-uniform)
            if (have && active) {
              const bool whole = rs >= E0 && re <= E1;
              out.template put_vec<VEC>(row, f0, acc, whole);
            }
#pragma unroll
            for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
            have = false;
            rs = re;
            ++row;
            if (row - wrow == 32) {
              wrow = row;
              rend = (wrow + lane < n_rows) ? rowptr[wrow + lane + 1] : INT64_MAX;
            }
            re = __shfl_sync(0xffffffffu, rend, static_cast<int>(row - wrow));
          }
          const float w = sval[e0 + u];
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[v] = fmaf(w, t[u][v], acc[v]);
          have = true;
        }
      }
    }
    if (have && active) {
      const bool whole = rs >= E0 && re <= E1;
      out.template put_vec<VEC>(row, f0, acc, whole);
    }
  }
}

// Item-based SpMM for F = 64 (the MPNN-LSTM width). The host plan cuts every
// row into items of at most kSpmmItemEdges edges (rows with no edges get one
// empty item, which stores the zero row) and gives each warp of a fixed grid a
// contiguous run of items of about equal edge count. A warp works on one item
// at a time, two edges per step: lanes 0-15 take the even edges, lanes 16-31 the
// odd ones, each lane one float4 of the 64 features, four edges in flight per
// half; the halves are summed by one shuffle and lanes 0-15 store the row.
// Items of rows split over several items add atomically into rows that a small
// kernel zeroed first. Against the edge-stream kernel above this halves the
// instructions per edge (a float4 per lane and no per-edge row-end test).
constexpr int kSpmmItemWarpsPerSm = 64;  // 8 blocks of 256 threads per SM

template <class Out>
struct zero_empty : std::true_type {};
template <>
struct zero_empty<PeerPush> : std::false_type {};  // nothing to push for a row without edges

template <class Rows, class Out>
__global__ void __launch_bounds__(256) spmm_items64_kernel(const int* __restrict__ items, int n_items,
                                                           const int* __restrict__ warp_off, int warps,
                                                           const int* __restrict__ col,
                                                           const float* __restrict__ val, const Rows rows,
                                                           const Out out) {
  const int lane = threadIdx.x & 31, half = lane >> 4, l16 = lane & 15;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (gw >= warps) return;  // warp-uniform
  const int i0 = warp_off[gw], i1 = warp_off[gw + 1];
  for (int it = i0; it < i1; ++it) {
    const int renc = items[it], e0 = items[n_items + it], e1 = items[2 * n_items + it];
    const bool whole = renc >= 0;
    const int r = whole ? renc : -renc - 1;
    if (e0 == e1 && !zero_empty<Out>::value) continue;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    int e = e0 + half;
    for (; e + 6 < e1; e += 8) {  // edges e, e + 2, e + 4, e + 6 of this half
      int c[4];
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        c[u] = col[e + 2 * u];
        v[u] = val[e + 2 * u];
      }
      float t[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u) load_vec<4>(rows.row(c[u]) + 4 * l16, t[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int j = 0; j < 4; ++j) a[j] = fmaf(v[u], t[u][j], a[j]);
    }
    for (; e < e1; e += 2) {
      float t[4];
      load_vec<4>(rows.row(col[e]) + 4 * l16, t);
      const float v = val[e];
#pragma unroll
      for (int j = 0; j < 4; ++j) a[j] = fmaf(v, t[j], a[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) a[j] += __shfl_xor_sync(0xffffffffu, a[j], 16);
    if (half == 0) out.template put_vec<4>(r, 4 * l16, a, whole);
  }
}

__global__ void zero_rows64_kernel(const int* __restrict__ rows_list, int n, float* __restrict__ out, int ld) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(n) * 16) return;
  const int r = rows_list[i >> 4];
  reinterpret_cast<float4*>(out + static_cast<int64_t>(r) * ld)[i & 15] = make_float4(0.f, 0.f, 0.f, 0.f);
}

template <class Rows, class Out>
static void launch_items(cudaStream_t st, const SpmmPlan& plan, const int* col, const float* val, const Rows& rows,
                         const Out& out) {
  if (plan.n_items == 0) return;
  count_launch();
  spmm_items64_kernel<<<(plan.warps + 7) / 8, 256, 0, st>>>(plan.items, plan.n_items, plan.warp_off, plan.warps, col,
                                                            val, rows, out);
}

// the plan applies: 64 features, a plain (non-accumulating) output
static bool plan_ok(const SpmmPlan* plan, int F) { return plan != nullptr && plan->items != nullptr && F == 64; }

int spmm_plan_warps(int device) { return num_sms(device) * kSpmmItemWarpsPerSm; }

template <class Rows, class Out>
static void launch_chunked(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val, const Rows& rows,
                           int64_t n_rows, int F, const Out& out) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int threads = 256;
  const int blocks = num_sms(dev) * 3;  // persistent: three 256-thread blocks per SM (80 registers a thread)
  count_launch();
  if (F % 128 == 0) spmm_chunked_kernel<4><<<blocks, threads, 0, st>>>(rowptr, col, val, rows, n_rows, F, out);
  else if (F % 64 == 0) spmm_chunked_kernel<2><<<blocks, threads, 0, st>>>(rowptr, col, val, rows, n_rows, F, out);
  else spmm_chunked_kernel<1><<<blocks, threads, 0, st>>>(rowptr, col, val, rows, n_rows, F, out);
}

void launch_spmm_csr(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val, const float* x,
                     int64_t n_rows, int F, float* out, int accumulate, const SpmmPlan* plan) {
  if (n_rows == 0) return;
  if (!accumulate && plan_ok(plan, F)) {
    if (plan->n_split > 0) {
      count_launch();
      zero_rows64_kernel<<<(plan->n_split * 16 + 255) / 256, 256, 0, st>>>(plan->split_rows, plan->n_split, out, F);
    }
    launch_items(st, *plan, col, val, LocalRows{x, F}, LocalOut{out, F, 0});
    return;
  }
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

// Halo rows pulled over NVLink once each: out[i] = row lrow[c] of owner[c]'s
// staging buffer for c = halo_src[i]. Sixteen-byte vectors, F / 4 lanes per row.
// Peers' staging rows have a stride of LD4 float4s (the staging width); the
// pulled rows are F4 float4s wide (the layer width, at most the staging width).
__global__ void halo_pull_kernel(const float* const* __restrict__ peers, const int* __restrict__ owner,
                                 const int* __restrict__ lrow, const int* __restrict__ halo_src, int64_t n_halo,
                                 int F4, int LD4, float4* __restrict__ out) {
  const int64_t total = n_halo * F4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t h = i / F4;
    const int v = static_cast<int>(i - h * F4);
    const int c = halo_src[h];
    const float4* src = reinterpret_cast<const float4*>(peers[owner[c]] + static_cast<int64_t>(lrow[c]) * LD4 * 4);
    out[i] = src[v];
  }
}

void launch_halo_pull(cudaStream_t st, const float* const* peers, const int* owner, const int* lrow,
                      const int* halo_src, int64_t n_halo, int F, int ld, float* out) {
  if (n_halo == 0) return;
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t total = n_halo * (F / 4);
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(num_sms(dev)) * 8));
  count_launch();
  halo_pull_kernel<<<blocks, 256, 0, st>>>(peers, owner, lrow, halo_src, n_halo, F / 4, ld / 4,
                                           reinterpret_cast<float4*>(out));
}

// Aggregation over [this rank's rows | pulled halo rows] (columns remapped once
// per graph: local sources -> their row in x, halo sources -> n_split + pull slot).
void launch_spmm_two_tables(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val, const float* x,
                            int x_ld, const float* halo, int n_split, int64_t n_rows, int F, float* out,
                            const SpmmPlan* plan) {
  if (n_rows == 0) return;
  if (plan_ok(plan, F)) {
    if (plan->n_split > 0) {
      count_launch();
      zero_rows64_kernel<<<(plan->n_split * 16 + 255) / 256, 256, 0, st>>>(plan->split_rows, plan->n_split, out, F);
    }
    launch_items(st, *plan, col, val, TwoTables{x, halo, n_split, F, x_ld}, LocalOut{out, F, 0});
    return;
  }
  cudaMemsetAsync(out, 0, static_cast<size_t>(n_rows) * F * sizeof(float), st);
  launch_chunked(st, rowptr, col, val, TwoTables{x, halo, n_split, F, x_ld}, n_rows, F, LocalOut{out, F, 0});
}

// Its backward over the transposed CSR (rows = source rows): each source row's
// gradient is pushed into the owner's gradient buffer with remote atomic adds.
void launch_spmm_peer_push(cudaStream_t st, const int64_t* rowptr_t, const int* col_t, const float* val_t,
                           const float* grad_dst, int64_t n_src, int F, int ld, float* const* peers,
                           const int* src_owner, const int* src_row, const SpmmPlan* plan) {
  if (n_src == 0) return;
  if (plan_ok(plan, F)) {  // pushes are atomic adds into the owners' zeroed buffers
    launch_items(st, *plan, col_t, val_t, LocalRows{grad_dst, F}, PeerPush{peers, src_owner, src_row, ld});
    return;
  }
  launch_chunked(st, rowptr_t, col_t, val_t, LocalRows{grad_dst, F}, n_src, F,
                 PeerPush{peers, src_owner, src_row, ld});
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
  const float* g = gates + lstm_gate_index(r, H, 0, c);  // i, f, g, o 16 floats apart
  const float i = g[0], f = g[16], gg = g[32], o = g[48];
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

// Four consecutive units of one row per thread (H, dh_ld, dc_ld multiples of 4,
// 16-byte aligned rows); the pre-activation gradients go out in bf16, the type in
// which the following GEMMs consume them (the rounding is the one their operand
// packing would apply to fp32 values).
__global__ void lstm_bwd4_kernel(const float* __restrict__ gates, const float* __restrict__ c_prev,
                                 const float* __restrict__ c_new, const float* __restrict__ dh, int dh_ld,
                                 const float* __restrict__ dc, int dc_ld, int64_t rows, int H,
                                 __nv_bfloat16* __restrict__ dpre, float* __restrict__ dc_prev) {
  const int H4 = H >> 2;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * H4) return;
  const int64_t r = idx / H4;
  const int c = static_cast<int>(idx % H4) * 4;
  const float* g = gates + lstm_gate_index(r, H, 0, c);
  const float4 i4 = ldg4(g), f4 = ldg4(g + 16), g4 = ldg4(g + 32), o4 = ldg4(g + 48);
  const float4 cn4 = ldg4(c_new + r * H + c);
  const float4 cp4 = c_prev ? ldg4(c_prev + r * H + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 dh4 = dh ? ldg4(dh + r * dh_ld + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 dc4 = dc ? ldg4(dc + r * dc_ld + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float iv[4] = {i4.x, i4.y, i4.z, i4.w}, fv[4] = {f4.x, f4.y, f4.z, f4.w};
  const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, ov[4] = {o4.x, o4.y, o4.z, o4.w};
  const float cn[4] = {cn4.x, cn4.y, cn4.z, cn4.w}, cp[4] = {cp4.x, cp4.y, cp4.z, cp4.w};
  const float dhv[4] = {dh4.x, dh4.y, dh4.z, dh4.w}, dcv[4] = {dc4.x, dc4.y, dc4.z, dc4.w};
  float di[4], df[4], dg[4], dout[4], dcp[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const float tc = tanhf(cn[u]);
    const float dct = dcv[u] + dhv[u] * ov[u] * (1.f - tc * tc);
    di[u] = dct * gv[u] * iv[u] * (1.f - iv[u]);
    df[u] = dct * cp[u] * fv[u] * (1.f - fv[u]);
    dg[u] = dct * iv[u] * (1.f - gv[u] * gv[u]);
    dout[u] = dhv[u] * tc * ov[u] * (1.f - ov[u]);
    dcp[u] = dct * fv[u];
  }
  auto put = [](__nv_bfloat16* p, const float (&v)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = w;
  };
  __nv_bfloat16* d = dpre + r * 4 * H + c;
  put(d, di);
  put(d + H, df);
  put(d + 2 * H, dg);
  put(d + 3 * H, dout);
  if (dc_prev) *reinterpret_cast<float4*>(dc_prev + r * H + c) = make_float4(dcp[0], dcp[1], dcp[2], dcp[3]);
}

// The same gate gradients written straight into the two packed bf16 images the
// following GEMMs read (no row-major copy, no packing pass): the K-major image
// of dpre [rows, 4H] for d[x || h] = dpre W, and the MN-major image of dpre^T
// for dW = dpre^T [x || h] (K = rows). Layout of both: block(tile, chunk) of
// 128 x 64 bf16 = 16 KB, then 8-row group * 1024 + 8-column group * 128 + row * 16.
// A thread takes 8 units of one row (one 16-byte vector per gate and image);
// rows past `rows` write zeros (tile padding of the K-major image, the K
// padding of the MN-major one, which the weight-gradient GEMM sums over).
// Requires H % 32 == 0 (whole 64-wide chunks of 4H and whole 128-row MN tiles).
__global__ void lstm_bwd_pack_kernel(const float* __restrict__ gates, const float* __restrict__ c_prev,
                                     const float* __restrict__ c_new, const float* __restrict__ dh, int dh_ld,
                                     const float* __restrict__ dc, int dc_ld, int64_t rows, int H,
                                     uint8_t* __restrict__ img_k, uint8_t* __restrict__ img_mn,
                                     float* __restrict__ dc_prev, int64_t rows_k, int64_t rows_mn) {
  const int H8 = H >> 3;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t r = idx / H8;
  if (r >= rows_k) return;
  const int u0 = static_cast<int>(idx - r * H8) * 8;
  float d[4][8];
  if (r < rows) {
    const float* g = gates + lstm_gate_index(r, H, 0, u0);  // i, f, g, o 16 floats apart
    const float zero[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float iv[8], fv[8], gv[8], ov[8], cn[8], cp[8], dhv[8], dcv[8];
    auto ld8 = [](const float* p, float (&v)[8]) {
      const float4 a = ldg4(p), b = ldg4(p + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    };
    ld8(g, iv);
    ld8(g + 16, fv);
    ld8(g + 32, gv);
    ld8(g + 48, ov);
    ld8(c_new + r * H + u0, cn);
    if (c_prev) ld8(c_prev + r * H + u0, cp);
    else for (int u = 0; u < 8; ++u) cp[u] = zero[u];
    if (dh) ld8(dh + r * dh_ld + u0, dhv);
    else for (int u = 0; u < 8; ++u) dhv[u] = zero[u];
    if (dc) ld8(dc + r * dc_ld + u0, dcv);
    else for (int u = 0; u < 8; ++u) dcv[u] = zero[u];
    float dcp[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float tc = tanhf(cn[u]);
      const float dct = dcv[u] + dhv[u] * ov[u] * (1.f - tc * tc);
      d[0][u] = dct * gv[u] * iv[u] * (1.f - iv[u]);
      d[1][u] = dct * cp[u] * fv[u] * (1.f - fv[u]);
      d[2][u] = dct * iv[u] * (1.f - gv[u] * gv[u]);
      d[3][u] = dhv[u] * tc * ov[u] * (1.f - ov[u]);
      dcp[u] = dct * fv[u];
    }
    if (dc_prev) {
      float4* o = reinterpret_cast<float4*>(dc_prev + r * H + u0);
      o[0] = make_float4(dcp[0], dcp[1], dcp[2], dcp[3]);
      o[1] = make_float4(dcp[4], dcp[5], dcp[6], dcp[7]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int u = 0; u < 8; ++u) d[q][u] = 0.f;
  }
  const int64_t nch_k = (4 * H) >> 6;
  const int64_t nch_mn = rows_mn >> 6;
  const int r8 = static_cast<int>(r & 7);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 v = pack_bf16x8(d[q]);
    const int k = q * H + u0;  // column of dpre = MN index of dpre^T
    const int64_t off_k = ((r >> 7) * nch_k + (k >> 6)) * 16384 + ((r & 127) >> 3) * 1024 + ((k & 63) >> 3) * 128 + r8 * 16;
    *reinterpret_cast<uint4*>(img_k + off_k) = v;
    if (r < rows_mn) {
      const int64_t off_m = (static_cast<int64_t>(k >> 7) * nch_mn + (r >> 6)) * 16384 + ((k & 127) >> 3) * 1024 +
                            ((r & 63) >> 3) * 128 + r8 * 16;
      *reinterpret_cast<uint4*>(img_mn + off_m) = v;
    }
  }
}

void launch_lstm_bwd_pack(cudaStream_t st, const float* gates, const float* c_prev, const float* c_new,
                          const float* dh, int dh_ld, const float* dc, int dc_ld, int64_t rows, int H, uint8_t* img_k,
                          uint8_t* img_mn, float* dc_prev) {
  const int64_t rows_k = (rows + 127) / 128 * 128;
  const int64_t rows_mn = (rows + 63) / 64 * 64;
  const int64_t n = rows_k * (H / 8);
  if (n == 0) return;
  count_launch();
  lstm_bwd_pack_kernel<<<(n + 255) / 256, 256, 0, st>>>(gates, c_prev, c_new, dh, dh_ld, dc, dc_ld, rows, H, img_k,
                                                        img_mn, dc_prev, rows_k, rows_mn);
}

void launch_lstm_bwd(cudaStream_t st, const float* gates, const float* c_prev, const float* c_new, const float* dh,
                     int dh_ld, const float* dc, int dc_ld, int64_t rows, int H, float* dpre, float* dc_prev) {
  const int64_t n = rows * H;
  if (n == 0) return;
  count_launch();
  lstm_bwd_kernel<<<(n + 255) / 256, 256, 0, st>>>(gates, c_prev, c_new, dh, dh_ld, dc, dc_ld, rows, H, dpre,
                                                   dc_prev);
}

bool lstm_bwd_bf16_ok(const float* gates, const float* c_prev, const float* c_new, const float* dh, int dh_ld,
                      const float* dc, int dc_ld, int H, const void* dpre, const float* dc_prev) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return H % 4 == 0 && dh_ld % 4 == 0 && dc_ld % 4 == 0 && al(gates) && al(c_prev) && al(c_new) && al(dh) &&
         al(dc) && al(dc_prev) && (reinterpret_cast<uintptr_t>(dpre) & 7) == 0;
}

void launch_lstm_bwd_bf16(cudaStream_t st, const float* gates, const float* c_prev, const float* c_new,
                          const float* dh, int dh_ld, const float* dc, int dc_ld, int64_t rows, int H,
                          __nv_bfloat16* dpre, float* dc_prev) {
  const int64_t n = rows * (H / 4);
  if (n == 0) return;
  count_launch();
  lstm_bwd4_kernel<<<(n + 255) / 256, 256, 0, st>>>(gates, c_prev, c_new, dh, dh_ld, dc, dc_ld, rows, H, dpre,
                                                    dc_prev);
}

// ---------------------------------------------------------------------------
// Reset-gated GRU cell backward (the elementwise parts; the GEMMs run on the
// tcgen05 kernel). Forward: z, r = sigmoid(...), c = tanh(W_c [x_c | r h] + b_c),
// h' = z h + (1 - z) c.
// ---------------------------------------------------------------------------
// dz_pre = dh' (h - c) z (1 - z) -> dzr[:, 0:H];  dc_pre = dh' (1 - z) (1 - c^2);  dh_acc = dh' z
__global__ void rgru_bwd1_kernel(const float* __restrict__ dhn, int dhn_ld, const float* __restrict__ h, int h_ld,
                                 const float* __restrict__ z, const float* __restrict__ c, int64_t rows, int H,
                                 float* __restrict__ dzr, float* __restrict__ dc_pre, float* __restrict__ dh_acc) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * H) return;
  const int64_t r = i / H;
  const int u = static_cast<int>(i - r * H);
  const float g = dhn[r * dhn_ld + u];
  const float hv = h ? h[r * h_ld + u] : 0.f;
  const float zv = z[i], cv = c[i];
  dzr[r * 2 * H + u] = g * (hv - cv) * zv * (1.f - zv);
  dc_pre[i] = g * (1.f - zv) * (1.f - cv * cv);
  if (dh_acc) dh_acc[i] = g * zv;
}

// dr_pre = drh h r (1 - r) -> dzr[:, H:2H];  dh_acc += drh r
__global__ void rgru_bwd2_kernel(const float* __restrict__ drh, int drh_ld, const float* __restrict__ h, int h_ld,
                                 const float* __restrict__ rg, int64_t rows, int H, float* __restrict__ dzr,
                                 float* __restrict__ dh_acc) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * H) return;
  const int64_t r = i / H;
  const int u = static_cast<int>(i - r * H);
  const float d = drh[r * drh_ld + u];
  const float rv = rg[i];
  const float hv = h ? h[r * h_ld + u] : 0.f;
  dzr[r * 2 * H + H + u] = d * hv * rv * (1.f - rv);
  if (dh_acc) dh_acc[i] += d * rv;
}

// out = a + b (b row-strided): the direct and the GEMM parts of dh
__global__ void add_rows_kernel(const float* __restrict__ a, const float* __restrict__ b, int b_ld, int64_t rows, int H,
                                float* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * H) return;
  const int64_t r = i / H;
  out[i] = a[i] + b[r * b_ld + (i - r * H)];
}

void launch_rgru_bwd1(cudaStream_t st, const float* dhn, int dhn_ld, const float* h, int h_ld, const float* z,
                      const float* c, int64_t rows, int H, float* dzr, float* dc_pre, float* dh_acc) {
  const int64_t n = rows * H;
  if (n == 0) return;
  count_launch();
  rgru_bwd1_kernel<<<(n + 255) / 256, 256, 0, st>>>(dhn, dhn_ld, h, h_ld, z, c, rows, H, dzr, dc_pre, dh_acc);
}
void launch_rgru_bwd2(cudaStream_t st, const float* drh, int drh_ld, const float* h, int h_ld, const float* r,
                      int64_t rows, int H, float* dzr, float* dh_acc) {
  const int64_t n = rows * H;
  if (n == 0) return;
  count_launch();
  rgru_bwd2_kernel<<<(n + 255) / 256, 256, 0, st>>>(drh, drh_ld, h, h_ld, r, rows, H, dzr, dh_acc);
}
void launch_add_rows(cudaStream_t st, const float* a, const float* b, int b_ld, int64_t rows, int H, float* out) {
  const int64_t n = rows * H;
  if (n == 0) return;
  count_launch();
  add_rows_kernel<<<(n + 255) / 256, 256, 0, st>>>(a, b, b_ld, rows, H, out);
}

}  // namespace su
