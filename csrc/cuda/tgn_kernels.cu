// TGN / CTDG training-step kernels for sm_100a.
//
// The step follows the reference online runtime (backends/ctdg/runtime/runtime.py:225-328):
//   prep      : unique roots of src ∪ dst, root index of every event, uniform
//               negatives from the destination pool (+1 shift on collision), the
//               per-root mailbox winners of the src and dst passes and ts_max.
//   sample    : most-recent / uniform-before-t neighbours from a T-CSR keyed by
//               destination (vendor/bts_sampler/sampler/include/sampler.h:213-261).
//   gru       : GRU over the K mailbox slots, then GRUCell(agg, mem) with the
//               result scattered straight into the memory table (fused epilogue).
//   mailbox   : [mem_prev(self) || mem_prev(other) || edge_feat] written at the
//               circular slot position (backends/ctdg/runtime/memory.py:183-248).
//   attention : per-root softmax over the sampled neighbours, dropout, weighted
//               sum of V (backends/ctdg/runtime/models.py:77-137), fwd and bwd.
//   out/LN    : W_out [agg || h] -> dropout -> ReLU -> LayerNorm, fused epilogue.
//   link/BCE  : src_fc/dst_fc/out_fc scoring and the two BCE terms with their
//               gradients (models.py:313-324, runtime.py:290-292), plus AP/AUC.
#include "kernels.h"

namespace su {

// ---------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t orderable_f32(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}



__global__ void __launch_bounds__(1024) tgn_prep_kernel(PrepArgs a) {
  __shared__ int s_R;
  __shared__ float s_tsmax;
  __shared__ int s_tag;
  const int n = min(*a.n_ev, a.bmax);
  if (threadIdx.x == 0) {
    s_R = 0;
    s_tsmax = -INFINITY;
    s_tag = static_cast<int>((*a.step_ctr) & 0x3FFFFFFF) + 1;
  }
  for (int r = threadIdx.x; r < 2 * a.rmax; r += blockDim.x) {
    a.win_key[r] = 0ull;
    a.cnt[r] = 0;
  }
  __syncthreads();
  const int tag = s_tag;
  // phase 1: claim unique roots
  float local_max = -INFINITY;
  for (int j = threadIdx.x; j < 2 * n; j += blockDim.x) {
    const int64_t v = j < n ? a.src[j] : a.dst[j - n];
    if (j < n) local_max = fmaxf(local_max, a.ts[j]);
    int cur = a.stamp[v];
    bool claimed = false;
    while (cur != tag) {
      const int prev = atomicCAS(&a.stamp[v], cur, tag);
      if (prev == cur) {
        claimed = true;
        break;
      }
      cur = prev;
    }
    if (claimed) {
      const int r = atomicAdd(&s_R, 1);
      if (r < a.rmax) {
        a.node2root[v] = r;
        a.roots[r] = v;
      } else {
        record_status(a.status, kTooLarge);
      }
    }
  }
  local_max = warp_max(local_max);
  __shared__ float s_wmax[32];
  if ((threadIdx.x & 31) == 0) s_wmax[threadIdx.x >> 5] = local_max;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int w = 0; w < (blockDim.x >> 5); ++w) m = fmaxf(m, s_wmax[w]);
    s_tsmax = n > 0 ? m : 0.f;
  }
  __syncthreads();
  const int R = min(s_R, a.rmax);
  // phase 2: event -> root indices, negatives, mailbox winners
  for (int i = threadIdx.x; i < a.bmax; i += blockDim.x) {
    if (i < n) {
      const int si = a.node2root[a.src[i]];
      const int di = a.node2root[a.dst[i]];
      a.src_idx[i] = si;
      a.dst_idx[i] = di;
      // negative: pool[randint(P)], shifted by one on collision with the true dst
      const uint4 rr = Philox::gen(a.seed, static_cast<uint64_t>(*a.step_ctr) * (uint64_t)a.bmax + i, 0x4E4547u);
      int64_t idx = static_cast<int64_t>(((static_cast<uint64_t>(rr.x) << 32) | rr.y) % (uint64_t)a.pool_size);
      int64_t ng = a.neg_pool[idx];
      if (ng == a.dst[i]) {
        idx = (idx + 1) % a.pool_size;
        ng = a.neg_pool[idx];
      }
      a.neg[i] = ng;
      a.neg_idx[i] = (a.stamp[ng] == tag) ? a.node2root[ng] : -1;
      const unsigned long long key =
          (static_cast<unsigned long long>(orderable_f32(a.ts[i])) << 32) | static_cast<unsigned int>(i);
      atomicMax(&a.win_key[si], key);
      atomicAdd(&a.cnt[si], 1);
      atomicMax(&a.win_key[a.rmax + di], key);
      atomicAdd(&a.cnt[a.rmax + di], 1);
    } else {
      a.src_idx[i] = -1;
      a.dst_idx[i] = -1;
      a.neg[i] = -1;
      a.neg_idx[i] = -1;
    }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < a.rmax; r += blockDim.x) {
    if (r >= R) a.roots[r] = -1;
    for (int p = 0; p < 2; ++p) {
      const unsigned long long k = a.win_key[p * a.rmax + r];
      a.win[p * a.rmax + r] = (r < R && a.cnt[p * a.rmax + r] > 0) ? static_cast<int>(k & 0xFFFFFFFFull) : -1;
    }
  }
  if (threadIdx.x == 0) {
    *a.n_roots = R;
    *a.ts_max = s_tsmax;
    *a.root_ts = static_cast<int64_t>(s_tsmax);
    *a.step_ctr += 1;
  }
}

// ---------------------------------------------------------------------------
// temporal neighbour sampling (warp per root)
// ---------------------------------------------------------------------------
__global__ void tgn_sample_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                  const int64_t* __restrict__ root_ts_scalar, const int64_t* __restrict__ root_ts_vec,
                                  const int64_t* __restrict__ rowptr, const int64_t* __restrict__ nbr,
                                  const int64_t* __restrict__ eid, const int64_t* __restrict__ ets, int k, int policy,
                                  uint64_t seed, const int64_t* __restrict__ step_ctr, int64_t* __restrict__ out_nbr,
                                  int64_t* __restrict__ out_eid, float* __restrict__ out_dt,
                                  int* __restrict__ out_cnt, int* __restrict__ edge_total) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rmax) return;
  const int R = *n_roots;
  const int r = warp;
  if (r >= R) {
    if (lane == 0) out_cnt[r] = 0;
    for (int j = lane; j < k; j += 32) {
      out_nbr[(int64_t)r * k + j] = -1;
      out_eid[(int64_t)r * k + j] = -1;
      out_dt[(int64_t)r * k + j] = 0.f;
    }
    return;
  }
  const int64_t v = roots[r];
  const int64_t rts = root_ts_vec ? root_ts_vec[r] : *root_ts_scalar;
  const int64_t lo = rowptr[v], hi = rowptr[v + 1];
  // lower_bound(ts[lo:hi], rts): first position with ts >= rts (strictly-earlier neighbours)
  int64_t a = lo, b = hi;
  while (a < b) {
    const int64_t m = (a + b) >> 1;
    if (ets[m] < rts) a = m + 1;
    else b = m;
  }
  const int64_t end = a;
  const int64_t avail = end - lo;
  int cnt;
  if (policy == 0 || avail <= k) {
    // recent: the last min(k, avail) entries in list (time) order
    cnt = static_cast<int>(avail < (int64_t)k ? avail : (int64_t)k);
    const int64_t start = end - cnt;
    for (int j = lane; j < k; j += 32) {
      const int64_t o = (int64_t)r * k + j;
      if (j < cnt) {
        const int64_t p = start + j;
        out_nbr[o] = nbr[p];
        out_eid[o] = eid[p];
        out_dt[o] = static_cast<float>(rts - ets[p]);
      } else {
        out_nbr[o] = -1;
        out_eid[o] = -1;
        out_dt[o] = 0.f;
      }
    }
  } else {
    // uniform with replacement over the avail strictly-earlier neighbours
    cnt = k;
    for (int j = lane; j < k; j += 32) {
      const uint4 rr = Philox::gen(seed, (static_cast<uint64_t>(*step_ctr) << 32) ^ ((uint64_t)r * k + j), 0x534D50u);
      const int64_t p = lo + static_cast<int64_t>(rr.x % static_cast<uint64_t>(avail));
      const int64_t o = (int64_t)r * k + j;
      out_nbr[o] = nbr[p];
      out_eid[o] = eid[p];
      out_dt[o] = static_cast<float>(rts - ets[p]);
    }
  }
  if (lane == 0) {
    out_cnt[r] = cnt;
    if (cnt > 0) atomicAdd(edge_total, cnt);
  }
}


// ---------------------------------------------------------------------------
// mailbox write (block of 128 threads per root, two passes in order src, dst)
// ---------------------------------------------------------------------------
__global__ void tgn_mailbox_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                   const int* __restrict__ win, const int* __restrict__ cnt,
                                   const int* __restrict__ src_idx, const int* __restrict__ dst_idx,
                                   const int64_t* __restrict__ ev_eid, const float* __restrict__ ev_ts,
                                   const float* __restrict__ mem_prev, int D, const void* __restrict__ efeat,
                                   int efeat_bf16, int efeat_ld, int e_raw, int E, float* __restrict__ mailbox,
                                   float* __restrict__ mailbox_ts, int64_t* __restrict__ next_pos, int K) {
  const int r = blockIdx.x;
  if (r >= *n_roots || r >= rmax) return;
  const int64_t v = roots[r];
  const int SW = 2 * D + E;
  const int64_t pos0 = next_pos[v];
  const int csrc = cnt[r], cdst = cnt[rmax + r];
  for (int p = 0; p < 2; ++p) {
    const int i = win[p * rmax + r];
    if (i < 0) continue;
    const int64_t pos = (p == 0 ? pos0 : (pos0 + csrc)) % K;
    const int self = p == 0 ? src_idx[i] : dst_idx[i];
    const int other = p == 0 ? dst_idx[i] : src_idx[i];
    float* slot = mailbox + (v * K + pos) * SW;
    const int64_t e = ev_eid[i];
    for (int c = threadIdx.x; c < SW; c += blockDim.x) {
      float x;
      if (c < D) x = mem_prev[(int64_t)self * D + c];
      else if (c < 2 * D) x = mem_prev[(int64_t)other * D + (c - D)];
      else {
        const int ce = c - 2 * D;
        x = 0.f;
        if (ce < e_raw)
          x = efeat_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(efeat)[e * efeat_ld + ce])
                         : static_cast<const float*>(efeat)[e * efeat_ld + ce];
      }
      slot[c] = x;
    }
    if (threadIdx.x == 0) mailbox_ts[v * K + pos] = ev_ts[i];
    __syncthreads();
  }
  if (threadIdx.x == 0) next_pos[v] = (pos0 + csrc + cdst) % K;
}

// ---------------------------------------------------------------------------
// temporal attention forward (warp per root; edges of a root on lanes)
// KV: [rmax*k, 2*Do] (K cols [0,Do), V cols [Do,2Do)); Q: [rmax, Do]
// ---------------------------------------------------------------------------

// Value of head h's per-edge quantity held by lane j. __shfl_sync evaluates its
// operand on the SOURCE lane, so every head is shuffled and the destination
// lane picks its own head afterwards.
__device__ __forceinline__ float shfl_head(const float (&v)[4], int H, int h, int j) {
  const float v0 = __shfl_sync(0xffffffffu, v[0], j);
  const float v1 = H > 1 ? __shfl_sync(0xffffffffu, v[1], j) : 0.f;
  const float v2 = H > 2 ? __shfl_sync(0xffffffffu, v[2], j) : 0.f;
  const float v3 = H > 3 ? __shfl_sync(0xffffffffu, v[3], j) : 0.f;
  return h == 0 ? v0 : h == 1 ? v1 : h == 2 ? v2 : v3;
}

// Per-head dot products of this warp's root row (columns spread over lanes,
// coalesced loads) with row `row` of a [*, ld] matrix at column offset `off`;
// the result is reduced over the warp, so every lane gets all H sums.
constexpr int kAttnMaxCols = 8;  // Do <= 256
__device__ __forceinline__ void head_dots(const float (&xv)[kAttnMaxCols], const float* __restrict__ row, int Do,
                                          int dh, int H, float (&out)[4]) {
  const int lane = threadIdx.x & 31;
  float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
  for (int c = 0; c < kAttnMaxCols; ++c) {
    const int d = lane + 32 * c;
    if (d < Do) {
      const float t = xv[c] * row[d];
      const int h = d / dh;
      if (h == 0) p0 += t;
      else if (h == 1) p1 += t;
      else if (h == 2) p2 += t;
      else p3 += t;
    }
  }
  out[0] = warp_sum(p0);
  out[1] = H > 1 ? warp_sum(p1) : 0.f;
  out[2] = H > 2 ? warp_sum(p2) : 0.f;
  out[3] = H > 3 ? warp_sum(p3) : 0.f;
}

__device__ __forceinline__ void load_row_cols(const float* __restrict__ row, int Do, float (&xv)[kAttnMaxCols]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < kAttnMaxCols; ++c) {
    const int d = lane + 32 * c;
    xv[c] = d < Do ? row[d] : 0.f;
  }
}

__global__ void tgn_attn_fwd_kernel(const float* __restrict__ Q, const float* __restrict__ KV,
                                    const int* __restrict__ cnt, const int* __restrict__ n_roots, int rmax, int k,
                                    int Do, int H, float att_drop, uint64_t seed, const int64_t* __restrict__ step_ctr,
                                    float* __restrict__ att_p, float* __restrict__ agg) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rmax) return;
  const int dh = Do / H;
  float* ag = agg + (int64_t)r * Do;
  const int nv = (r < *n_roots) ? cnt[r] : 0;
  if (nv == 0) {
    for (int d = lane; d < Do; d += 32) ag[d] = 0.f;
    return;
  }
  const uint64_t dseed = seed ^ (static_cast<uint64_t>(*step_ctr) * 0x9E3779B97F4A7C15ull);
  const float* q = Q + (int64_t)r * Do;
  const int64_t e = (int64_t)r * k + lane;
  // raw scores q . K_j per head: edges one at a time with columns over lanes (coalesced),
  // then lane j keeps edge j's sums
  float qv[kAttnMaxCols];
  load_row_cols(q, Do, qv);
  float raw[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < nv; ++j) {
    float hd[4];
    head_dots(qv, KV + ((int64_t)r * k + j) * (2 * Do), Do, dh, H, hd);
    if (lane == j) {
      raw[0] = hd[0];
      raw[1] = hd[1];
      raw[2] = hd[2];
      raw[3] = hd[3];
    }
  }
  float att[4] = {0.f, 0.f, 0.f, 0.f};
  const bool on = lane < nv;
  for (int h = 0; h < H && h < 4; ++h) {
    float s = -INFINITY;
    if (on) {
      const float acc = raw[h];
      s = acc > 0.f ? acc : 0.2f * acc;  // LeakyReLU(0.2)
    }
    const float m = warp_max(s);
    const float ex = on ? expf(s - m) : 0.f;
    const float sum = warp_sum(ex);
    const float p = ex / sum;
    if (on) att_p[e * H + h] = p;
    float a = p;
    if (on && att_drop > 0.f)
      a = dropout_keep(dseed, (uint64_t)(e * H + h), kStreamAttDrop, att_drop) ? p / (1.f - att_drop) : 0.f;
    att[h] = on ? a : 0.f;
  }
  // aggregate: lanes over feature columns (every lane runs every iteration so
  // the shuffles see a full warp; columns past Do are masked)
  for (int d0 = 0; d0 < Do; d0 += 32) {
    const int d = d0 + lane;
    const bool col = d < Do;
    const int h = col ? d / dh : 0;
    float acc = 0.f;
    for (int j = 0; j < nv; ++j) {
      const float a = shfl_head(att, H, h, j);
      if (col) acc = fmaf(a, KV[((int64_t)r * k + j) * (2 * Do) + Do + d], acc);
    }
    if (col) ag[d] = acc;
  }
}

// Attention forward for k * H <= 32 and k <= 16 (the configured fanouts): one
// warp per root. Every lane issues all its K-row loads at once (columns lane +
// 32 c of the k rows), accumulates per-(edge, head) partial dot products in
// registers and one transposed butterfly (31 shuffles) leaves the full score of
// (edge j, head h) in lane j * H + h. The softmax runs across the lanes of one
// head; the aggregation reads the V rows with the weights fetched by shuffle.
// Same outputs and dropout stream as tgn_attn_fwd_kernel.
template <int KMAX, int H>
__global__ void __launch_bounds__(256) tgn_attn_fwd_wide_kernel(
    const float* __restrict__ Q, const float* __restrict__ KV, const int* __restrict__ cnt,
    const int* __restrict__ n_roots, int rmax, int k, int Do, float att_drop, uint64_t seed,
    const int64_t* __restrict__ step_ctr, float* __restrict__ att_p, float* __restrict__ agg) {
  static_assert(KMAX * H <= 32, "one score per lane");
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rmax) return;
  const int dh = Do / H;
  float* ag = agg + (int64_t)r * Do;
  const int nv = (r < *n_roots) ? min(cnt[r], k) : 0;
  if (nv == 0) {
    for (int d = lane; d < Do; d += 32) ag[d] = 0.f;
    return;
  }
  const float* q = Q + (int64_t)r * Do;
  const float* kv = KV + (int64_t)r * k * (2 * Do);
  float qv[kAttnMaxCols];
  load_row_cols(q, Do, qv);
  // part[j * H + h]: this lane's share of score (j, h)
  float part[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) part[i] = 0.f;
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    if (j < nv) {
      const float* row = kv + (int64_t)j * (2 * Do);
#pragma unroll
      for (int c = 0; c < kAttnMaxCols; ++c) {
        const int d = lane + 32 * c;
        if (d < Do) {
          const float t = qv[c] * __ldg(row + d);
          const int h = d / dh;
#pragma unroll
          for (int hh = 0; hh < H; ++hh)
            if (h == hh) part[j * H + hh] += t;
        }
      }
    }
  }
  // transposed butterfly: after it, lane l holds the warp total of part[l]
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = up ? part[i] : part[i + off];
      const float keep = up ? part[i + off] : part[i];
      part[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  const int j = lane / H;
  const int h = lane % H;
  const bool on = j < nv;
  float sc = -INFINITY;
  if (on) sc = part[0] > 0.f ? part[0] : 0.2f * part[0];  // LeakyReLU(0.2)
  float m = sc;
  for (int o = H; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float ex = on ? expf(sc - m) : 0.f;
  float sum = ex;
  for (int o = H; o < 32; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float p = on ? ex / sum : 0.f;
  const int64_t e = (int64_t)r * k + j;
  float a = p;
  if (on) {
    att_p[e * H + h] = p;
    if (att_drop > 0.f) {
      const uint64_t dseed = seed ^ (static_cast<uint64_t>(*step_ctr) * 0x9E3779B97F4A7C15ull);
      a = dropout_keep(dseed, (uint64_t)(e * H + h), kStreamAttDrop, att_drop) ? p / (1.f - att_drop) : 0.f;
    }
  }
  // aggregate: lanes over feature columns, weights of (edge jj, head of column d) by shuffle
#pragma unroll
  for (int c = 0; c < kAttnMaxCols; ++c) {
    const int d = lane + 32 * c;
    if (32 * c >= Do) break;  // warp-uniform
    const int hd = d < Do ? d / dh : 0;
    float acc = 0.f;
#pragma unroll
    for (int jj = 0; jj < KMAX; ++jj) {
      if (jj < nv) {
        const float w = __shfl_sync(0xffffffffu, a, jj * H + hd);
        if (d < Do) acc = fmaf(w, __ldg(kv + (int64_t)jj * (2 * Do) + Do + d), acc);
      }
    }
    if (d < Do) ag[d] = acc;
  }
}

// Backward of the attention: dagg -> dKV (rows of invalid edges stay zero), dQ.
__global__ void tgn_attn_bwd_kernel(const float* __restrict__ Q, const float* __restrict__ KV,
                                    const float* __restrict__ att_p, const float* __restrict__ dagg,
                                    const int* __restrict__ cnt, const int* __restrict__ n_roots, int rmax, int k,
                                    int Do, int H, float att_drop, uint64_t seed, const int64_t* __restrict__ step_ctr,
                                    float* __restrict__ dKV, float* __restrict__ dQ) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rmax) return;
  const int dh = Do / H;
  const int nv = (r < *n_roots) ? cnt[r] : 0;
  float* dq = dQ + (int64_t)r * Do;
  // zero rows of padded edges
  for (int j = nv; j < k; ++j)
    for (int d = lane; d < 2 * Do; d += 32) dKV[((int64_t)r * k + j) * (2 * Do) + d] = 0.f;
  if (nv == 0) {
    for (int d = lane; d < Do; d += 32) dq[d] = 0.f;
    return;
  }
  // step_ctr was already advanced by this step's prep kernel, use the same value as forward
  const uint64_t dseed = seed ^ (static_cast<uint64_t>(*step_ctr) * 0x9E3779B97F4A7C15ull);
  const float* q = Q + (int64_t)r * Do;
  const float* g = dagg + (int64_t)r * Do;
  const int64_t e = (int64_t)r * k + lane;
  const bool on = lane < nv;
  // per edge, columns over lanes: g . V_j (attention-weight gradient) and q . K_j (raw score)
  float qv[kAttnMaxCols], gv[kAttnMaxCols];
  load_row_cols(q, Do, qv);
  load_row_cols(g, Do, gv);
  float draw[4] = {0.f, 0.f, 0.f, 0.f}, sraw[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < nv; ++j) {
    const float* kr = KV + ((int64_t)r * k + j) * (2 * Do);
    float hv[4], hk[4];
    head_dots(gv, kr + Do, Do, dh, H, hv);
    head_dots(qv, kr, Do, dh, H, hk);
    if (lane == j) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        draw[h] = hv[h];
        sraw[h] = hk[h];
      }
    }
  }
  float att[4] = {0.f, 0.f, 0.f, 0.f};
  float dsc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int h = 0; h < H && h < 4; ++h) {
    float p = 0.f, keep = 0.f, datt = 0.f, s = 0.f;
    if (on) {
      p = att_p[e * H + h];
      keep = 1.f;
      if (att_drop > 0.f)
        keep = dropout_keep(dseed, (uint64_t)(e * H + h), kStreamAttDrop, att_drop) ? 1.f / (1.f - att_drop) : 0.f;
      datt = draw[h];
      s = sraw[h];
    }
    att[h] = p * keep;
    const float dp = datt * keep;               // through dropout
    const float dot = warp_sum(on ? p * dp : 0.f);
    const float ds = on ? p * (dp - dot) : 0.f;  // softmax backward
    dsc[h] = on ? ds * (s > 0.f ? 1.f : 0.2f) : 0.f;  // LeakyReLU backward
  }
  for (int d0 = 0; d0 < Do; d0 += 32) {
    const int d = d0 + lane;
    const bool col = d < Do;
    const int h = col ? d / dh : 0;
    float dqa = 0.f;
    for (int j = 0; j < nv; ++j) {
      const float a = shfl_head(att, H, h, j);
      const float sj = shfl_head(dsc, H, h, j);
      if (!col) continue;
      float* row = dKV + ((int64_t)r * k + j) * (2 * Do);
      row[Do + d] = a * g[d];                               // dV
      row[d] = sj * q[d];                                   // dK
      dqa = fmaf(sj, KV[((int64_t)r * k + j) * (2 * Do) + d], dqa);  // dQ
    }
    if (col) dq[d] = dqa;
  }
}


// LayerNorm + ReLU + dropout backward (warp per row).
__device__ __forceinline__ void tgn_out_bwd_row(const float* __restrict__ dout, const float* __restrict__ xsave,
                                                const float* __restrict__ mean, const float* __restrict__ rstd,
                                                const float* __restrict__ gamma, int r, int lane, int Do, float drop,
                                                uint64_t seed, const int64_t* __restrict__ step_ctr,
                                                float* __restrict__ dpre, float* s_red) {
  float* dp = dpre + (int64_t)r * Do;
  const uint64_t dseed = seed ^ (static_cast<uint64_t>(*step_ctr) * 0x9E3779B97F4A7C15ull);
  const float mu = mean[r], rs = rstd[r];
  const float* x = xsave + (int64_t)r * Do;
  const float* dy = dout + (int64_t)r * Do;
  float sa = 0.f, sb = 0.f;
  for (int c = lane; c < Do; c += 32) {
    const float xh = (x[c] - mu) * rs;
    const float dxh = dy[c] * gamma[c];
    sa += dxh;
    sb += dxh * xh;
    atomicAdd(&s_red[c], dy[c] * xh);
    atomicAdd(&s_red[Do + c], dy[c]);
  }
  sa = warp_sum(sa) / Do;
  sb = warp_sum(sb) / Do;
  for (int c = lane; c < Do; c += 32) {
    const float xh = (x[c] - mu) * rs;
    const float dxh = dy[c] * gamma[c];
    float dx = rs * (dxh - sa - xh * sb);
    dx = x[c] > 0.f ? dx : 0.f;  // ReLU
    if (drop > 0.f)
      dx = dropout_keep(dseed, (uint64_t)r * Do + c, kStreamOutDrop, drop) ? dx / (1.f - drop) : 0.f;
    dp[c] = dx;
  }
}

__global__ void tgn_out_bwd_kernel(const float* __restrict__ dout, const float* __restrict__ xsave,
                                   const float* __restrict__ mean, const float* __restrict__ rstd,
                                   const float* __restrict__ gamma, const int* __restrict__ n_roots, int rmax, int Do,
                                   float drop, uint64_t seed, const int64_t* __restrict__ step_ctr,
                                   const int* __restrict__ edge_total, float* __restrict__ dpre,
                                   float* __restrict__ dgamma, float* __restrict__ dbeta) {
  // dgamma / dbeta: summed over the block's rows in shared memory, then one global
  // atomic per column and block (every row adds to the same Do addresses)
  extern __shared__ float s_red[];  // [2 * Do]
  for (int c = threadIdx.x; c < 2 * Do; c += blockDim.x) s_red[c] = 0.f;
  __syncthreads();
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  bool act = r < rmax;
  if (act && (r >= *n_roots || *edge_total == 0)) {
    float* dp = dpre + (int64_t)r * Do;
    for (int c = lane; c < Do; c += 32) dp[c] = 0.f;
    act = false;
  }
  if (act) tgn_out_bwd_row(dout, xsave, mean, rstd, gamma, r, lane, Do, drop, seed, step_ctr, dpre, s_red);
  __syncthreads();
  for (int c = threadIdx.x; c < Do; c += blockDim.x) {
    if (s_red[c] != 0.f) atomicAdd(&dgamma[c], s_red[c]);
    if (s_red[Do + c] != 0.f) atomicAdd(&dbeta[c], s_red[Do + c]);
  }
}

// ---------------------------------------------------------------------------
// link predictor scoring + BCE loss + gradients (warp per event)
// P: [rmax, 2D] per-root projections (src_fc | dst_fc incl. bias)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tgn_link_event(const float* __restrict__ P, const int* __restrict__ src_idx,
                                               const int* __restrict__ dst_idx, const int* __restrict__ neg_idx,
                                               int n, int i, int lane, int bmax, int D,
                                               const float* __restrict__ b_dst, const float* __restrict__ w_out,
                                               const float* __restrict__ b_out, int need_grad,
                                               float* __restrict__ scores, float* __restrict__ loss,
                                               float* __restrict__ dP, float* s_red) {
  const int si = src_idx[i], di = dst_idx[i], ni = neg_idx[i];
  const float* ps = P + (int64_t)si * 2 * D;
  const float* pd = P + (int64_t)di * 2 * D + D;
  const float* pn = ni >= 0 ? P + (int64_t)ni * 2 * D + D : nullptr;
  float sp = 0.f, sn = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float a = ps[d] + pd[d];
    const float bneg = ps[d] + (pn ? pn[d] : b_dst[d]);
    sp = fmaf(w_out[d], fmaxf(a, 0.f), sp);
    sn = fmaf(w_out[d], fmaxf(bneg, 0.f), sn);
  }
  sp = warp_sum(sp) + b_out[0];
  sn = warp_sum(sn) + b_out[0];
  if (lane == 0) {
    scores[i] = sp;
    scores[bmax + i] = sn;
    // BCE-with-logits: softplus(-x) for label 1, softplus(x) for label 0 (means over events)
    const float lp = fmaxf(-sp, 0.f) + log1pf(expf(-fabsf(sp)));
    const float ln = fmaxf(sn, 0.f) + log1pf(expf(-fabsf(sn)));
    atomicAdd(loss, (lp + ln) / n);
  }
  if (!need_grad) return;
  const float dpos = (sigmoidf_(sp) - 1.f) / n;
  const float dneg = sigmoidf_(sn) / n;
  float* dps = dP + (int64_t)si * 2 * D;
  float* dpd = dP + (int64_t)di * 2 * D + D;
  float* dpn = ni >= 0 ? dP + (int64_t)ni * 2 * D + D : nullptr;
  for (int d = lane; d < D; d += 32) {
    const float a = ps[d] + pd[d];
    const float bneg = ps[d] + (pn ? pn[d] : b_dst[d]);
    atomicAdd(&s_red[d], dpos * fmaxf(a, 0.f) + dneg * fmaxf(bneg, 0.f));
    const float da = a > 0.f ? dpos * w_out[d] : 0.f;
    const float db = bneg > 0.f ? dneg * w_out[d] : 0.f;
    atomicAdd(&dps[d], da + db);
    atomicAdd(&dpd[d], da);
    if (dpn) atomicAdd(&dpn[d], db);
    else atomicAdd(&s_red[D + d], db);
  }
  if (lane == 0) atomicAdd(&s_red[2 * D], dpos + dneg);
}

__global__ void tgn_link_kernel(const float* __restrict__ P, const int* __restrict__ src_idx,
                                const int* __restrict__ dst_idx, const int* __restrict__ neg_idx,
                                const int* __restrict__ n_ev, int bmax, int D, const float* __restrict__ b_dst,
                                const float* __restrict__ w_out, const float* __restrict__ b_out, int need_grad,
                                float* __restrict__ scores, float* __restrict__ loss, float* __restrict__ dP,
                                float* __restrict__ g_w_out, float* __restrict__ g_b_out, float* __restrict__ g_b_dst) {
  // g_w_out, g_b_dst, g_b_out: summed over the block's events in shared memory, then
  // one global atomic per entry and block (every event adds to the same addresses)
  // and the loss: [g_w_out (D) | g_b_dst (D) | g_b_out | loss]
  extern __shared__ float s_red[];  // [2 * D + 2]
  for (int c = threadIdx.x; c < 2 * D + 2; c += blockDim.x) s_red[c] = 0.f;
  __syncthreads();
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int n = *n_ev;
  if (i < bmax && i < n) tgn_link_event(P, src_idx, dst_idx, neg_idx, n, i, lane, bmax, D, b_dst, w_out, b_out,
                                        need_grad, scores, s_red + 2 * D + 1, dP, s_red);
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * D + 2; c += blockDim.x) {
    const float v = s_red[c];
    if (v == 0.f) continue;
    if (c < D) atomicAdd(&g_w_out[c], v);
    else if (c < 2 * D) atomicAdd(&g_b_dst[c - D], v);
    else if (c == 2 * D) atomicAdd(g_b_out, v);
    else atomicAdd(loss, v);
  }
}

// AP (sklearn semantics), ROC-AUC (ties count 1/2) and the pairwise "mrr" of the reference.
// Scores are staged in shared memory; each thread owns positives.
__global__ void __launch_bounds__(1024) tgn_metrics_kernel(const float* __restrict__ scores,
                                                           const int* __restrict__ n_ev, int bmax,
                                                           float* __restrict__ out) {
  extern __shared__ float sh_scores[];  // [2 * n]
  __shared__ float s_ap, s_auc, s_gt;
  const int n = min(*n_ev, bmax);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    sh_scores[i] = scores[i];
    sh_scores[n + i] = scores[bmax + i];
  }
  if (threadIdx.x == 0) { s_ap = 0.f; s_auc = 0.f; s_gt = 0.f; }
  __syncthreads();
  float ap = 0.f, auc = 0.f, gt = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float sp = sh_scores[i];
    int pos_ge = 0, neg_ge = 0, neg_lt = 0, neg_eq = 0;
    for (int j = 0; j < n; ++j) {
      const float p2 = sh_scores[j], n2 = sh_scores[n + j];
      pos_ge += p2 >= sp;
      neg_ge += n2 >= sp;
      neg_lt += n2 < sp;
      neg_eq += n2 == sp;
    }
    ap += static_cast<float>(pos_ge) / static_cast<float>(pos_ge + neg_ge);
    auc += neg_lt + 0.5f * neg_eq;
    gt += neg_lt;
  }
  ap = warp_sum(ap); auc = warp_sum(auc); gt = warp_sum(gt);
  if ((threadIdx.x & 31) == 0) { atomicAdd(&s_ap, ap); atomicAdd(&s_auc, auc); atomicAdd(&s_gt, gt); }
  __syncthreads();
  if (threadIdx.x == 0) {
    const float nn = fmaxf(1.f, static_cast<float>(n));
    out[0] = s_ap / nn;
    out[1] = s_auc / (nn * nn);
    out[2] = s_gt / (nn * nn);
  }
}


// ---------------------------------------------------------------------------
// launchers (called from the torch-side wrappers)
// ---------------------------------------------------------------------------
void launch_tgn_prep(dim3 grid, dim3 block, cudaStream_t st, PrepArgs a) {
  count_launch();
  tgn_prep_kernel<<<grid, block, 0, st>>>(a);
}

void launch_tgn_sample(dim3 grid, dim3 block, cudaStream_t st, const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                  const int64_t* __restrict__ root_ts_scalar, const int64_t* __restrict__ root_ts_vec,
                                  const int64_t* __restrict__ rowptr, const int64_t* __restrict__ nbr,
                                  const int64_t* __restrict__ eid, const int64_t* __restrict__ ets, int k, int policy,
                                  uint64_t seed, const int64_t* __restrict__ step_ctr, int64_t* __restrict__ out_nbr,
                                  int64_t* __restrict__ out_eid, float* __restrict__ out_dt,
                                  int* __restrict__ out_cnt, int* __restrict__ edge_total) {
  count_launch();
  tgn_sample_kernel<<<grid, block, 0, st>>>(roots, n_roots, rmax, root_ts_scalar, root_ts_vec, rowptr, nbr, eid, ets, k, policy, seed, step_ctr, out_nbr, out_eid, out_dt, out_cnt, edge_total);
}

void launch_tgn_mailbox(dim3 grid, dim3 block, cudaStream_t st, const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                   const int* __restrict__ win, const int* __restrict__ cnt,
                                   const int* __restrict__ src_idx, const int* __restrict__ dst_idx,
                                   const int64_t* __restrict__ ev_eid, const float* __restrict__ ev_ts,
                                   const float* __restrict__ mem_prev, int D, const void* __restrict__ efeat,
                                   int efeat_bf16, int efeat_ld, int e_raw, int E, float* __restrict__ mailbox,
                                   float* __restrict__ mailbox_ts, int64_t* __restrict__ next_pos, int K) {
  count_launch();
  tgn_mailbox_kernel<<<grid, block, 0, st>>>(roots, n_roots, rmax, win, cnt, src_idx, dst_idx, ev_eid, ev_ts, mem_prev, D, efeat, efeat_bf16, efeat_ld, e_raw, E, mailbox, mailbox_ts, next_pos, K);
}

void launch_tgn_attn_fwd(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ Q, const float* __restrict__ KV,
                                    const int* __restrict__ cnt, const int* __restrict__ n_roots, int rmax, int k,
                                    int Do, int H, float att_drop, uint64_t seed, const int64_t* __restrict__ step_ctr,
                                    float* __restrict__ att_p, float* __restrict__ agg) {
  count_launch();
  if (Do % H == 0 && Do <= 32 * kAttnMaxCols) {
#define SU_ATTN_WIDE(KM, HH)                                                                                  \
  tgn_attn_fwd_wide_kernel<KM, HH><<<grid, block, 0, st>>>(Q, KV, cnt, n_roots, rmax, k, Do, att_drop, seed, \
                                                           step_ctr, att_p, agg);                            \
  return;
    if (H == 1 && k <= 8) { SU_ATTN_WIDE(8, 1) }
    if (H == 1 && k <= 16) { SU_ATTN_WIDE(16, 1) }
    if (H == 2 && k <= 8) { SU_ATTN_WIDE(8, 2) }
    if (H == 2 && k <= 16) { SU_ATTN_WIDE(16, 2) }
    if (H == 4 && k <= 8) { SU_ATTN_WIDE(8, 4) }
#undef SU_ATTN_WIDE
  }
  tgn_attn_fwd_kernel<<<grid, block, 0, st>>>(Q, KV, cnt, n_roots, rmax, k, Do, H, att_drop, seed, step_ctr, att_p, agg);
}

void launch_tgn_attn_bwd(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ Q, const float* __restrict__ KV,
                                    const float* __restrict__ att_p, const float* __restrict__ dagg,
                                    const int* __restrict__ cnt, const int* __restrict__ n_roots, int rmax, int k,
                                    int Do, int H, float att_drop, uint64_t seed, const int64_t* __restrict__ step_ctr,
                                    float* __restrict__ dKV, float* __restrict__ dQ) {
  count_launch();
  tgn_attn_bwd_kernel<<<grid, block, 0, st>>>(Q, KV, att_p, dagg, cnt, n_roots, rmax, k, Do, H, att_drop, seed, step_ctr, dKV, dQ);
}

void launch_tgn_out_bwd(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ dout, const float* __restrict__ xsave,
                                   const float* __restrict__ mean, const float* __restrict__ rstd,
                                   const float* __restrict__ gamma, const int* __restrict__ n_roots, int rmax, int Do,
                                   float drop, uint64_t seed, const int64_t* __restrict__ step_ctr,
                                   const int* __restrict__ edge_total, float* __restrict__ dpre,
                                   float* __restrict__ dgamma, float* __restrict__ dbeta) {
  count_launch();
  tgn_out_bwd_kernel<<<grid, block, 2 * Do * sizeof(float), st>>>(dout, xsave, mean, rstd, gamma, n_roots, rmax, Do, drop, seed, step_ctr, edge_total, dpre, dgamma, dbeta);
}

void launch_tgn_link(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ P, const int* __restrict__ src_idx,
                                const int* __restrict__ dst_idx, const int* __restrict__ neg_idx,
                                const int* __restrict__ n_ev, int bmax, int D, const float* __restrict__ b_dst,
                                const float* __restrict__ w_out, const float* __restrict__ b_out, int need_grad,
                                float* __restrict__ scores, float* __restrict__ loss, float* __restrict__ dP,
                                float* __restrict__ g_w_out, float* __restrict__ g_b_out, float* __restrict__ g_b_dst) {
  count_launch();
  tgn_link_kernel<<<grid, block, (2 * D + 2) * sizeof(float), st>>>(P, src_idx, dst_idx, neg_idx, n_ev, bmax, D, b_dst, w_out, b_out, need_grad, scores, loss, dP, g_w_out, g_b_out, g_b_dst);
}

void launch_tgn_metrics(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ scores,
                                                           const int* __restrict__ n_ev, int bmax,
                                                           float* __restrict__ out) {
  const int smem = 2 * bmax * static_cast<int>(sizeof(float));
  if (smem > 48 * 1024) cudaFuncSetAttribute(tgn_metrics_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  count_launch();
  tgn_metrics_kernel<<<grid, block, smem, st>>>(scores, n_ev, bmax, out);
}

}  // namespace su


namespace su {

// Time-encoder gradient from the products accumulated by the W_kv weight-gradient
// GEMM (M_t = dKV^T (-sin(w t + b) t), M_1 = dKV^T (-sin(w t + b))) and the b_q
// gradient (row sums of dQ; roots encode t = 0):
//   dw[c] += sum_o Wk[o, ct + c] M_t[o, c] + Wv[o, ct + c] M_t[Do + o, c]
//   db[c] += (same with M_1) - sin(b[c]) * sum_o Wq[o, cq + c] gbq[o]
__global__ void __launch_bounds__(1024) time_grad_finish_kernel(
    const float* __restrict__ wk, const float* __restrict__ wv, int ldw, int ct, const float* __restrict__ wq,
    int ldq, int cq, int Do, int T, const float* __restrict__ Mt, const float* __restrict__ M1,
    const float* __restrict__ gbq, const float* __restrict__ b, float* __restrict__ dw, float* __restrict__ db) {
  // block: 32 columns (lanes) x 32 warps over the output features o
  __shared__ float red[3][32][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float sw = 0.f, sb = 0.f, sq = 0.f;
  if (c < T) {
    for (int o = warp; o < Do; o += 32) {
      const float a = wk[static_cast<int64_t>(o) * ldw + ct + c];
      const float v = wv[static_cast<int64_t>(o) * ldw + ct + c];
      sw = fmaf(a, Mt[static_cast<int64_t>(o) * T + c], sw);
      sw = fmaf(v, Mt[static_cast<int64_t>(Do + o) * T + c], sw);
      sb = fmaf(a, M1[static_cast<int64_t>(o) * T + c], sb);
      sb = fmaf(v, M1[static_cast<int64_t>(Do + o) * T + c], sb);
      sq = fmaf(wq[static_cast<int64_t>(o) * ldq + cq + c], gbq[o], sq);
    }
  }
  red[0][warp][lane] = sw;
  red[1][warp][lane] = sb;
  red[2][warp][lane] = sq;
  __syncthreads();
  if (warp == 0 && c < T) {
    float tw = 0.f, tb = 0.f, tq = 0.f;
    for (int w = 0; w < 32; ++w) {
      tw += red[0][w][lane];
      tb += red[1][w][lane];
      tq += red[2][w][lane];
    }
    dw[c] += tw;
    db[c] += tb - sinf(b[c]) * tq;
  }
}

void launch_time_grad_finish(cudaStream_t st, const float* wk, const float* wv, int ldw, int ct, const float* wq,
                             int ldq, int cq, int Do, int T, const float* Mt, const float* M1, const float* gbq,
                             const float* b, float* dw, float* db) {
  if (T <= 0) return;
  count_launch();
  time_grad_finish_kernel<<<(T + 31) / 32, 1024, 0, st>>>(wk, wv, ldw, ct, wq, ldq, cq, Do, T, Mt, M1, gbq, b, dw,
                                                          db);
}

// ---------------------------------------------------------------------------
// JODIE time-projection embedding (warp per root row)
//   prev_ts[r] = memory_ts of root r before this step's memory update
//   z[r, c]    = h[r, c] * (1 + w[c] * dt_r + b[c]),  dt_r = (root_ts - prev_ts[r]) * dt_scale (0 if never updated)
// h = the updated memory row: table row roots[r], or row r of `fresh` (multi-GPU step buffer).
// ---------------------------------------------------------------------------
__global__ void jodie_prev_ts_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                     const float* __restrict__ mem_ts, const float* const* __restrict__ ts_peers,
                                     const int* __restrict__ owner, float* __restrict__ prev_ts) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rmax) return;
  if (r >= *n_roots) {
    prev_ts[r] = -1.f;
    return;
  }
  const int64_t v = roots[r];
  prev_ts[r] = ts_peers ? ts_peers[owner[v]][v] : mem_ts[v];
}

__global__ void jodie_project_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                     const float* __restrict__ mem, const float* __restrict__ fresh, int D,
                                     const float* __restrict__ prev_ts, const int64_t* __restrict__ root_ts,
                                     float dt_scale, const float* __restrict__ w, const float* __restrict__ b,
                                     float* __restrict__ out, float* __restrict__ dt_out) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rmax || r >= *n_roots) return;
  const float pt = prev_ts[r];
  const float dt = pt >= 0.f ? (static_cast<float>(*root_ts) - pt) * dt_scale : 0.f;
  if (lane == 0) dt_out[r] = dt;
  const float* h = fresh ? fresh + static_cast<int64_t>(r) * D : mem + roots[r] * D;
  float* o = out + static_cast<int64_t>(r) * D;
  for (int c = lane; c < D; c += 32) o[c] = h[c] * (1.f + fmaf(w[c], dt, b[c]));
}

// dw[c] += sum_r dz[r,c] h[r,c] dt_r ;  db[c] += sum_r dz[r,c] h[r,c]   (threads over columns, blocks over rows)
__global__ void jodie_project_bwd_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                         const float* __restrict__ mem, const float* __restrict__ fresh, int D,
                                         const float* __restrict__ dt, const float* __restrict__ dz,
                                         float* __restrict__ dw, float* __restrict__ db) {
  const int c = threadIdx.x;
  if (c >= D) return;
  const int r0 = blockIdx.x * 32;
  const int n = min(*n_roots, rmax);
  float gw = 0.f, gb = 0.f;
  for (int r = r0; r < r0 + 32 && r < n; ++r) {
    const float* h = fresh ? fresh + static_cast<int64_t>(r) * D : mem + roots[r] * D;
    const float g = dz[static_cast<int64_t>(r) * D + c] * h[c];
    gb += g;
    gw = fmaf(g, dt[r], gw);
  }
  atomicAdd(&dw[c], gw);
  atomicAdd(&db[c], gb);
}

void launch_jodie_prev_ts(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const float* mem_ts,
                          const float* const* ts_peers, const int* owner, float* prev_ts) {
  if (rmax <= 0) return;
  count_launch();
  jodie_prev_ts_kernel<<<(rmax + 255) / 256, 256, 0, st>>>(roots, n_roots, rmax, mem_ts, ts_peers, owner, prev_ts);
}

void launch_jodie_project(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const float* mem,
                          const float* fresh, int D, const float* prev_ts, const int64_t* root_ts, float dt_scale,
                          const float* w, const float* b, float* out, float* dt_out) {
  if (rmax <= 0) return;
  count_launch();
  jodie_project_kernel<<<(rmax * 32 + 255) / 256, 256, 0, st>>>(roots, n_roots, rmax, mem, fresh, D, prev_ts,
                                                                 root_ts, dt_scale, w, b, out, dt_out);
}

void launch_jodie_project_bwd(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const float* mem,
                              const float* fresh, int D, const float* dt, const float* dz, float* dw, float* db) {
  if (rmax <= 0) return;
  count_launch();
  jodie_project_bwd_kernel<<<(rmax + 31) / 32, (D + 31) / 32 * 32, 0, st>>>(roots, n_roots, rmax, mem, fresh, D, dt,
                                                                            dz, dw, db);
}

}  // namespace su
