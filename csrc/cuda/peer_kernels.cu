// Kernels that talk to peer GPUs through NVLink / NVSwitch with plain loads,
// stores and atomics on peer memory mapped into this process (symmetric
// allocations): no NCCL call and no TMA on these paths.
//
//  peer_barrier      : device-side barrier over W ranks. Rank r stores the
//                      barrier epoch into slot r of every peer's flag array
//                      (st.release.sys) and waits until all peers' slots in its
//                      own array reach the epoch (ld.acquire.sys). The wait is
//                      bounded: on expiry it records kPeerTimeout and returns.
//  peer_signal / the wait inside tgn_peer_wait_claim: the same barrier split in
//                      two halves, so that work placed between them (the next
//                      step's sampling) overlaps the peers' arrival.
//  peer_allreduce_adam: gradient all-reduce fused with the Adam update. Every
//                      rank reads the W gradient buffers, sums them in rank
//                      order (bit-identical sums on all ranks), scales and
//                      applies Adam to its own parameter copy.
//  peer_rs_adam_ag   : the traffic-optimal form: rank r sums only its 1/W shard
//                      of the gradient over the W buffers (reduce-scatter),
//                      applies Adam to that shard and stores the new parameter
//                      shard into every rank's parameter buffer (all-gather):
//                      2 (W-1)/W of the buffer crosses NVLink per rank instead
//                      of (W-1) x. Each element is computed by one rank only,
//                      so the replicas stay bit-identical.
//  tgn_peer_wait_claim: (after the end-of-step wait) each rank proposes its
//                      final mail for each root with the key (ts, event id),
//                      claimed with a 64-bit atomicMax on the owner. Claims are
//                      posted before the step's barrier, so the winners can
//                      write right after it without a second barrier.
//  tgn_peer_push     : per root, the new memory row stored into the owner
//                      rank's memory table (memory_ts = max over writers; rows
//                      of one node written by several ranks are identical, they
//                      come from the same state) and, for the claim winner, the
//                      mailbox slot.
//
// The multi-rank orchestration lives in starry_unigraph/parallel (reference
// semantics: backends/ctdg/runtime/memory.py:328-553 pushes memory and mail to
// owners; here the push is a direct store into the owner's table).
#include "kernels.h"

namespace su {

__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t orderable_ts(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------
// barrier (one block of 32 threads; W <= 32)
// ---------------------------------------------------------------------------
__global__ void peer_barrier_kernel(uint64_t* const* __restrict__ flag_ptrs, int rank, int W,
                                    int64_t* __restrict__ epoch, int* __restrict__ status, long long budget) {
  const int p = threadIdx.x;
  const uint64_t e = static_cast<uint64_t>(*epoch) + 1ull;
  __threadfence_system();  // this rank's earlier peer stores are visible before the signal
  if (p < W && p != rank) st_release_sys_u64(flag_ptrs[p] + rank, e);
  if (p < W && p != rank) {
    const uint64_t* mine = flag_ptrs[rank] + p;
    const long long t0 = clock64();
    while (ld_acquire_sys_u64(mine) < e) {
      if (clock64() - t0 > budget) {
        record_status(status, kPeerTimeout);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  if (p == 0) *epoch = static_cast<int64_t>(e);
}

void launch_peer_barrier(cudaStream_t st, uint64_t* const* flag_ptrs, int rank, int W, int64_t* epoch, int* status,
                         long long budget) {
  count_launch();
  peer_barrier_kernel<<<1, 32, 0, st>>>(flag_ptrs, rank, W, epoch, status, budget);
}

// Split barrier: signal (store the next epoch into this rank's slot of every
// peer's flag array, no wait) ...
__global__ void peer_signal_kernel(uint64_t* const* __restrict__ flag_ptrs, int rank, int W,
                                   int64_t* __restrict__ epoch) {
  const int p = threadIdx.x;
  const uint64_t e = static_cast<uint64_t>(*epoch) + 1ull;
  __threadfence_system();  // this rank's earlier stores to peer memory are visible before the flag
  if (p < W && p != rank) st_release_sys_u64(flag_ptrs[p] + rank, e);
  __syncthreads();
  if (p == 0) *epoch = static_cast<int64_t>(e);
}

void launch_peer_signal(cudaStream_t st, uint64_t* const* flag_ptrs, int rank, int W, int64_t* epoch) {
  count_launch();
  peer_signal_kernel<<<1, 32, 0, st>>>(flag_ptrs, rank, W, epoch);
}

// ... and, later, wait (bounded) until every peer's slot in this rank's own
// flag array has reached this rank's current epoch. Called by one warp (lanes
// = peers); the caller synchronises the block afterwards.
__device__ __forceinline__ void peer_wait_warp(const uint64_t* __restrict__ my_flags, int rank, int W,
                                               const int64_t* __restrict__ epoch, int* status, long long budget) {
  const int p = threadIdx.x & 31;
  const uint64_t e = static_cast<uint64_t>(*epoch);
  if (p < W && p != rank) {
    const long long t0 = clock64();
    while (ld_acquire_sys_u64(my_flags + p) < e) {
      if (clock64() - t0 > budget) {
        record_status(status, kPeerTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
}

__global__ void peer_wait_kernel(const uint64_t* __restrict__ my_flags, int rank, int W,
                                 const int64_t* __restrict__ epoch, int* status, long long budget) {
  peer_wait_warp(my_flags, rank, W, epoch, status, budget);
}

void launch_peer_wait(cudaStream_t st, const uint64_t* my_flags, int rank, int W, const int64_t* epoch, int* status,
                      long long budget) {
  count_launch();
  peer_wait_kernel<<<1, 32, 0, st>>>(my_flags, rank, W, epoch, status, budget);
}

// ---------------------------------------------------------------------------
// all-reduce + Adam
// ---------------------------------------------------------------------------
__global__ void peer_allreduce_adam_kernel(const float* const* __restrict__ grads, int W, float* __restrict__ p,
                                           float* __restrict__ m, float* __restrict__ v, int64_t n,
                                           int64_t* __restrict__ step, unsigned int* __restrict__ done, float lr,
                                           float b1, float b2, float eps, float wd, float scale) {
  const float t = static_cast<float>(*step + 1);
  const float bc1 = 1.f - powf(b1, t);
  const float bc2_sqrt = sqrtf(1.f - powf(b2, t));
  const float step_size = lr / bc1;
  const int64_t n4 = n / 4;  // n is a multiple of 4 (flat buffers are padded)
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 g = reinterpret_cast<const float4*>(grads[0])[i];
    for (int q = 1; q < W; ++q) {
      const float4 h = reinterpret_cast<const float4*>(grads[q])[i];
      g.x += h.x;
      g.y += h.y;
      g.z += h.z;
      g.w += h.w;
    }
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pa = &pp.x;
    float* ma = &mm.x;
    float* va = &vv.x;
    const float* ga = &g.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gr = ga[j] * scale + wd * pa[j];
      ma[j] = b1 * ma[j] + (1.f - b1) * gr;
      va[j] = b2 * va[j] + (1.f - b2) * gr * gr;
      pa[j] -= step_size * ma[j] / (sqrtf(va[j]) / bc2_sqrt + eps);
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      *step += 1;
      *done = 0u;
      __threadfence();
    }
  }
}

void launch_peer_allreduce_adam(cudaStream_t st, int blocks, const float* const* grads, int W, float* p, float* m,
                                float* v, int64_t n, int64_t* step, unsigned int* done, float lr, float b1, float b2,
                                float eps, float wd, float scale) {
  count_launch();
  peer_allreduce_adam_kernel<<<blocks, 256, 0, st>>>(grads, W, p, m, v, n, step, done, lr, b1, b2, eps, wd, scale);
}

// ---------------------------------------------------------------------------
// reduce-scatter + Adam + all-gather over peer memory
//
// Rank r owns float4 elements [r * shard4, (r + 1) * shard4): it sums them over
// the W gradient buffers in rank order, applies Adam (its moments are kept
// for its own shard only) and stores the new values into the parameter buffer
// of every rank, its own included.
// ---------------------------------------------------------------------------
// Per thread kRsUnroll float4 of the shard, strided by the grid: all W gradient
// loads of the group (local and over NVLink) are issued before any arithmetic,
// so each thread keeps kRsUnroll * W 16-byte loads in flight instead of W.
constexpr int kRsUnroll = 4;

__device__ __forceinline__ float4 adam4(float4 g, float4& pp, float4& mm, float4& vv, float b1, float b2,
                                        float eps, float wd, float scale, float step_size, float bc2_sqrt) {
  float* pa = &pp.x;
  float* ma = &mm.x;
  float* va = &vv.x;
  const float* ga = &g.x;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float gr = ga[j] * scale + wd * pa[j];
    ma[j] = b1 * ma[j] + (1.f - b1) * gr;
    va[j] = b2 * va[j] + (1.f - b2) * gr * gr;
    pa[j] -= step_size * ma[j] / (sqrtf(va[j]) / bc2_sqrt + eps);
  }
  return pp;
}

__global__ void peer_rs_adam_ag_kernel(const float* const* __restrict__ grads, float* const* __restrict__ params,
                                       int W, int rank, float* __restrict__ m, float* __restrict__ v, int64_t n4,
                                       int64_t shard4, int64_t* __restrict__ step, unsigned int* __restrict__ done,
                                       float lr, float b1, float b2, float eps, float wd, float scale) {
  const float t = static_cast<float>(*step + 1);
  const float bc1 = 1.f - powf(b1, t);
  const float bc2_sqrt = sqrtf(1.f - powf(b2, t));
  const float step_size = lr / bc1;
  const int64_t lo = static_cast<int64_t>(rank) * shard4;
  const int64_t hi = min(n4, lo + shard4);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const float4* mine = reinterpret_cast<const float4*>(params[rank]);
  for (int64_t base = lo + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; base < hi;
       base += stride * kRsUnroll) {
    float4 g[kRsUnroll];
#pragma unroll
    for (int u = 0; u < kRsUnroll; ++u) {
      const int64_t i = base + u * stride;
      g[u] = i < hi ? reinterpret_cast<const float4*>(grads[0])[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int q = 1; q < W; ++q) {
      const float4* gq = reinterpret_cast<const float4*>(grads[q]);
      float4 h[kRsUnroll];
#pragma unroll
      for (int u = 0; u < kRsUnroll; ++u) {
        const int64_t i = base + u * stride;
        h[u] = i < hi ? gq[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kRsUnroll; ++u) {  // rank order: every replica sums identically
        g[u].x += h[u].x;
        g[u].y += h[u].y;
        g[u].z += h[u].z;
        g[u].w += h[u].w;
      }
    }
#pragma unroll
    for (int u = 0; u < kRsUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i >= hi) break;
      float4 pp = mine[i];
      float4 mm = reinterpret_cast<float4*>(m)[i];
      float4 vv = reinterpret_cast<float4*>(v)[i];
      adam4(g[u], pp, mm, vv, b1, b2, eps, wd, scale, step_size, bc2_sqrt);
      reinterpret_cast<float4*>(m)[i] = mm;
      reinterpret_cast<float4*>(v)[i] = vv;
      for (int q = 0; q < W; ++q) reinterpret_cast<float4*>(params[q])[i] = pp;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      *step += 1;
      *done = 0u;
      __threadfence();
    }
  }
}

void launch_peer_rs_adam_ag(cudaStream_t st, int blocks, const float* const* grads, float* const* params, int W,
                            int rank, float* m, float* v, int64_t n, int64_t* step, unsigned int* done, float lr,
                            float b1, float b2, float eps, float wd, float scale) {
  const int64_t n4 = n / 4;  // n is a multiple of 4 (flat buffers are padded)
  const int64_t shard4 = (n4 + W - 1) / W;
  count_launch();
  peer_rs_adam_ag_kernel<<<blocks, 256, 0, st>>>(grads, params, W, rank, m, v, n4, shard4, step, done, lr, b1, b2,
                                                  eps, wd, scale);
}

// ---------------------------------------------------------------------------
// CTDG memory write-back (block of 64 threads per root, D columns)
//
// Optional historical-cache filter (reference backends/ctdg/runtime/cache.py:
// MemShare-style): a root owned by another rank keeps a cached copy of the last
// row this rank pushed; the new row is pushed only when it was never pushed or
// its cosine distance to the cached row exceeds `thresh` (= 1 - alpha). A pushed
// row refreshes the cache.
// ---------------------------------------------------------------------------
// Stores root r's new memory row into the owner's table (unless the historical
// filter drops it). Block-uniform control flow; blockDim.x is a multiple of 32
// and at most 256.
__device__ __forceinline__ void writeback_root(int r, const int64_t* __restrict__ roots,
                                               const float* __restrict__ mem_new, int D,
                                               const int* __restrict__ owner, float* const* __restrict__ mem_tables,
                                               float* const* __restrict__ ts_tables, const float* __restrict__ ts_max,
                                               const HistCache& hc) {
  const int64_t v = roots[r];
  const int o = owner[v];
  const float* src = mem_new + static_cast<int64_t>(r) * D;
  if (hc.cache != nullptr && o != hc.rank) {
    const int64_t slot = hc.slot_of[v];
    if (slot >= 0) {
      float* cr = hc.cache + slot * D;
      float dot = 0.f, na = 0.f, nb = 0.f;
      for (int c = threadIdx.x; c < D; c += blockDim.x) {
        const float a = src[c], b = cr[c];
        dot += a * b;
        na += a * a;
        nb += b * b;
      }
      __shared__ float red[3][8];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        dot += __shfl_xor_sync(0xffffffffu, dot, off);
        na += __shfl_xor_sync(0xffffffffu, na, off);
        nb += __shfl_xor_sync(0xffffffffu, nb, off);
      }
      const int w = threadIdx.x >> 5;
      if ((threadIdx.x & 31) == 0) {
        red[0][w] = dot;
        red[1][w] = na;
        red[2][w] = nb;
      }
      __syncthreads();
      dot = na = nb = 0.f;
      for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) {
        dot += red[0][i];
        na += red[1][i];
        nb += red[2][i];
      }
      __syncthreads();  // red is reused by the next root of this block
      const bool never = hc.cache_ts[slot] < 0.f;
      const float cosv = dot / fmaxf(sqrtf(na) * sqrtf(nb), 1e-8f);
      if (!never && 1.f - cosv <= hc.thresh) return;  // block-uniform: skip the push
      for (int c = threadIdx.x; c < D; c += blockDim.x) cr[c] = src[c];
      if (threadIdx.x == 0) hc.cache_ts[slot] = *ts_max;
    }
  }
  float* dst = mem_tables[o] + v * D;
  if ((D & 3) == 0) {
    for (int c = threadIdx.x; c < D / 4; c += blockDim.x)
      reinterpret_cast<float4*>(dst)[c] = reinterpret_cast<const float4*>(src)[c];
  } else {
    for (int c = threadIdx.x; c < D; c += blockDim.x) dst[c] = src[c];
  }
  if (threadIdx.x == 0) {
    // timestamps are >= 0, so their bit patterns order like signed ints
    atomicMax(reinterpret_cast<int*>(ts_tables[o] + v), __float_as_int(*ts_max));
  }
}

__global__ void tgn_peer_writeback_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                          const float* __restrict__ mem_new, int D, const int* __restrict__ owner,
                                          float* const* __restrict__ mem_tables, float* const* __restrict__ ts_tables,
                                          const float* __restrict__ ts_max, HistCache hc) {
  const int r = blockIdx.x;
  if (r >= rmax || r >= *n_roots) return;
  writeback_root(r, roots, mem_new, D, owner, mem_tables, ts_tables, ts_max, hc);
}

void launch_tgn_peer_writeback(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax,
                               const float* mem_new, int D, const int* owner, float* const* mem_tables,
                               float* const* ts_tables, const float* ts_max, const HistCache& hc) {
  if (rmax <= 0) return;
  count_launch();
  tgn_peer_writeback_kernel<<<rmax, 64, 0, st>>>(roots, n_roots, rmax, mem_new, D, owner, mem_tables, ts_tables,
                                                 ts_max, hc);
}

// ---------------------------------------------------------------------------
// mailbox (one slot): claim then write
// ---------------------------------------------------------------------------
// The final local mail of root r is the dst-pass winner when the root is a
// destination in this batch, else the src-pass winner (the order in which the
// single-GPU mailbox kernel writes the slot).
__device__ __forceinline__ int final_mail_event(const int* win, int rmax, int r, int& pass) {
  const int d = win[rmax + r];
  if (d >= 0) {
    pass = 1;
    return d;
  }
  pass = 0;
  return win[r];
}

__device__ __forceinline__ unsigned long long mail_key(float ts, int64_t eid) {
  return (static_cast<unsigned long long>(orderable_ts(ts)) << 32) |
         static_cast<unsigned long long>(static_cast<uint32_t>(eid));
}

__device__ __forceinline__ void claim_root(int r, int rmax, const int64_t* __restrict__ roots,
                                           const int* __restrict__ win, const int64_t* __restrict__ ev_eid,
                                           const float* __restrict__ ev_ts, const int* __restrict__ owner,
                                           unsigned long long* const* __restrict__ claim_tables) {
  int pass = 0;
  const int i = final_mail_event(win, rmax, r, pass);
  if (i < 0) return;
  const int64_t v = roots[r];
  atomicMax(claim_tables[owner[v]] + v, mail_key(ev_ts[i], ev_eid[i]));
}

__global__ void tgn_peer_mail_claim_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots,
                                           int rmax, const int* __restrict__ win, const int64_t* __restrict__ ev_eid,
                                           const float* __restrict__ ev_ts, const int* __restrict__ owner,
                                           unsigned long long* const* __restrict__ claim_tables) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rmax || r >= *n_roots) return;
  claim_root(r, rmax, roots, win, ev_eid, ev_ts, owner, claim_tables);
}

// The second half of the split end-of-step barrier fused with this step's
// claims: every block first waits (bounded) until all peers signalled the end
// of the previous step, i.e. finished their write-backs and mail writes into
// the tables and their reads of this rank's gradient buffer.
__global__ void tgn_peer_wait_claim_kernel(const uint64_t* __restrict__ my_flags, int rank, int W,
                                           const int64_t* __restrict__ epoch, int* status, long long budget,
                                           const int64_t* __restrict__ roots, const int* __restrict__ n_roots,
                                           int rmax, const int* __restrict__ win, const int64_t* __restrict__ ev_eid,
                                           const float* __restrict__ ev_ts, const int* __restrict__ owner,
                                           unsigned long long* const* __restrict__ claim_tables) {
  if (threadIdx.x < 32) peer_wait_warp(my_flags, rank, W, epoch, status, budget);
  __syncthreads();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rmax || r >= *n_roots) return;
  claim_root(r, rmax, roots, win, ev_eid, ev_ts, owner, claim_tables);
}

// Root r's final mail written into the owner's slot when this rank's claim won.
__device__ __forceinline__ void mail_write_root(int r, int rmax, const int64_t* __restrict__ roots,
                                                const int* __restrict__ win, const int* __restrict__ src_idx,
                                                const int* __restrict__ dst_idx, const int64_t* __restrict__ ev_eid,
                                                const float* __restrict__ ev_ts, const float* __restrict__ mem_prev,
                                                int D, const void* __restrict__ efeat, int efeat_bf16, int efeat_ld,
                                                int e_raw, int E, const int* __restrict__ owner,
                                                const unsigned long long* const* __restrict__ claim_tables,
                                                float* const* __restrict__ mail_tables,
                                                float* const* __restrict__ mail_ts_tables) {
  int pass = 0;
  const int i = final_mail_event(win, rmax, r, pass);
  if (i < 0) return;
  const int64_t v = roots[r];
  const int o = owner[v];
  const unsigned long long key = mail_key(ev_ts[i], ev_eid[i]);
  if (claim_tables[o][v] != key) return;  // another rank holds a newer mail for this node
  const int SW = 2 * D + E;
  const int self = pass == 0 ? src_idx[i] : dst_idx[i];
  const int other = pass == 0 ? dst_idx[i] : src_idx[i];
  const int64_t e = ev_eid[i];
  float* slot = mail_tables[o] + v * SW;
  for (int c = threadIdx.x; c < SW; c += blockDim.x) {
    float x;
    if (c < D) x = mem_prev[static_cast<int64_t>(self) * D + c];
    else if (c < 2 * D) x = mem_prev[static_cast<int64_t>(other) * D + (c - D)];
    else {
      const int ce = c - 2 * D;
      x = 0.f;
      if (ce < e_raw) {
        x = efeat_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(efeat)[e * efeat_ld + ce])
                       : static_cast<const float*>(efeat)[e * efeat_ld + ce];
      }
    }
    slot[c] = x;
  }
  if (threadIdx.x == 0) mail_ts_tables[o][v] = ev_ts[i];
}

__global__ void tgn_peer_mail_write_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots,
                                           int rmax, const int* __restrict__ win, const int* __restrict__ src_idx,
                                           const int* __restrict__ dst_idx, const int64_t* __restrict__ ev_eid,
                                           const float* __restrict__ ev_ts, const float* __restrict__ mem_prev, int D,
                                           const void* __restrict__ efeat, int efeat_bf16, int efeat_ld, int e_raw,
                                           int E, const int* __restrict__ owner,
                                           const unsigned long long* const* __restrict__ claim_tables,
                                           float* const* __restrict__ mail_tables,
                                           float* const* __restrict__ mail_ts_tables) {
  const int r = blockIdx.x;
  if (r >= rmax || r >= *n_roots) return;
  mail_write_root(r, rmax, roots, win, src_idx, dst_idx, ev_eid, ev_ts, mem_prev, D, efeat, efeat_bf16, efeat_ld,
                  e_raw, E, owner, claim_tables, mail_tables, mail_ts_tables);
}

// End-of-step push of one root per block: memory write-back (historical
// filter included) and, for the claim winner, the mailbox slot. Blocks loop
// over roots so that the grid need not cover rmax.
__global__ void tgn_peer_push_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                     const float* __restrict__ mem_new, const float* __restrict__ ts_max,
                                     float* const* __restrict__ mem_tables, float* const* __restrict__ ts_tables,
                                     HistCache hc, const int* __restrict__ win, const int* __restrict__ src_idx,
                                     const int* __restrict__ dst_idx, const int64_t* __restrict__ ev_eid,
                                     const float* __restrict__ ev_ts, const float* __restrict__ mem_prev, int D,
                                     const void* __restrict__ efeat, int efeat_bf16, int efeat_ld, int e_raw, int E,
                                     const int* __restrict__ owner,
                                     const unsigned long long* const* __restrict__ claim_tables,
                                     float* const* __restrict__ mail_tables,
                                     float* const* __restrict__ mail_ts_tables) {
  const int n = min(rmax, *n_roots);
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    writeback_root(r, roots, mem_new, D, owner, mem_tables, ts_tables, ts_max, hc);
    if (mail_tables != nullptr)
      mail_write_root(r, rmax, roots, win, src_idx, dst_idx, ev_eid, ev_ts, mem_prev, D, efeat, efeat_bf16,
                      efeat_ld, e_raw, E, owner, claim_tables, mail_tables, mail_ts_tables);
  }
}

void launch_tgn_peer_mail_claim(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const int* win,
                                const int64_t* ev_eid, const float* ev_ts, const int* owner,
                                unsigned long long* const* claim_tables) {
  if (rmax <= 0) return;
  count_launch();
  tgn_peer_mail_claim_kernel<<<(rmax + 127) / 128, 128, 0, st>>>(roots, n_roots, rmax, win, ev_eid, ev_ts, owner,
                                                                  claim_tables);
}

void launch_tgn_peer_mail_write(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const int* win,
                                const int* src_idx, const int* dst_idx, const int64_t* ev_eid, const float* ev_ts,
                                const float* mem_prev, int D, const void* efeat, int efeat_bf16, int efeat_ld,
                                int e_raw, int E, const int* owner, const unsigned long long* const* claim_tables,
                                float* const* mail_tables, float* const* mail_ts_tables) {
  if (rmax <= 0) return;
  count_launch();
  tgn_peer_mail_write_kernel<<<rmax, 128, 0, st>>>(roots, n_roots, rmax, win, src_idx, dst_idx, ev_eid, ev_ts,
                                                   mem_prev, D, efeat, efeat_bf16, efeat_ld, e_raw, E, owner,
                                                   claim_tables, mail_tables, mail_ts_tables);
}

void launch_tgn_peer_wait_claim(cudaStream_t st, const uint64_t* my_flags, int rank, int W, const int64_t* epoch,
                                int* status, long long budget, const int64_t* roots, const int* n_roots, int rmax,
                                const int* win, const int64_t* ev_eid, const float* ev_ts, const int* owner,
                                unsigned long long* const* claim_tables) {
  count_launch();
  const int blocks = rmax > 0 ? (rmax + 127) / 128 : 1;
  tgn_peer_wait_claim_kernel<<<blocks, 128, 0, st>>>(my_flags, rank, W, epoch, status, budget, roots, n_roots, rmax,
                                                      win, ev_eid, ev_ts, owner, claim_tables);
}

void launch_tgn_peer_push(cudaStream_t st, int blocks, const int64_t* roots, const int* n_roots, int rmax,
                          const float* mem_new, const float* ts_max, float* const* mem_tables,
                          float* const* ts_tables, const HistCache& hc, const int* win, const int* src_idx,
                          const int* dst_idx, const int64_t* ev_eid, const float* ev_ts, const float* mem_prev, int D,
                          const void* efeat, int efeat_bf16, int efeat_ld, int e_raw, int E, const int* owner,
                          const unsigned long long* const* claim_tables, float* const* mail_tables,
                          float* const* mail_ts_tables) {
  if (rmax <= 0) return;
  count_launch();
  tgn_peer_push_kernel<<<blocks, 128, 0, st>>>(roots, n_roots, rmax, mem_new, ts_max, mem_tables, ts_tables, hc, win,
                                               src_idx, dst_idx, ev_eid, ev_ts, mem_prev, D, efeat, efeat_bf16,
                                               efeat_ld, e_raw, E, owner, claim_tables, mail_tables, mail_ts_tables);
}

}  // namespace su
