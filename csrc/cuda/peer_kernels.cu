// Kernels that talk to peer GPUs through NVLink / NVSwitch with plain loads,
// stores and atomics on peer memory mapped into this process (symmetric
// allocations): no NCCL call and no TMA on these paths.
//
//  peer_barrier      : device-side barrier over W ranks. Rank r stores the
//                      barrier epoch into slot r of every peer's flag array
//                      (st.release.sys) and waits until all peers' slots in its
//                      own array reach the epoch (ld.acquire.sys). The wait is
//                      bounded: on expiry it records kPeerTimeout and returns.
//  peer_allreduce_adam: gradient all-reduce fused with the Adam update. Every
//                      rank reads the W gradient buffers, sums them in rank
//                      order (bit-identical sums on all ranks), scales and
//                      applies Adam to its own parameter copy.
//  tgn_peer_writeback: new memory rows of this step's roots stored into the
//                      owner rank's memory table; memory_ts = max over writers.
//  tgn_peer_mail_claim/write: one mailbox slot per node (mailbox_slots = 1):
//                      each rank proposes its final mail for each root with the
//                      key (ts, event id); the key is claimed with a 64-bit
//                      atomicMax on the owner; after a barrier the winner
//                      writes the slot into the owner's mailbox.
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
// CTDG memory write-back (block of 64 threads per root, D columns)
//
// Optional historical-cache filter (reference backends/ctdg/runtime/cache.py:
// MemShare-style): a root owned by another rank keeps a cached copy of the last
// row this rank pushed; the new row is pushed only when it was never pushed or
// its cosine distance to the cached row exceeds `thresh` (= 1 - alpha). A pushed
// row refreshes the cache.
// ---------------------------------------------------------------------------
__global__ void tgn_peer_writeback_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                          const float* __restrict__ mem_new, int D, const int* __restrict__ owner,
                                          float* const* __restrict__ mem_tables, float* const* __restrict__ ts_tables,
                                          const float* __restrict__ ts_max, HistCache hc) {
  const int r = blockIdx.x;
  if (r >= rmax || r >= *n_roots) return;
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
      __shared__ float red[3][2];
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
      dot = red[0][0] + red[0][1];
      na = red[1][0] + red[1][1];
      nb = red[2][0] + red[2][1];
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

__global__ void tgn_peer_mail_claim_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots,
                                           int rmax, const int* __restrict__ win, const int64_t* __restrict__ ev_eid,
                                           const float* __restrict__ ev_ts, const int* __restrict__ owner,
                                           unsigned long long* const* __restrict__ claim_tables) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rmax || r >= *n_roots) return;
  int pass = 0;
  const int i = final_mail_event(win, rmax, r, pass);
  if (i < 0) return;
  const int64_t v = roots[r];
  atomicMax(claim_tables[owner[v]] + v, mail_key(ev_ts[i], ev_eid[i]));
}

__global__ void tgn_peer_mail_write_kernel(const int64_t* __restrict__ roots, const int* __restrict__ n_roots,
                                           int rmax, const int* __restrict__ win, const int* __restrict__ src_idx,
                                           const int* __restrict__ dst_idx, const int64_t* __restrict__ ev_eid,
                                           const float* __restrict__ ev_ts, const float* __restrict__ mem_prev, int D,
                                           const float* __restrict__ efeat, int efeat_ld, int e_raw, int E,
                                           const int* __restrict__ owner,
                                           const unsigned long long* const* __restrict__ claim_tables,
                                           float* const* __restrict__ mail_tables,
                                           float* const* __restrict__ mail_ts_tables) {
  const int r = blockIdx.x;
  if (r >= rmax || r >= *n_roots) return;
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
      x = (ce < e_raw) ? efeat[e * efeat_ld + ce] : 0.f;
    }
    slot[c] = x;
  }
  if (threadIdx.x == 0) mail_ts_tables[o][v] = ev_ts[i];
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
                                const float* mem_prev, int D, const float* efeat, int efeat_ld, int e_raw, int E,
                                const int* owner, const unsigned long long* const* claim_tables,
                                float* const* mail_tables, float* const* mail_ts_tables) {
  if (rmax <= 0) return;
  count_launch();
  tgn_peer_mail_write_kernel<<<rmax, 128, 0, st>>>(roots, n_roots, rmax, win, src_idx, dst_idx, ev_eid, ev_ts,
                                                   mem_prev, D, efeat, efeat_ld, e_raw, E, owner, claim_tables,
                                                   mail_tables, mail_ts_tables);
}

}  // namespace su
