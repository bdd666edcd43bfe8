// tcgen05 GEMM over pre-packed bf16 operands.
//
// The operands of the framework's GEMMs are gathers, concatenations and
// on-the-fly time encodings of fp32 tensors (SegSource / WeightSource, see
// tc_gemm.cuh). Building those tiles inside the GEMM leaves 4 producer warps
// per SM latency-bound on dependent gathers. Here the work is split:
//
//   pack_kernel : a full-occupancy grid builds each operand once, as bf16, in
//                 the exact shared-memory tile image the MMA reads (no-swizzle
//                 core matrices; K-major or MN-major), block (tile, k-chunk)
//                 after block, zero-padded to whole tiles.
//   tc_gemm_packed_kernel : warp-specialised tcgen05 GEMM. One thread streams
//                 the blocks into a multi-stage smem ring with bulk async
//                 copies (cp.async.bulk, completion on an mbarrier, no
//                 multicast), one thread issues tcgen05.mma into a TMEM
//                 accumulator, four warps run the fused epilogue.
//
// Every wait is bounded; on expiry the kernel records a status code, waits
// (bounded) for its copies in flight, frees TMEM and returns.
#pragma once

#include <type_traits>
#include <utility>

#include "tc_gemm.cuh"

namespace su {

// warps 0-7 epilogue (warp w reads TMEM lanes 32*(w%4).. and, for epilogues with
// independent columns, column half w/4), warp 8 copy producer, warp 9 MMA + TMEM owner
constexpr int kPackedThreads = 320;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;

template <int BN, int NSUB>
constexpr int packed_stage_bytes() {
  return kBM * kBK * 2 + BN * NSUB * kBK * 2;
}
// ring depth: as many stages as fit (at most 6) next to the barriers, the
// epilogue scratch and the alignment slack, within 224 KB of dynamic smem
template <int BN, int NSUB, int SCRATCH>
constexpr int packed_stages() {
  return (224 * 1024 - 2048 - 2 * SCRATCH) / packed_stage_bytes<BN, NSUB>() >= 6
             ? 6
             : (224 * 1024 - 2048 - 2 * SCRATCH) / packed_stage_bytes<BN, NSUB>();
}
template <int BN, int NSUB, class Epi>
constexpr int packed_smem_bytes() {
  return packed_stages<BN, NSUB, Epi::kScratchBytes>() * packed_stage_bytes<BN, NSUB>() + 1024 /*barriers*/ +
         2 * Epi::kScratchBytes + 1024 /*align*/;
}

#ifdef __CUDACC__
// Epilogues with staging scratch reduce through shared memory with a named
// barrier per 128-thread group; the rest take the plain call.
template <class Epi>
__device__ __forceinline__ void call_epilogue(const Epi& e, int row, bool valid, int n0, uint32_t taddr, int cols,
                                              uint8_t* scratch, int group) {
  if constexpr (Epi::kScratchBytes > 0) {
    e.run(row, valid, n0, taddr, cols, reinterpret_cast<float*>(scratch + group * Epi::kScratchBytes), 1 + group);
  } else {
    e(row, valid, n0, taddr, cols);
  }
}

// Epilogues that read per-row inputs from global memory (the LSTM's c_prev) may
// declare kPrefetch and a prefetch(row, valid, n0, cols) that pulls the rows of
// the CTA's NEXT tile toward L2 while the current tile is waited on and processed.
template <class Epi, class = void>
struct has_prefetch : std::false_type {};
template <class Epi>
struct has_prefetch<Epi, std::void_t<decltype(Epi::kPrefetch)>> : std::integral_constant<bool, Epi::kPrefetch> {};

// Epilogues that issue asynchronous stores (TMA) declare finish(), run by every
// epilogue thread after its last tile, before the CTA's shared memory is released.
template <class Epi, class = void>
struct has_finish : std::false_type {};
template <class Epi>
struct has_finish<Epi, std::void_t<decltype(std::declval<const Epi&>().finish())>> : std::true_type {};
#endif

// K elements per 128-byte chunk row of a packed image: 64 bf16 or 32 tf32
constexpr int chunk_k(bool tf32) { return tf32 ? kBK / 2 : kBK; }

// bytes of a packed operand with `mn` rows (MN extent) and K extent `k`
inline size_t packed_bytes(int mn, int k, int rows_per_tile, bool tf32 = false) {
  const size_t tiles = (static_cast<size_t>(mn) + rows_per_tile - 1) / rows_per_tile;
  const size_t ck = static_cast<size_t>(chunk_k(tf32));
  const size_t chunks = (static_cast<size_t>(k) + ck - 1) / ck;
  return tiles * chunks * static_cast<size_t>(rows_per_tile) * 128;
}

#ifdef __CUDACC__

// One thread = one 16-byte vector (8 bf16) of the packed image.
// Vector index -> (tile t, chunk kc, 8-row group g, k-vector kv, r8):
//   K-major : row = t*ROWS + g*8 + r8, columns [kc*64 + kv*8, +8)
//   MN-major: MN group t*ROWS/8 + g (8 consecutive MN indices), k = kc*64 + kv*8 + r8
// both land at block(t, kc) + g*1024 + kv*128 + r8*16.
// Programmatic dependent launch: a kernel launched with the programmatic-
// serialisation attribute may start while its predecessor drains; it waits
// here before touching anything the predecessor writes. Kernels let their
// dependents start early once their last loads are issued.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

template <int ROWS, class Src>
__device__ __forceinline__ void pack_range(const Src& src, uint8_t* __restrict__ out, int tiles, int nchunks,
                                           int lim, int64_t first, int64_t stride) {
  const int64_t total = static_cast<int64_t>(tiles) * nchunks * (ROWS / 8) * 64;
  for (int64_t idx = first; idx < total; idx += stride) {
    const int r8 = static_cast<int>(idx & 7);
    const int kv = static_cast<int>((idx >> 3) & 7);
    int64_t rest = idx >> 6;
    const int g = static_cast<int>(rest % (ROWS / 8));
    rest /= (ROWS / 8);
    const int kc = static_cast<int>(rest % nchunks);
    const int t = static_cast<int>(rest / nchunks);
    if (t * ROWS >= lim) continue;  // tiles past the (device-side) row count are never read
    float f[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = 0.f;
    if constexpr (!Src::kMN) {
      const int row = t * ROWS + g * 8 + r8;
      if (row < lim) src.load8f(row, kc * (kBK / 8) + kv, lim, f);
    } else {
      const int mng = t * (ROWS / 8) + g;
      if (mng * 8 < lim) src.load8f(mng, kc * kBK + kv * 8 + r8, lim, f);
    }
    *reinterpret_cast<uint4*>(out + (static_cast<int64_t>(t) * nchunks + kc) * (ROWS * 128) + g * 1024 + kv * 128 +
                              r8 * 16) = pack_bf16x8(f);
  }
}

// TF32 images, always K-major: a chunk row holds 32 K values as eight 16-byte
// vectors of four. Row sources: one item = 8 consecutive K of one row (two
// vectors). Transposed (MN-view) sources: one item = 8 consecutive MN x 4
// consecutive K, transposed in registers into eight vectors (the tf32 MMA
// reads both operands K-major).
template <int ROWS, class Src>
__device__ __forceinline__ void pack_range_tf32(const Src& src, uint8_t* __restrict__ out, int tiles, int nchunks,
                                                int lim, int64_t first, int64_t stride) {
  constexpr int CK = chunk_k(true);
  if constexpr (!Src::kMN) {
    const int64_t total = static_cast<int64_t>(tiles) * nchunks * (ROWS / 8) * 32;
    for (int64_t idx = first; idx < total; idx += stride) {
      const int r8 = static_cast<int>(idx & 7);
      const int kv2 = static_cast<int>((idx >> 3) & 3);
      int64_t rest = idx >> 5;
      const int g = static_cast<int>(rest % (ROWS / 8));
      rest /= (ROWS / 8);
      const int kc = static_cast<int>(rest % nchunks);
      const int t = static_cast<int>(rest / nchunks);
      if (t * ROWS >= lim) continue;
      float f[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = 0.f;
      const int row = t * ROWS + g * 8 + r8;
      if (row < lim) src.load8f(row, kc * (CK / 8) + kv2, lim, f);
      uint8_t* base = out + (static_cast<int64_t>(t) * nchunks + kc) * (ROWS * 128) + g * 1024 + r8 * 16;
      *reinterpret_cast<uint4*>(base + (2 * kv2) * 128) = pack_tf32x4(f);
      *reinterpret_cast<uint4*>(base + (2 * kv2 + 1) * 128) = pack_tf32x4(f + 4);
    }
  } else {
    const int64_t total = static_cast<int64_t>(tiles) * nchunks * (ROWS / 8) * 8;
    for (int64_t idx = first; idx < total; idx += stride) {
      const int kq = static_cast<int>(idx & 7);
      int64_t rest = idx >> 3;
      const int g = static_cast<int>(rest % (ROWS / 8));
      rest /= (ROWS / 8);
      const int kc = static_cast<int>(rest % nchunks);
      const int t = static_cast<int>(rest / nchunks);
      if (t * ROWS >= lim) continue;
      float f[4][8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[j][i] = 0.f;
      }
      const int mng = t * (ROWS / 8) + g;
      if (mng * 8 < lim) {
#pragma unroll
        for (int j = 0; j < 4; ++j) src.load8f(mng, kc * CK + kq * 4 + j, lim, f[j]);
      }
      uint8_t* base = out + (static_cast<int64_t>(t) * nchunks + kc) * (ROWS * 128) + g * 1024 + kq * 128;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float v[4] = {f[0][i], f[1][i], f[2][i], f[3][i]};
        *reinterpret_cast<uint4*>(base + i * 16) = pack_tf32x4(v);
      }
    }
  }
}

// Work items of pack_range / pack_range_tf32 for an operand of `tiles` x `nchunks` blocks
template <int ROWS, bool TF32, bool MN>
constexpr int64_t pack_items(int tiles, int nchunks) {
  return static_cast<int64_t>(tiles) * nchunks * (ROWS / 8) * (TF32 ? (MN ? 8 : 32) : 64);
}

template <int ROWS, bool TF32, class Src>
__device__ __forceinline__ void pack_any(const Src& src, uint8_t* __restrict__ out, int tiles, int nchunks, int lim,
                                         int64_t first, int64_t stride) {
  if constexpr (TF32) pack_range_tf32<ROWS>(src, out, tiles, nchunks, lim, first, stride);
  else pack_range<ROWS>(src, out, tiles, nchunks, lim, first, stride);
}

// One thread = one 16-byte vector (8 bf16) of the packed image.
// Vector index -> (tile t, chunk kc, 8-row group g, k-vector kv, r8):
//   K-major : row = t*ROWS + g*8 + r8, columns [kc*64 + kv*8, +8)
//   MN-major: MN group t*ROWS/8 + g (8 consecutive MN indices), k = kc*64 + kv*8 + r8
// both land at block(t, kc) + g*1024 + kv*128 + r8*16.
template <int ROWS, class Src, bool TF32 = false>
__global__ void __launch_bounds__(256) pack_kernel(const __grid_constant__ Src src, uint8_t* __restrict__ out,
                                                   int tiles, int nchunks, int limit, const int* limit_dev,
                                                   int nrows) {
  pdl_wait();
  int lim = limit;
  if (limit_dev != nullptr) lim = min(lim, *limit_dev);
  (void)nrows;
  pack_any<ROWS, TF32>(src, out, tiles, nchunks, lim, static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x,
                       static_cast<int64_t>(gridDim.x) * blockDim.x);
  pdl_launch_dependents();
}

// Both operands of one GEMM in one launch: blocks [0, blocks_a) pack A, the rest pack B.
template <int ROWS_A, class SrcA, int ROWS_B, class SrcB, bool TF32 = false>
__global__ void __launch_bounds__(256) pack2_kernel(const __grid_constant__ SrcA a, const __grid_constant__ SrcB b,
                                                    uint8_t* __restrict__ out_a, uint8_t* __restrict__ out_b,
                                                    int tiles_a, int tiles_b, int nchunks, int lim_a,
                                                    const int* lim_a_dev, int lim_b, int blocks_a) {
  pdl_wait();
  if (static_cast<int>(blockIdx.x) < blocks_a) {
    int lim = lim_a;
    if (lim_a_dev != nullptr) lim = min(lim, *lim_a_dev);
    pack_any<ROWS_A, TF32>(a, out_a, tiles_a, nchunks, lim,
                           static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x,
                           static_cast<int64_t>(blocks_a) * blockDim.x);
  } else {
    const int bb = static_cast<int>(blockIdx.x) - blocks_a;
    const int nb = static_cast<int>(gridDim.x) - blocks_a;
    pack_any<ROWS_B, TF32>(b, out_b, tiles_b, nchunks, lim_b, static_cast<int64_t>(bb) * blockDim.x + threadIdx.x,
                           static_cast<int64_t>(nb) * blockDim.x);
  }
  pdl_launch_dependents();
}

template <int BN, int NSUB, bool AMN, bool BMN, class Epi, bool TF32 = false>
__global__ void __launch_bounds__(kPackedThreads, 1)
    tc_gemm_packed_kernel(const uint8_t* __restrict__ pa, const uint8_t* __restrict__ pb,
                          const __grid_constant__ Epi epi, const GemmShape shape, int* status) {
  static_assert(!TF32 || (!AMN && !BMN), "tf32 operands are packed K-major");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 must be a multiple of 16 in [16, 256]");
  static_assert(NSUB >= 1 && BN * NSUB <= 512, "accumulator exceeds TMEM");
  constexpr int A_BYTES = kBM * kBK * 2;
  constexpr int B_ROWS = BN * NSUB;
  constexpr int B_BYTES = B_ROWS * kBK * 2;
  constexpr int STAGES = packed_stages<BN, NSUB, Epi::kScratchBytes>();
  static_assert(STAGES >= 2, "shared memory too small for a two-stage ring");
  static_assert(packed_smem_bytes<BN, NSUB, Epi>() <= 227 * 1024, "dynamic shared memory above the sm_100 limit");
  // two accumulators when they fit in TMEM: the epilogue of tile i overlaps the MMA of tile i+1
  constexpr int NACC = (2 * B_ROWS <= 512) ? 2 : 1;
  constexpr uint32_t TMEM_COLS = tmem_cols_for(NACC * B_ROWS);
  constexpr uint32_t IDESC = TF32 ? umma_idesc_tf32_f32(kBM, BN)
                                  : (umma_idesc_bf16_f32(kBM, BN) | (AMN ? (1u << 15) : 0u) | (BMN ? (1u << 16) : 0u));
  constexpr int CK = chunk_k(TF32);        // K elements per chunk (128 bytes per row either way)
  constexpr int KSTEP = TF32 ? 8 : 16;     // K per MMA instruction (32 bytes per row either way)

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* smemA = smem;
  uint8_t* smemB = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smemB + STAGES * B_BYTES);
  uint64_t* full = bars;                 // [STAGES] copies landed (1 arrival + tx bytes)
  uint64_t* empty = bars + STAGES;       // [STAGES] MMA done with the stage
  uint64_t* acc_full = bars + 2 * STAGES;  // [NACC]
  uint64_t* acc_empty = acc_full + 2;      // [NACC]
  uint64_t* drain = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* epi_scratch = reinterpret_cast<uint8_t*>(bars) + 1024;  // 2 * Epi::kScratchBytes

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], Epi::kSplitCols ? 256 : 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the prologue above overlapped the pack kernel; its images are complete from here on

  int M = shape.M;
  if (shape.m_dev != nullptr) M = min(M, *shape.m_dev);
  const int tiles_m = (M + kBM - 1) / kBM;
  const int tiles_n = (shape.N + B_ROWS - 1) / B_ROWS;
  const int nchunks = (shape.K + CK - 1) / CK;
  const int ksplit = max(1, shape.ksplit);
  const int cps = (nchunks + ksplit - 1) / ksplit;
  const int total = tiles_m * tiles_n * ksplit;

  if (warp < 8) {
    // ------------------------------ epilogue ------------------------------
    const int q = warp & 3;       // TMEM lane quarter
    const int half = warp >> 2;   // column half (epilogues with independent columns)
    const bool active = Epi::kSplitCols || half == 0;
    int tl = 0;  // tiles with work (the MMA warp counts the same ones)
    for (int tile = blockIdx.x; active && tile < total; tile += gridDim.x) {
      const int mn = tile / ksplit;
      const int nt = mn % tiles_n;
      const int mt = mn / tiles_n;
      const int ks = tile % ksplit;
      if (ks * cps >= nchunks) continue;  // empty split: nothing was accumulated
      const int slot = tl % NACC;
      constexpr int kCols = Epi::kSplitCols ? B_ROWS / 2 : B_ROWS;
      const int c0 = Epi::kSplitCols ? half * kCols : 0;
      if constexpr (has_prefetch<Epi>::value) {
        const int nx = tile + gridDim.x;
        if (nx < total) {
          const int mnx = nx / ksplit;
          const int rowx = (mnx / tiles_n) * kBM + q * 32 + lane;
          epi.prefetch(rowx, rowx < M, (mnx % tiles_n) * B_ROWS + c0, kCols);
        }
      }
      if (!mbar_wait_bounded(&acc_full[slot], (tl / NACC) & 1) || *abort_flag) {
        record_status(status, kTimeoutAccum);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = mt * kBM + q * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(slot * B_ROWS + c0);
      call_epilogue(epi, row, row < M, nt * B_ROWS + c0, taddr, kCols, epi_scratch, half);
      tc_fence_before();
      mbar_arrive(&acc_empty[slot]);
      ++tl;
    }
    if constexpr (has_finish<Epi>::value) {
      if (active) epi.finish();
    }
  } else if (warp == kProducerWarp) {
    // --------------------------- copy producer ----------------------------
    if (lane == 0) {
      int cg = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const int ks = tile % ksplit;
        const int mn = tile / ksplit;
        const int nt = mn % tiles_n;
        const int mt = mn / tiles_n;
        const int kc0 = ks * cps;
        const int kc1 = min(nchunks, kc0 + cps);
        for (int kc = kc0; kc < kc1; ++kc, ++cg) {
          const int s = cg % STAGES;
          const uint32_t ph = (cg / STAGES) & 1;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1) || *abort_flag) {
            record_status(status, kTimeoutEmpty);
            *abort_flag = 1;
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
          bulk_g2s(smemA + s * A_BYTES, pa + (static_cast<size_t>(mt) * nchunks + kc) * A_BYTES, A_BYTES, &full[s]);
          bulk_g2s(smemB + s * B_BYTES, pb + (static_cast<size_t>(nt) * nchunks + kc) * B_BYTES, B_BYTES, &full[s]);
        }
      }
      // copies still in flight complete on their full barriers: wait for the
      // last STAGES issued (bounded) so none targets smem of an exited CTA
      for (int c = max(0, cg - STAGES); c < cg; ++c) {
        if (!mbar_wait_bounded(&full[c % STAGES], (c / STAGES) & 1)) {
          record_status(status, kTimeoutFull);
          break;
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      int cg = 0;
      int tl = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const int ks = tile % ksplit;
        const int kc0 = ks * cps;
        const int kc1 = min(nchunks, kc0 + cps);
        if (kc0 >= kc1) continue;
        const int slot = tl % NACC;
        if (!mbar_wait_bounded(&acc_empty[slot], ((tl / NACC) & 1) ^ 1) || *abort_flag) {
          record_status(status, kTimeoutTmemFree);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem_base + static_cast<uint32_t>(slot * B_ROWS);
        for (int kc = kc0; kc < kc1; ++kc, ++cg) {
          const int s = cg % STAGES;
          const uint32_t ph = (cg / STAGES) & 1;
          if (!mbar_wait_bounded(&full[s], ph) || *abort_flag) {
            record_status(status, kTimeoutFull);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smemA + s * A_BYTES);
          const uint32_t b_base = smem_u32(smemB + s * B_BYTES);
          const int ksteps = min(CK / KSTEP, (shape.K - kc * CK + KSTEP - 1) / KSTEP);
          for (int kk = 0; kk < ksteps; ++kk) {
            const uint64_t adesc = umma_desc_kmajor_noswizzle(a_base + kk * 256, 128, 1024);
#pragma unroll
            for (int sub = 0; sub < NSUB; ++sub) {
              const uint64_t bdesc =
                  umma_desc_kmajor_noswizzle(b_base + sub * (BN / 8) * 1024 + kk * 256, 128, 1024);
              if constexpr (TF32) umma_tf32(acc + sub * BN, adesc, bdesc, IDESC, (kc > kc0 || kk > 0) ? 1u : 0u);
              else umma_bf16(acc + sub * BN, adesc, bdesc, IDESC, (kc > kc0 || kk > 0) ? 1u : 0u);
            }
            issued = true;
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[slot]);
        ++tl;
      }
      if (issued) {  // no tensor-core work may be in flight when TMEM is released
        umma_commit(drain);
        if (!mbar_wait_bounded(drain, 0)) record_status(status, kTimeoutAccum);
      }
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

#endif  // __CUDACC__

}  // namespace su
