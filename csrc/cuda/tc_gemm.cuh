// Generic tcgen05 (5th-generation tensor core) GEMM for sm_100a with fused
// operand producers and pluggable epilogues.
//
//   D[M, N] = A[M, K] . B[N, K]^T      (bf16 operands, fp32 accumulate in TMEM)
//
// Operands are never materialised in global memory in bf16: producer warps
// evaluate them on the fly from "sources" (gather by index, concatenation of
// column segments, cosine time encoding, peer-GPU shards, transposed views)
// and write them into shared memory in the canonical K-major no-swizzle UMMA
// layout (core matrices of 8 rows x 16 bytes). One elected thread issues
// tcgen05.mma (M = 128, N = BN per instruction, NSUB instructions side by side)
// accumulating into TMEM; tcgen05.commit releases shared-memory stages and
// signals the accumulator. The four producer warps then act as the epilogue:
// each thread owns one TMEM lane (= one output row), reads its accumulator
// columns with tcgen05.ld and applies the epilogue functor (bias, activation,
// recurrent-cell gates, scatter, atomic split-K accumulation, ...).
//
// Warp roles (160 threads):
//   warps 0-3 : operand producers, then epilogue for the same tile
//   warp  4   : TMEM allocator + MMA issuer (lane 0)
//
// Every wait is bounded (common.cuh); on timeout the CTA records a status code,
// drains its in-flight tensor-core work and frees TMEM before returning.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace su {

constexpr int kBM = 128;          // rows per tile (UMMA M)
constexpr int kBK = 64;           // K elements per pipeline stage (4 UMMA k-steps of 16)
constexpr int kStages = 2;
constexpr int kGemmThreads = 160;
constexpr int kMaxSeg = 6;
constexpr int kMaxBlk = 4;

// Byte offset of the 16-byte vector (row r, K-vector kv) inside a stage tile
// laid out as 8-row groups of (kBK / 8) core matrices of 128 bytes each.
#ifdef __CUDACC__
__device__ __forceinline__ uint32_t tile_vec_off(int r, int kv) {
  return static_cast<uint32_t>((r >> 3) * 1024 + kv * 128 + (r & 7) * 16);
}

#endif  // __CUDACC__

#ifdef __CUDACC__
// cos / sin of w * t + b. For large phases (time deltas reach 1e8 s) the phase is
// formed and reduced modulo 2*pi in double precision before the single-precision
// call: exact to fp32 rounding of the reduced phase, and it keeps the trig
// functions on their short-argument path.
__device__ __forceinline__ float reduced_phase(float w, float t, float b) {
  const float x = fmaf(w, t, b);
  if (fabsf(x) < 8192.f) return x;
  const double xd = fma(static_cast<double>(w), static_cast<double>(t), static_cast<double>(b));
  const double two_pi = 6.283185307179586476925286766559;
  const double inv_two_pi = 0.15915494309189533576888376337251;
  return static_cast<float>(fma(-two_pi, rint(xd * inv_two_pi), xd));
}
__device__ __forceinline__ float cos_phase(float w, float t, float b) { return cosf(reduced_phase(w, t, b)); }
__device__ __forceinline__ float sin_phase(float w, float t, float b) { return sinf(reduced_phase(w, t, b)); }
#endif

// ---------------------------------------------------------------------------
// Activation sources: row-wise concatenation of column segments
// ---------------------------------------------------------------------------
enum SegKind : int {
  kSegF32 = 0,      // fp32 matrix rows (optionally gathered through an int64 index)
  kSegBF16 = 1,     // bf16 matrix rows (optionally gathered)
  kSegTime = 2,     // cos(w[c] * t[row] + b[c]) time encoding (t == nullptr -> t = 0)
  kSegOnes = 3,     // a single constant-1 column (bias trick for weight gradients)
  kSegSharded = 4,  // fp32 rows owned by peer GPUs: peers[owner[id]] + lrow[id] * ld
  kSegZero = 5,     // zero padding
  kSegTimeSin = 6,  // -sin(w[c] * t[row] + b[c]), times t[row] when `tmul` (time-encoder gradient terms)
};

struct ASeg {
  int kind = kSegZero;
  int kpad = 0;    // padded width in the K space (multiple of 8)
  int width = 0;   // valid columns
  int ld = 0;      // row stride (elements)
  int col0 = 0;    // first column
  int vec = 0;     // 1 if 16-byte vector loads are legal for this segment
  const void* ptr = nullptr;
  const int64_t* index = nullptr;    // row -> source row (nullptr: identity); < 0 -> zeros
  const float* tdt = nullptr;        // time-encoding input per row
  const float* tw = nullptr;
  const float* tb = nullptr;
  int tmul = 0;                      // kSegTimeSin: multiply by t
  const float* const* peers = nullptr;  // sharded: per-rank base pointers
  const int* owner = nullptr;           // sharded: owning rank per global id
  const int64_t* lrow = nullptr;        // sharded: row inside the owner's shard (nullptr: the global id)
  // sharded, optional: rows of ids stamped in this step (stamp[id] == step tag)
  // are read from the local `fresh` rows at node2root[id] instead of the owner
  const int* stamp = nullptr;
  const int* node2root = nullptr;
  const int64_t* step_ctr = nullptr;    // the step tag is ((*step_ctr - 1) & 0x3FFFFFFF) + 1
  const float* fresh = nullptr;
  int fresh_ld = 0;
  // kSegF32 without index, optional: values kept only where mask[row, col] > 0
  // (the ReLU derivative from the forward output, applied as the operand is packed)
  const float* mask = nullptr;
  int mask_ld = 0;
};

#ifdef __CUDACC__
__device__ __forceinline__ const float* seg_row_f32(const ASeg& g, int row) {
  int64_t r = g.index ? g.index[row] : row;
  if (r < 0) return nullptr;
  if (g.kind == kSegSharded) {
    if (g.stamp != nullptr) {
      const int tag = static_cast<int>(((*g.step_ctr) - 1) & 0x3FFFFFFF) + 1;
      if (g.stamp[r] == tag) return g.fresh + static_cast<int64_t>(g.node2root[r]) * g.fresh_ld + g.col0;
    }
    const int o = g.owner ? g.owner[r] : 0;
    const int64_t lr = g.lrow ? g.lrow[r] : r;
    return g.peers[o] + lr * g.ld + g.col0;
  }
  return static_cast<const float*>(g.ptr) + r * g.ld + g.col0;
}

__device__ __forceinline__ void seg_fill8(const ASeg& g, int row, int c, float (&f)[8]) {
  switch (g.kind) {
    case kSegF32:
    case kSegSharded: {
      const float* p = seg_row_f32(g, row);
      if (p == nullptr) return;
      if (g.vec && c + 8 <= g.width) {
        const float4 a = *reinterpret_cast<const float4*>(p + c);
        const float4 b = *reinterpret_cast<const float4*>(p + c + 4);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
        if (g.mask != nullptr) {
          const float* m = g.mask + static_cast<int64_t>(row) * g.mask_ld + g.col0 + c;
          const float4 ma = *reinterpret_cast<const float4*>(m);
          const float4 mb = *reinterpret_cast<const float4*>(m + 4);
          const float mv[8] = {ma.x, ma.y, ma.z, ma.w, mb.x, mb.y, mb.z, mb.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = mv[i] > 0.f ? f[i] : 0.f;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = (c + i < g.width) ? p[c + i] : 0.f;
        if (g.mask != nullptr) {
          const float* m = g.mask + static_cast<int64_t>(row) * g.mask_ld + g.col0 + c;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (c + i < g.width && !(m[i] > 0.f)) f[i] = 0.f;
        }
      }
      break;
    }
    case kSegBF16: {
      int64_t r = g.index ? g.index[row] : row;
      if (r < 0) return;
      const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(g.ptr) + r * g.ld + g.col0;
      if (g.vec && c + 8 <= g.width) {
        const uint4 w = *reinterpret_cast<const uint4*>(p + c);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          f[2 * i] = __uint_as_float(ws[i] << 16);
          f[2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = (c + i < g.width) ? __bfloat162float(p[c + i]) : 0.f;
      }
      break;
    }
    case kSegTime: {
      const float t = g.tdt ? g.tdt[row] : 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = (c + i < g.width) ? cos_phase(g.tw[c + i], t, g.tb[c + i]) : 0.f;
      break;
    }
    case kSegTimeSin: {
      const float t = g.tdt ? g.tdt[row] : 0.f;
      const float m = g.tmul ? -t : -1.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = (c + i < g.width) ? m * sin_phase(g.tw[c + i], t, g.tb[c + i]) : 0.f;
      break;
    }
    case kSegOnes:
      if (c == 0) f[0] = 1.f;
      break;
    default:
      break;
  }
}

__device__ __forceinline__ float seg_load1(const ASeg& g, int row, int c) {
  if (c >= g.width) return 0.f;
  switch (g.kind) {
    case kSegF32:
    case kSegSharded: {
      const float* p = seg_row_f32(g, row);
      if (p == nullptr) return 0.f;
      if (g.mask != nullptr && !(g.mask[static_cast<int64_t>(row) * g.mask_ld + g.col0 + c] > 0.f)) return 0.f;
      return p[c];
    }
    case kSegBF16: {
      int64_t r = g.index ? g.index[row] : row;
      if (r < 0) return 0.f;
      return __bfloat162float(static_cast<const __nv_bfloat16*>(g.ptr)[r * g.ld + g.col0 + c]);
    }
    case kSegTime: {
      const float t = g.tdt ? g.tdt[row] : 0.f;
      return cos_phase(g.tw[c], t, g.tb[c]);
    }
    case kSegTimeSin: {
      const float t = g.tdt ? g.tdt[row] : 0.f;
      return (g.tmul ? -t : -1.f) * sin_phase(g.tw[c], t, g.tb[c]);
    }
    case kSegOnes:
      return c == 0 ? 1.f : 0.f;
    default:
      return 0.f;
  }
}

#endif  // __CUDACC__

struct SegSource {
  static constexpr bool kMN = false;
  ASeg seg[kMaxSeg];
  int nseg = 0;
  int group = 1;                 // rows come in groups (edges of one root) ...
  const int* gcount = nullptr;   // ... of which only the first gcount[g] are valid
  const int* nrows_dev = nullptr;  // optional device-side row count

#ifdef __CUDACC__
  __device__ __forceinline__ bool row_valid(int row, int nrows) const {
    if (row >= nrows) return false;
    if (nrows_dev != nullptr && row >= *nrows_dev) return false;
    if (gcount != nullptr && (row % group) >= gcount[row / group]) return false;
    return true;
  }
#endif
  // 8 consecutive K elements [kv*8, kv*8+8) of row `row`.
#ifdef __CUDACC__
  __device__ __forceinline__ void load8f(int row, int kv, int nrows, float (&f)[8]) const {
    if (row_valid(row, nrows)) {
      int k = kv * 8;
#pragma unroll
      for (int s = 0; s < kMaxSeg; ++s) {
        if (s >= nseg) break;
        if (k < seg[s].kpad) {
          seg_fill8(seg[s], row, k, f);
          break;
        }
        k -= seg[s].kpad;
      }
    }
  }
#endif
#ifdef __CUDACC__
  __device__ __forceinline__ float load1(int row, int k, int nrows) const {
    if (!row_valid(row, nrows)) return 0.f;
#pragma unroll
    for (int s = 0; s < kMaxSeg; ++s) {
      if (s >= nseg) break;
      if (k < seg[s].kpad) return seg_load1(seg[s], row, k);
      k -= seg[s].kpad;
    }
    return 0.f;
  }
#endif
};

// MN-major view of a row source: the GEMM operand's MN index runs along the
// inner source's K space and the GEMM's K index along the inner rows, i.e.
// operand(mn, k) = inner(row = k, col = mn). The producer loads 8 consecutive mn
// of one k (one 16-byte vector of the inner row) and the tile is consumed with
// the MN-major bit of the instruction descriptor, so weight gradients
// (reduction over samples) and data gradients (W^T) need no transposition.
template <class Inner>
struct MNView {
  static constexpr bool kMN = true;
  Inner inner;
  int inner_rows = 0;  // static bound of the inner rows (the GEMM K extent)
#ifdef __CUDACC__
  __device__ __forceinline__ void load8f(int mn_group, int k, int /*nrows*/, float (&f)[8]) const {
    inner.load8f(k, mn_group, inner_rows, f);
  }
#endif
};

// An A operand whose packed image was written by an earlier kernel of the caller
// in the layout of pack_range (tc_gemm_packed.cuh) (K-major when !MN, MN-major when MN), zero
// padded to whole tiles and chunks. The GEMM then packs B only.
template <bool MN>
struct Prepacked {
  static constexpr bool kMN = MN;
  const uint8_t* image = nullptr;
};
template <class T>
struct is_prepacked : std::false_type {};
template <bool MN>
struct is_prepacked<Prepacked<MN>> : std::true_type {};

// ---------------------------------------------------------------------------
// Weight sources: rows = concatenated output blocks, K = concatenated input
// segments; each (block, segment) cell maps to an fp32 nn.Linear weight
// region or to zeros. Weights are read in fp32 and rounded to bf16 on the fly.
// ---------------------------------------------------------------------------
struct WCell {
  const float* ptr = nullptr;  // nullptr -> zero block
  int ld = 0;
  int row0 = 0;
  int col0 = 0;
  int width = 0;
  int vec = 0;                 // 16-byte loads legal (ld, col0 multiples of 4, aligned base)
};

struct WeightLayout {
  int nblk = 0, nseg = 0;
  int blk_rows[kMaxBlk] = {0, 0, 0, 0};  // valid rows of each output block
  int blk_pad[kMaxBlk] = {0, 0, 0, 0};   // padded rows of each output block
  int seg_kpad[kMaxSeg] = {0, 0, 0, 0, 0, 0};  // padded K width of each input segment
  WCell cell[kMaxBlk][kMaxSeg];

#ifdef __CUDACC__
  __device__ __forceinline__ bool find_blk(int n, int& b, int& r) const {
#pragma unroll
    for (int i = 0; i < kMaxBlk; ++i) {
      if (i >= nblk) break;
      if (n < blk_pad[i]) {
        b = i;
        r = n;
        return r < blk_rows[i];
      }
      n -= blk_pad[i];
    }
    return false;
  }
#endif
#ifdef __CUDACC__
  __device__ __forceinline__ bool find_seg(int k, int& s, int& c) const {
#pragma unroll
    for (int i = 0; i < kMaxSeg; ++i) {
      if (i >= nseg) break;
      if (k < seg_kpad[i]) {
        s = i;
        c = k;
        return true;
      }
      k -= seg_kpad[i];
    }
    return false;
  }
#endif
};

// B[n, k] = W[n, k] (forward projection; n = output feature). MNView<WeightSource>
// gives W^T (data gradients).
struct WeightSource {
  static constexpr bool kMN = false;
  WeightLayout L;
  // gate_group > 0: rows are interleaved by gate in groups of gate_group units, so an
  // N tile of 4 * gate_group rows holds all four gates of the same hidden units
  // (recurrent-cell epilogues then need only one tile per unit group).
  int gate_group = 0;
#ifdef __CUDACC__
  __device__ __forceinline__ bool map_row(int row, int& b, int& r) const {
    if (gate_group > 0) {
      const int t = row / (L.nblk * gate_group), w = row % (L.nblk * gate_group);
      b = w / gate_group;
      r = t * gate_group + w % gate_group;
      return r < L.blk_rows[b];
    }
    return L.find_blk(row, b, r);
  }
  __device__ __forceinline__ void load8f(int row, int kv, int /*nrows*/, float (&f)[8]) const {
    int b, r, s, c;
    if (map_row(row, b, r) && L.find_seg(kv * 8, s, c)) {
      const WCell& e = L.cell[b][s];
      if (e.ptr != nullptr) {
        const float* p = e.ptr + (int64_t)(e.row0 + r) * e.ld + e.col0;
        if (e.vec && c + 8 <= e.width) {
          const float4 a = *reinterpret_cast<const float4*>(p + c);
          const float4 b = *reinterpret_cast<const float4*>(p + c + 4);
          f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
          f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = (c + i < e.width) ? p[c + i] : 0.f;
        }
      }
    }
  }
#endif
};

// ---------------------------------------------------------------------------
// Generic epilogues
// ---------------------------------------------------------------------------
enum Act : int { kActNone = 0, kActRelu = 1, kActSigmoid = 2, kActTanh = 3 };

#ifdef __CUDACC__
__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
    case kActRelu: return fmaxf(v, 0.f);
    case kActSigmoid: return sigmoidf_(v);
    case kActTanh: return tanhf(v);
    default: return v;
  }
}

template <int ACT>
__device__ __forceinline__ float act_ct(float v) {
  if constexpr (ACT == kActRelu) return fmaxf(v, 0.f);
  else if constexpr (ACT == kActSigmoid) return sigmoidf_(v);
  else if constexpr (ACT == kActTanh) return tanhf(v);
  else return v;
}

// Bias of 4 consecutive columns [col, col + 4) of a linear epilogue with an
// optional second bias from column `split` on (split % 4 == 0, both 16-byte aligned).
__device__ __forceinline__ float4 bias4(const float* b, const float* b2, int split, int col) {
  const float* p = col < split ? (b ? b + col : nullptr) : (b2 ? b2 + (col - split) : nullptr);
  return p ? __ldg(reinterpret_cast<const float4*>(p)) : make_float4(0.f, 0.f, 0.f, 0.f);
}
#endif  // __CUDACC__

// out[row, col] (=|+=) act(scale * acc + bias[col]); optional row scatter.
struct EpiLinear {
  static constexpr bool kSplitCols = true;  // columns are independent: two warps may share a row
  static constexpr int kScratchBytes = 0;
  float* out = nullptr;
  __nv_bfloat16* out_bf16 = nullptr;
  int ldo = 0;
  int ncols = 0;         // valid output columns
  const float* bias = nullptr;
  const float* bias2 = nullptr;  // bias of the columns >= bias_split (two fused projections)
  int bias_split = 1 << 30;
  int act = kActNone;
  float scale = 1.f;
  int accumulate = 0;    // 1: out += value (non-atomic), 2: atomicAdd
  const int64_t* scatter = nullptr;  // row -> output row

#ifdef __CUDACC__
  // Per batch of up to 64 columns: every TMEM load and the columns' bias (the same
  // for every row: broadcast loads) are in flight together before one wait.
  // Plain fp32 stores of whole 16-column groups run a loop specialised on the
  // activation (a warp-uniform switch outside it); a runtime activation switch or
  // a bias load inside the per-element loop costs several times the stores
  // themselves. Everything else (scatter rows, accumulation, bf16 copies, ragged
  // column groups) takes the generic per-element path.
  __device__ __forceinline__ bool vec_bias_ok() const {
    return (bias == nullptr || (reinterpret_cast<uintptr_t>(bias) & 15) == 0) &&
           (bias2 == nullptr || ((reinterpret_cast<uintptr_t>(bias2) & 15) == 0 && (bias_split & 3) == 0));
  }
  template <int ACT>
  __device__ __forceinline__ void store16(float* o, const uint32_t* r, const float4* b) const {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      reinterpret_cast<float4*>(o)[j] =
          make_float4(act_ct<ACT>(fmaf(scale, __uint_as_float(r[4 * j]), b[j].x)),
                      act_ct<ACT>(fmaf(scale, __uint_as_float(r[4 * j + 1]), b[j].y)),
                      act_ct<ACT>(fmaf(scale, __uint_as_float(r[4 * j + 2]), b[j].z)),
                      act_ct<ACT>(fmaf(scale, __uint_as_float(r[4 * j + 3]), b[j].w)));
    }
  }
  template <int ACT>
  __device__ __forceinline__ void store_groups(float* o, int groups, const uint32_t (&r)[64],
                                               const float4 (&b)[16]) const {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (k < groups) store16<ACT>(o + 16 * k, r + 16 * k, b + 4 * k);
  }
  struct Vals16 {
    float v[16];
  };
  // Generic per-element stores of up to 16 columns from col0 (scatter rows,
  // accumulation, bf16 copies, ragged groups). Out of line: inlined once per
  // column group, its runtime activation switch made the epilogue's code large
  // enough to slow every tile.
  __device__ __noinline__ void store_generic(int64_t orow, int col0, int n, Vals16 x) const {
    for (int i = 0; i < n; ++i) {
      const int col = col0 + i;
      const float bv = col < bias_split ? (bias ? bias[col] : 0.f) : (bias2 ? bias2[col - bias_split] : 0.f);
      const float y = apply_act(scale * x.v[i] + bv, act);
      if (out != nullptr) {
        float* o = out + orow * ldo + col;
        if (accumulate == 2) atomicAdd(o, y);
        else if (accumulate == 1) *o += y;
        else *o = y;
      }
      if (out_bf16) out_bf16[orow * ldo + col] = __float2bfloat16(y);
    }
  }
  __device__ __forceinline__ void operator()(int row, bool valid, int n0, uint32_t taddr, int tile_cols) const {
    int64_t orow = row;
    if (valid && scatter != nullptr) {
      orow = scatter[row];
      if (orow < 0) valid = false;
    }
    const int lim = min(ncols - n0, tile_cols);
    const bool vec_ok = out != nullptr && accumulate == 0 && out_bf16 == nullptr && (ldo & 3) == 0 &&
                        (reinterpret_cast<uintptr_t>(out) & 15) == 0 && (n0 & 3) == 0 && vec_bias_ok();
    for (int b0 = 0; b0 < lim; b0 += 64) {
      const int cols = min(64, lim - b0);
      const int groups = vec_ok ? cols / 16 : 0;  // whole 16-column groups on the vector path
      uint32_t r[64];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (16 * k < cols) {  // warp-uniform
          uint32_t (&rk)[16] = *reinterpret_cast<uint32_t (*)[16]>(r + 16 * k);
          tmem_ld16_issue(taddr + b0 + 16 * k, rk);
        }
      }
      float4 b[16];
#pragma unroll
      for (int q = 0; q < 16; ++q)
        b[q] = (q < 4 * groups && valid) ? bias4(bias, bias2, bias_split, n0 + b0 + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
      tmem_wait_ld_all(r);
      if (!valid) continue;
      if (groups > 0) {
        float* o = out + orow * ldo + n0 + b0;
        switch (act) {
          case kActRelu: store_groups<kActRelu>(o, groups, r, b); break;
          case kActSigmoid: store_groups<kActSigmoid>(o, groups, r, b); break;
          case kActTanh: store_groups<kActTanh>(o, groups, r, b); break;
          default: store_groups<kActNone>(o, groups, r, b); break;
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (16 * k >= cols || k < groups) continue;  // warp-uniform
        Vals16 x;
#pragma unroll
        for (int i = 0; i < 16; ++i) x.v[i] = __uint_as_float(r[16 * k + i]);
        store_generic(orow, n0 + b0 + 16 * k, min(16, cols - 16 * k), x);
      }
    }
  }
#endif
};

// Plain fp32 stores of EpiLinear (no scatter, no accumulation) for large row
// counts: each epilogue warp moves its 32 rows x 32 columns from TMEM into a
// 128-byte-swizzled shared-memory box (conflict-free 16-byte stores) and one
// lane writes the box out with a tiled TMA store. A warp's plain per-row stores
// touch 32 cache lines per instruction; the TMA store writes whole lines. Two
// boxes per warp alternate, so the TMEM loads of chunk k+1 overlap the store of
// chunk k. Rows past M and columns past ncols are clipped by the tensor map.
struct EpiLinearTma {
  static constexpr bool kSplitCols = true;
  static constexpr int kBoxBytes = 32 * 32 * 4;  // 32 rows x 128 bytes
  // per 4-warp column half: 4 warps x 2 boxes, then one 1 KB line of per-warp box counters
  static constexpr int kScratchBytes = 4 * 2 * kBoxBytes + 1024;
  alignas(64) CUtensorMap tmap;  // [M rows, ncols] fp32, row stride ldo, box 32 x 32, 128-byte swizzle
  int ncols = 0;
  const float* bias = nullptr;
  const float* bias2 = nullptr;
  int bias_split = 1 << 30;
  int act = kActNone;
  float scale = 1.f;

#ifdef __CUDACC__
  template <int ACT>
  __device__ __forceinline__ void stage(uint8_t* box, int lane, const uint32_t (&r)[32], const float4 (&b)[8]) const {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // 128-byte swizzle: 16-byte chunk j of row `lane` sits at chunk j ^ (lane % 8)
      *reinterpret_cast<float4*>(box + lane * 128 + ((j ^ (lane & 7)) << 4)) =
          make_float4(act_ct<ACT>(fmaf(scale, __uint_as_float(r[4 * j]), b[j].x)),
                      act_ct<ACT>(fmaf(scale, __uint_as_float(r[4 * j + 1]), b[j].y)),
                      act_ct<ACT>(fmaf(scale, __uint_as_float(r[4 * j + 2]), b[j].z)),
                      act_ct<ACT>(fmaf(scale, __uint_as_float(r[4 * j + 3]), b[j].w)));
    }
  }
  __device__ __forceinline__ void run(int row, bool /*valid*/, int n0, uint32_t taddr, int tile_cols, float* scratch,
                                      int /*barrier*/) const {
    const int lane = threadIdx.x & 31;
    const int wq = (threadIdx.x >> 5) & 3;
    uint8_t* base = reinterpret_cast<uint8_t*>(scratch);
    uint8_t* boxes = base + wq * 2 * kBoxBytes;  // 1024-byte aligned (the swizzle pattern's period)
    volatile int* counter = reinterpret_cast<volatile int*>(base + 4 * 2 * kBoxBytes) + wq;
    const int row0 = row - lane;  // first row of this warp's 32
    const int lim = min(ncols - n0, tile_cols);
    int k = *counter;  // boxes written so far by this warp (any start value works: only its parity is used)
    for (int c0 = 0; c0 < lim; c0 += 32, ++k) {
      uint8_t* box = boxes + (k & 1) * kBoxBytes;
      uint32_t r[32];
      {
        uint32_t (&r0)[16] = *reinterpret_cast<uint32_t (*)[16]>(r);
        uint32_t (&r1)[16] = *reinterpret_cast<uint32_t (*)[16]>(r + 16);
        tmem_ld16_issue(taddr + c0, r0);
        tmem_ld16_issue(taddr + c0 + 16, r1);
      }
      float4 b[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int col = n0 + c0 + 4 * q;
        if (col + 4 <= ncols) {
          b[q] = bias4(bias, bias2, bias_split, col);
        } else {  // ragged last quad: columns past ncols are clipped by the store
          float t[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int cu = col + u;
            t[u] = cu >= ncols ? 0.f : cu < bias_split ? (bias ? bias[cu] : 0.f) : (bias2 ? bias2[cu - bias_split] : 0.f);
          }
          b[q] = make_float4(t[0], t[1], t[2], t[3]);
        }
      }
      tmem_wait_ld_all(r);
      // the store issued from this box two chunks ago must have finished reading it
      if (lane == 0) bulk_wait_group_read<1>();
      __syncwarp();
      switch (act) {
        case kActRelu: stage<kActRelu>(box, lane, r, b); break;
        case kActSigmoid: stage<kActSigmoid>(box, lane, r, b); break;
        case kActTanh: stage<kActTanh>(box, lane, r, b); break;
        default: stage<kActNone>(box, lane, r, b); break;
      }
      fence_proxy_async_smem();  // generic-proxy writes visible to the TMA engine
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&tmap, box, n0 + c0, row0);
        bulk_commit_group();
      }
    }
    __syncwarp();
    if (lane == 0) *counter = k;
    __syncwarp();
  }
  // after the last tile: this warp's stores complete before the CTA (and its shared memory) goes away
  __device__ __forceinline__ void finish() const {
    if ((threadIdx.x & 31) == 0) bulk_wait_group<0>();
    __syncwarp();
  }
#endif
};

// Weight gradient accumulation: rows = output features (blocks of the layout),
// columns = padded input K space (segments). Segment kinds flagged as bias
// accumulate into the bias gradient of the block.
struct EpiWeightGrad {
  static constexpr bool kSplitCols = true;
  static constexpr int kScratchBytes = 0;
  WeightLayout L;                 // cell ptrs point at gradient buffers
  float* bias_grad[kMaxBlk] = {nullptr, nullptr, nullptr, nullptr};
  int bias_seg = -1;              // segment index carrying the ones column
  int ncols = 0;                  // total K space width of the inner source

#ifdef __CUDACC__
  __device__ __forceinline__ void operator()(int row, bool valid, int n0, uint32_t taddr, int tile_cols) const {
    int b = 0, r = 0;
    if (valid) valid = L.find_blk(row, b, r);
    const int lim = min(ncols - n0, tile_cols);
    for (int c0 = 0; c0 < lim; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
      if (!valid) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // four columns of one cell: one 16-byte vector reduction instead of four atomics
        // (segments start at multiples of 8, so an aligned quad never straddles one)
        {
          const int n = n0 + c0 + 4 * j;
          int s, c;
          if (L.find_seg(n, s, c) && s != bias_seg) {
            const WCell& e = L.cell[b][s];
            if (e.vec && e.ptr != nullptr && (c & 3) == 0 && c + 4 <= e.width) {
              float* dst = const_cast<float*>(e.ptr) + (int64_t)(e.row0 + r) * e.ld + e.col0 + c;
              asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(dst), "f"(v[4 * j]),
                           "f"(v[4 * j + 1]), "f"(v[4 * j + 2]), "f"(v[4 * j + 3])
                           : "memory");
              continue;
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = 4 * j + u;
          const int n = n0 + c0 + i;
          int s, c;
          if (!L.find_seg(n, s, c)) continue;
          if (s == bias_seg) {
            if (c == 0 && bias_grad[b] != nullptr) atomicAdd(bias_grad[b] + r, v[i]);
            continue;
          }
          const WCell& e = L.cell[b][s];
          if (e.ptr != nullptr && c < e.width)
            atomicAdd(const_cast<float*>(e.ptr) + (int64_t)(e.row0 + r) * e.ld + e.col0 + c, v[i]);
        }
      }
    }
  }
#endif
};

struct GemmShape {
  int M = 0;                  // static row bound (grid sizing)
  const int* m_dev = nullptr; // optional device row count (<= M)
  int N = 0;                  // columns of D (rows of B)
  int K = 0;                  // reduction extent
  int ksplit = 1;             // split-K factor (epilogue must accumulate atomically)
  int tf32 = 0;               // 1: fp32 operands read as TF32 (kind::tf32), else bf16 operands (kind::f16)
};

constexpr int tmem_cols_for(int n) {
  return n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : n <= 256 ? 256 : 512;
}

template <int BN, int NSUB>
constexpr int gemm_smem_bytes() {
  return kStages * (kBM * kBK * 2 + BN * NSUB * kBK * 2) + 1024 /*barriers*/ + 1024 /*align slack*/;
}

#ifdef __CUDACC__
// Fill one stage tile of ROWS operand rows x kBK K elements. K-major sources give
// 8 consecutive K of one row per 16-byte vector; MN-major sources give 8
// consecutive MN of one K. Both canonical layouts use 128-byte core matrices,
// LBO = 128 (K direction) and SBO = 1024 (MN direction).
template <int ROWS, class Src>
__device__ __forceinline__ void produce_tile(const Src& src, uint8_t* tile, int mn0, int kc, int nrows, int limit) {
  // All global loads of a batch are issued before any conversion so that the
  // producer keeps many requests in flight (memory-level parallelism).
  if constexpr (!Src::kMN) {
    for (int r = threadIdx.x; r < ROWS; r += 128) {
      const int row = mn0 + r;
      float f[kBK / 8][8];
#pragma unroll
      for (int kv = 0; kv < kBK / 8; ++kv) {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[kv][i] = 0.f;
        if (row < limit) src.load8f(row, kc * (kBK / 8) + kv, nrows, f[kv]);
      }
#pragma unroll
      for (int kv = 0; kv < kBK / 8; ++kv)
        *reinterpret_cast<uint4*>(tile + tile_vec_off(r, kv)) = pack_bf16x8(f[kv]);
    }
  } else {
    const int k = threadIdx.x & (kBK - 1);
    const uint32_t koff = static_cast<uint32_t>((k >> 3) * 128 + (k & 7) * 16);
    constexpr int G = ROWS / 8;          // MN groups in the tile
    constexpr int STEP = 128 / kBK;      // threads per K index
    constexpr int BATCH = 8;
    for (int g0 = threadIdx.x / kBK; g0 < G; g0 += STEP * BATCH) {
      float f[BATCH][8];
#pragma unroll
      for (int j = 0; j < BATCH; ++j) {
        const int g = g0 + j * STEP;
#pragma unroll
        for (int i = 0; i < 8; ++i) f[j][i] = 0.f;
        if (g < G && mn0 + g * 8 < limit) src.load8f((mn0 >> 3) + g, kc * kBK + k, nrows, f[j]);
      }
#pragma unroll
      for (int j = 0; j < BATCH; ++j) {
        const int g = g0 + j * STEP;
        if (g < G) *reinterpret_cast<uint4*>(tile + g * 1024 + koff) = pack_bf16x8(f[j]);
      }
    }
  }
}

template <int BN, int NSUB, class ASrc, class BSrc, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    tc_gemm_kernel(const __grid_constant__ ASrc asrc, const __grid_constant__ BSrc bsrc,
                   const __grid_constant__ Epi epi, const GemmShape shape, int* status) {
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 must be a multiple of 16 in [16, 256]");
  static_assert(NSUB >= 1 && BN * NSUB <= 512, "accumulator exceeds TMEM");
  constexpr int A_BYTES = kBM * kBK * 2;
  constexpr int B_ROWS = BN * NSUB;
  constexpr int B_BYTES = B_ROWS * kBK * 2;
  constexpr uint32_t TMEM_COLS = tmem_cols_for(B_ROWS);
  constexpr uint32_t IDESC = umma_idesc_bf16_f32(kBM, BN) | (ASrc::kMN ? (1u << 15) : 0u) |
                             (BSrc::kMN ? (1u << 16) : 0u);

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* smemA = smem;
  uint8_t* smemB = smem + kStages * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smemB + kStages * B_BYTES);
  uint64_t* full = bars;                  // [kStages] producers -> MMA
  uint64_t* empty = bars + kStages;       // [kStages] MMA -> producers
  uint64_t* acc_full = bars + 2 * kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  int M = shape.M;
  if (shape.m_dev != nullptr) M = min(M, *shape.m_dev);
  const int tiles_m = (M + kBM - 1) / kBM;
  const int tiles_n = (shape.N + B_ROWS - 1) / B_ROWS;
  const int nchunks = (shape.K + kBK - 1) / kBK;
  const int ksplit = max(1, shape.ksplit);
  const int cps = (nchunks + ksplit - 1) / ksplit;
  const int total = tiles_m * tiles_n * ksplit;

  if (warp < 4) {
    // ------------------------- producers + epilogue -------------------------
    int cg = 0;
    int tl = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++tl) {
      const int ks = tile % ksplit;
      const int mn = tile / ksplit;
      const int nt = mn % tiles_n;
      const int mt = mn / tiles_n;
      const int kc0 = ks * cps;
      const int kc1 = min(nchunks, kc0 + cps);
      for (int kc = kc0; kc < kc1; ++kc, ++cg) {
        const int s = cg % kStages;
        const uint32_t ph = (cg / kStages) & 1;
        if (!mbar_wait_bounded(&empty[s], ph ^ 1) || *abort_flag) {
          record_status(status, kTimeoutEmpty);
          *abort_flag = 1;
          ok = false;
          break;
        }
        uint8_t* a = smemA + s * A_BYTES;
        uint8_t* b = smemB + s * B_BYTES;
        produce_tile<kBM>(asrc, a, mt * kBM, kc, M, M);
        produce_tile<B_ROWS>(bsrc, b, nt * B_ROWS, kc, shape.N, shape.N);
        fence_proxy_async_smem();
        mbar_arrive(&full[s]);
      }
      if (!ok) break;
      // epilogue for this tile
      if (!mbar_wait_bounded(acc_full, tl & 1) || *abort_flag) {
        record_status(status, kTimeoutAccum);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = mt * kBM + warp * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
      epi(row, row < M, nt * B_ROWS, taddr, B_ROWS);
      tc_fence_before();
      mbar_arrive(acc_empty);
    }
  } else {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      int cg = 0;
      int tl = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++tl) {
        const int ks = tile % ksplit;
        const int kc0 = ks * cps;
        const int kc1 = min(nchunks, kc0 + cps);
        if (!mbar_wait_bounded(acc_empty, (tl & 1) ^ 1) || *abort_flag) {
          record_status(status, kTimeoutTmemFree);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        for (int kc = kc0; kc < kc1; ++kc, ++cg) {
          const int s = cg % kStages;
          const uint32_t ph = (cg / kStages) & 1;
          if (!mbar_wait_bounded(&full[s], ph) || *abort_flag) {
            record_status(status, kTimeoutFull);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smemA + s * A_BYTES);
          const uint32_t b_base = smem_u32(smemB + s * B_BYTES);
          const int ksteps = min(kBK / 16, (shape.K - kc * kBK + 15) / 16);
          for (int kk = 0; kk < ksteps; ++kk) {
            const uint64_t adesc = umma_desc_kmajor_noswizzle(a_base + kk * 256, 128, 1024);
#pragma unroll
            for (int sub = 0; sub < NSUB; ++sub) {
              const uint64_t bdesc = umma_desc_kmajor_noswizzle(b_base + sub * (BN / 8) * 1024 + kk * 256, 128, 1024);
              umma_bf16(tmem_base + sub * BN, adesc, bdesc, IDESC, (kc > kc0 || kk > 0) ? 1u : 0u);
            }
            issued = true;
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(acc_full);
      }
      // make sure no tensor-core work is in flight before TMEM is released
      if (issued) {
        umma_commit(drain);
        if (!mbar_wait_bounded(drain, 0)) record_status(status, kTimeoutAccum);
      }
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

#endif  // __CUDACC__

}  // namespace su
