// Model-specific GEMM epilogues (TGN memory updater, output projection with
// LayerNorm, time-encoder gradient). Data members are host-visible so the
// torch-side wrappers can fill them; device code is compiled by nvcc only.
#pragma once

#include "tc_gemm.cuh"

namespace su {

constexpr uint32_t kStreamAttDrop = 0xA77D0u;
constexpr uint32_t kStreamOutDrop = 0x0D7D0u;

// ---------------------------------------------------------------------------
// GRU gates epilogue. Accumulator columns hold four blocks of DP columns:
//   [ x W_ir^T + h W_hr^T | x W_iz^T + h W_hz^T | x W_in^T | h W_hn^T ]
// (PyTorch GRU gate convention). Produces h' = (1 - z) * n + z * h.
// ---------------------------------------------------------------------------
struct EpiGRU {
  // a unit's four gate columns must meet in one thread: with gate groups of 16
  // units, each half of a 128-column tile holds whole groups, so two warps split it
  static constexpr bool kSplitCols = true;
  static constexpr int kScratchBytes = 0;
  int D = 0, DP = 0;  // DP = gate group width G: tile columns are [r | z | n_i | n_h] x G units
  int ngates = 4;     // 4: GRU cell; 1: tanh RNN cell h' = tanh(W_ih x + b_ih + W_hh h + b_hh) (JODIE)
  const float* b_ih = nullptr;   // [3D] (RNN: [D])
  const float* b_hh = nullptr;   // [3D] (RNN: [D])
  const float* hprev = nullptr;  // previous hidden rows (nullptr -> zeros)
  const int64_t* hprev_index = nullptr;
  int hprev_ld = 0;
  const float* const* hprev_peers = nullptr;  // optional: hprev rows live in the owner rank's table
  const int* hprev_owner = nullptr;
  float* hout = nullptr;         // dense output rows (optional)
  int hout_ld = 0;
  float* save_prev = nullptr;    // copy of the previous hidden rows (optional)
  float* scatter = nullptr;      // memory table written at rows scatter_index[row] (optional)
  const int64_t* scatter_index = nullptr;
  int scatter_ld = 0;
  float* scatter_ts = nullptr;   // memory_ts[scatter_index[row]] = *ts_value
  const float* ts_value = nullptr;
  // 1: D, hprev_ld, hout_ld and scatter_ld are multiples of 4 and every pointer
  // (peer tables included) is 16-byte aligned: 16-byte loads and stores
  int vec = 0;

#ifdef __CUDACC__
  // every gate group of ngates*DP columns in the range this thread was given
  __device__ __forceinline__ void operator()(int row, bool valid, int n0, uint32_t taddr, int tile_cols) const {
    for (int g0 = 0; g0 < tile_cols; g0 += ngates * DP) group(row, valid, n0 + g0, taddr + g0);
  }
  __device__ __forceinline__ void group(int row, bool valid, int n0, uint32_t taddr) const {
    const int u0 = (n0 / (ngates * DP)) * DP;  // first hidden unit of this group
    const float* hp = nullptr;
    if (valid && hprev != nullptr) {
      const int64_t hr = hprev_index ? hprev_index[row] : row;
      if (hr >= 0) hp = (hprev_peers ? hprev_peers[hprev_owner[hr]] : hprev) + hr * hprev_ld;
    }
    int64_t srow = -1;
    if (valid && scatter != nullptr) srow = scatter_index[row];
    if (ngates == 1) {
      for (int c0 = 0; c0 < DP; c0 += 16) {
        const int cb = u0 + c0;
        if (vec && cb + 16 <= D) {
          uint32_t rp[16];
          tmem_ld16_issue(taddr + c0, rp);
          float4 h4[4], b4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            h4[q] = (hp && save_prev) ? *reinterpret_cast<const float4*>(hp + cb + 4 * q)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 a = ldg4(b_ih + cb + 4 * q), b = ldg4(b_hh + cb + 4 * q);
            b4[q] = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
          }
          tmem_wait_ld4(rp, rp, rp, rp);
          if (!valid) continue;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 o4 = make_float4(tanh_fast(__uint_as_float(rp[4 * q]) + b4[q].x),
                                          tanh_fast(__uint_as_float(rp[4 * q + 1]) + b4[q].y),
                                          tanh_fast(__uint_as_float(rp[4 * q + 2]) + b4[q].z),
                                          tanh_fast(__uint_as_float(rp[4 * q + 3]) + b4[q].w));
            if (save_prev) *reinterpret_cast<float4*>(save_prev + (int64_t)row * D + cb + 4 * q) = h4[q];
            if (hout) *reinterpret_cast<float4*>(hout + (int64_t)row * hout_ld + cb + 4 * q) = o4;
            if (srow >= 0) *reinterpret_cast<float4*>(scatter + srow * scatter_ld + cb + 4 * q) = o4;
          }
          continue;
        }
        float pre[16];
        tmem_ld16(taddr + c0, pre);
        if (!valid) continue;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c = u0 + c0 + i;
          if (c >= D) break;
          const float h = hp ? hp[c] : 0.f;
          const float hn = tanh_fast(pre[i] + b_ih[c] + b_hh[c]);
          if (save_prev) save_prev[(int64_t)row * D + c] = h;
          if (hout) hout[(int64_t)row * hout_ld + c] = hn;
          if (srow >= 0) scatter[srow * scatter_ld + c] = hn;
        }
      }
      if (valid && srow >= 0 && scatter_ts != nullptr && u0 == 0) scatter_ts[srow] = *ts_value;
      return;
    }
    for (int c0 = 0; c0 < DP; c0 += 16) {
      const int cb = u0 + c0;
      if (vec && cb + 16 <= D) {
        // whole group of 16 units (warp-uniform branch): the previous hidden rows of
        // all 16 are in flight before the first TMEM load, and every load precedes
        // every store (a row may be read from and written to the same table); the
        // gates come in two halves of 8 units
        float4 h4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          h4[q] = hp ? *reinterpret_cast<const float4*>(hp + cb + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 o4[4];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t rr[8], rz[8], rni[8], rnh[8];
          tmem_ld8_issue(taddr + c0 + 8 * hh, rr);
          tmem_ld8_issue(taddr + DP + c0 + 8 * hh, rz);
          tmem_ld8_issue(taddr + 2 * DP + c0 + 8 * hh, rni);
          tmem_ld8_issue(taddr + 3 * DP + c0 + 8 * hh, rnh);
          tmem_wait_ld4n<8>(rr, rz, rni, rnh);
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            const int q = 2 * hh + qq;
            const int cq = cb + 4 * q;
            const float4 a = ldg4(b_ih + cq), b = ldg4(b_hh + cq);
            const float4 c = ldg4(b_ih + D + cq), d = ldg4(b_hh + D + cq);
            const float4 e = ldg4(b_ih + 2 * D + cq), f = ldg4(b_hh + 2 * D + cq);
            const float br[4] = {a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w};
            const float bz[4] = {c.x + d.x, c.y + d.y, c.z + d.z, c.w + d.w};
            const float bni[4] = {e.x, e.y, e.z, e.w}, bnh[4] = {f.x, f.y, f.z, f.w};
            const float hv[4] = {h4[q].x, h4[q].y, h4[q].z, h4[q].w};
            float hn[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int i = 4 * qq + u;
              const float rg = sigmoid_fast(__uint_as_float(rr[i]) + br[u]);
              const float zg = sigmoid_fast(__uint_as_float(rz[i]) + bz[u]);
              const float ng = tanh_fast(__uint_as_float(rni[i]) + bni[u] + rg * (__uint_as_float(rnh[i]) + bnh[u]));
              hn[u] = (1.f - zg) * ng + zg * hv[u];
            }
            o4[q] = make_float4(hn[0], hn[1], hn[2], hn[3]);
          }
        }
        if (!valid) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (save_prev) *reinterpret_cast<float4*>(save_prev + (int64_t)row * D + cb + 4 * q) = h4[q];
          if (hout) *reinterpret_cast<float4*>(hout + (int64_t)row * hout_ld + cb + 4 * q) = o4[q];
          if (srow >= 0) *reinterpret_cast<float4*>(scatter + srow * scatter_ld + cb + 4 * q) = o4[q];
        }
        continue;
      }
      float r[16], z[16], ni[16], nh[16];
      tmem_ld16(taddr + c0, r);
      tmem_ld16(taddr + DP + c0, z);
      tmem_ld16(taddr + 2 * DP + c0, ni);
      tmem_ld16(taddr + 3 * DP + c0, nh);
      if (!valid) continue;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int c = u0 + c0 + i;
        if (c >= D) break;
        const float h = hp ? hp[c] : 0.f;
        const float rg = sigmoid_fast(r[i] + b_ih[c] + b_hh[c]);
        const float zg = sigmoid_fast(z[i] + b_ih[D + c] + b_hh[D + c]);
        const float ng = tanh_fast(ni[i] + b_ih[2 * D + c] + rg * (nh[i] + b_hh[2 * D + c]));
        const float hn = (1.f - zg) * ng + zg * h;
        if (save_prev) save_prev[(int64_t)row * D + c] = h;
        if (hout) hout[(int64_t)row * hout_ld + c] = hn;
        if (srow >= 0) scatter[srow * scatter_ld + c] = hn;
      }
    }
    if (valid && srow >= 0 && scatter_ts != nullptr && u0 == 0) scatter_ts[srow] = *ts_value;
  }
#endif
};


// ---------------------------------------------------------------------------
// output projection epilogue: dropout -> ReLU -> LayerNorm (row owned by thread)
// ---------------------------------------------------------------------------
struct EpiOutLN {
  static constexpr bool kSplitCols = false;  // LayerNorm needs the whole row
  static constexpr int kScratchBytes = 0;
  int Do = 0;
  const float* bias = nullptr;
  const float* gamma = nullptr;
  const float* beta = nullptr;
  float drop = 0.f;
  uint64_t seed = 0;
  const int64_t* step_ctr = nullptr;
  const int* edge_total = nullptr;  // no sampled edge in the whole block -> zero output
  float* out = nullptr;    // [rows, Do]
  float* xsave = nullptr;  // post-ReLU pre-LN activations [rows, Do]
  float* mean = nullptr;   // [rows]
  float* rstd = nullptr;   // [rows]

#ifdef __CUDACC__
  __device__ __forceinline__ void operator()(int row, bool valid, int /*n0*/, uint32_t taddr, int /*tile_cols*/) const {
    const uint64_t dseed = seed ^ (static_cast<uint64_t>(*step_ctr) * 0x9E3779B97F4A7C15ull);
    const float inv_keep = drop > 0.f ? 1.f / (1.f - drop) : 1.f;
    float s1 = 0.f, s2 = 0.f;
    float* xs = xsave + (int64_t)row * Do;
    float* o = out + (int64_t)row * Do;
    // 4-column groups: one Philox call and one 16-byte store each (Do % 4 == 0 keeps
    // every row 16-byte aligned); a ragged tail goes element by element
    const bool vec = (Do & 3) == 0 && (reinterpret_cast<uintptr_t>(xsave) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    for (int c0 = 0; c0 < Do; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
      if (!valid) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = c0 + 4 * j;
        if (c >= Do) break;
        if (vec) {
          bool k[4];
          dropout_keep4(dseed, (uint64_t)row * Do + c, kStreamOutDrop, drop, k);
          float x[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float t = (v[4 * j + u] + bias[c + u]) * inv_keep;
            x[u] = k[u] ? fmaxf(t, 0.f) : 0.f;
            s1 += x[u];
            s2 += x[u] * x[u];
          }
          *reinterpret_cast<float4*>(xs + c) = make_float4(x[0], x[1], x[2], x[3]);
        } else {
          for (int u = 0; u < 4 && c + u < Do; ++u) {
            float x = v[4 * j + u] + bias[c + u];
            if (drop > 0.f)
              x = dropout_keep(dseed, (uint64_t)row * Do + c + u, kStreamOutDrop, drop) ? x * inv_keep : 0.f;
            x = fmaxf(x, 0.f);
            xs[c + u] = x;
            s1 += x;
            s2 += x * x;
          }
        }
      }
    }
    if (!valid) return;
    if (edge_total != nullptr && *edge_total == 0) {
      for (int c = 0; c < Do; ++c) o[c] = 0.f;
      mean[row] = 0.f;
      rstd[row] = 0.f;
      return;
    }
    const float mu = s1 / Do;
    const float var = fmaxf(s2 / Do - mu * mu, 0.f);
    const float rs = rsqrtf(var + 1e-5f);
    mean[row] = mu;
    rstd[row] = rs;
    if (vec) {
      for (int c = 0; c < Do; c += 4) {
        const float4 x = *reinterpret_cast<const float4*>(xs + c);
        *reinterpret_cast<float4*>(o + c) =
            make_float4((x.x - mu) * rs * gamma[c] + beta[c], (x.y - mu) * rs * gamma[c + 1] + beta[c + 1],
                        (x.z - mu) * rs * gamma[c + 2] + beta[c + 2], (x.w - mu) * rs * gamma[c + 3] + beta[c + 3]);
      }
    } else {
      for (int c = 0; c < Do; ++c) o[c] = (xs[c] - mu) * rs * gamma[c] + beta[c];
    }
  }
#endif
};




}  // namespace su

namespace su {

// LSTM cell epilogue (reference runtime/modules/rnn_cells.py:92-116): the accumulator
// holds four blocks of DP columns [x W_i^T + h ... | f | g | o] (one nn.Linear per gate
// over [x || h]). i, f, o = sigmoid, g = tanh, c' = f c + i g, h' = o tanh(c').
// Saves the post-activation gates for the backward pass in the tile's own order:
// per row, per group of 16 units, [i(16) f(16) g(16) o(16)]
//   gates[row * 64 * ceil(H/16) + (u / 16) * 64 + gate * 16 + u % 16],
// so a row's group is 256 contiguous bytes.
constexpr int kLstmGroup = 16;
__host__ __device__ inline int64_t lstm_gate_index(int64_t row, int H, int gate, int u) {
  const int groups = (H + kLstmGroup - 1) / kLstmGroup;
  return row * 64 * groups + (u / kLstmGroup) * 64 + gate * kLstmGroup + u % kLstmGroup;
}

struct EpiLSTM {
  static constexpr bool kSplitCols = true;  // gate groups of 16 units (see EpiGRU)
  // staging rows for the coalesced stores of the packed kernel: per warp 32 rows x
  // [i f g o c' h'] x 16 units, row stride padded to 100 floats (conflict-free
  // 16-byte accesses); per 4-warp column half
  static constexpr int kStageStride = 100;
  static constexpr int kScratchBytes = 4 * 32 * kStageStride * 4;
  int H = 0, DP = 0;  // DP = gate group width (16): tile columns are [i | f | g | o] x 16 units
  const float* b_i = nullptr;
  const float* b_f = nullptr;
  const float* b_g = nullptr;
  const float* b_o = nullptr;
  const float* c_prev = nullptr;  // [rows, H] (nullptr -> zeros)
  float* h_out = nullptr;         // [rows, H]
  float* c_out = nullptr;         // [rows, H]
  float* gates = nullptr;         // grouped layout above, optional
  int vec = 0;  // 1: H % 4 == 0 and every pointer 16-byte aligned (16-byte loads and stores)
  static constexpr bool kPrefetch = true;
  // TMA stores (packed kernel, whole 16-unit groups): per warp and group the 32
  // rows' [i f | g o] gates go out as two 32 x 32 fp32 boxes (128-byte swizzle)
  // and c', h' as 16 x 32 boxes (64-byte swizzle) from a 12 KB shared-memory region
  int tma = 0;
  alignas(64) CUtensorMap map_g;  // gates [rows, 64 * H / 16], box 32 x 32
  alignas(64) CUtensorMap map_c;  // c_out [rows, H], box 16 x 32
  alignas(64) CUtensorMap map_h;  // h_out [rows, H], box 16 x 32
  static constexpr int kTmaRegion = 12 * 1024;

#ifdef __CUDACC__
  // c_prev of the next tile's rows toward L2 (one 64-byte segment per group)
  __device__ __forceinline__ void prefetch(int row, bool valid, int n0, int tile_cols) const {
    if (!valid || c_prev == nullptr) return;
    for (int g0 = 0; g0 < tile_cols; g0 += 4 * DP) {
      const int u0 = ((n0 + g0) / (4 * DP)) * DP;
      if (u0 < H) asm volatile("prefetch.global.L2 [%0];" ::"l"(c_prev + (int64_t)row * H + u0));
    }
  }
  // fused-producer kernel: every gate group of 4*DP columns in the range, direct stores
  __device__ __forceinline__ void operator()(int row, bool valid, int n0, uint32_t taddr, int tile_cols) const {
#pragma unroll 1
    for (int g0 = 0; g0 < tile_cols; g0 += 4 * DP) group(row, valid, n0 + g0, taddr + g0, nullptr);
  }
  // packed kernel: whole groups are staged in this warp's rows of `scratch`
  // and written out row-contiguously (4 full cache lines per gate store
  // instruction instead of 32 partial ones)
  __device__ __forceinline__ void run(int row, bool valid, int n0, uint32_t taddr, int tile_cols, float* scratch,
                                      int /*barrier*/) const {
    if (tma) {
      uint8_t* reg = reinterpret_cast<uint8_t*>(scratch) + ((threadIdx.x >> 5) & 3) * kTmaRegion;
#pragma unroll 1
      for (int g0 = 0; g0 < tile_cols; g0 += 4 * DP) group_tma(row, valid, n0 + g0, taddr + g0, reg);
      return;
    }
    float* ws = scratch + ((threadIdx.x >> 5) & 3) * 32 * kStageStride;
#pragma unroll 1
    for (int g0 = 0; g0 < tile_cols; g0 += 4 * DP) group(row, valid, n0 + g0, taddr + g0, ws);
  }
  __device__ __forceinline__ void finish() const {
    if (tma && (threadIdx.x & 31) == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  // One 16-unit group (DP == 16, H % 16 == 0) through TMA stores. The region is
  // 1024-byte aligned: [gates i f | gates g o | c' | h'] at 0, 4 KB, 8 KB, 10 KB.
  // Rows past the matrix are clipped by the tensor maps.
  __device__ __forceinline__ void group_tma(int row, bool valid, int n0, uint32_t taddr, uint8_t* reg) const {
    const int lane = threadIdx.x & 31;
    const int cb = (n0 / (4 * DP)) * DP;  // first unit of the group
    if (cb >= H) return;                  // warp-uniform
    const int64_t rb = (int64_t)row * H + cb;
    float4 cp4[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      cp4[q] = (valid && c_prev) ? ldg4(c_prev + rb + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
    // the previous group's boxes must have been read out by the TMA engine
    if (lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
    const int s128 = lane & 7;         // 128-byte swizzle: chunk j of a 128-byte row at j ^ (row % 8)
    const int s64 = (lane >> 1) & 3;   // 64-byte swizzle: chunk j of a 64-byte row at j ^ ((row / 2) % 4)
    compute16(taddr, 0, cb, valid, cp4, [&](int q, float4 i4, float4 f4, float4 g4, float4 o4, float4 c4, float4 h4) {
      *reinterpret_cast<float4*>(reg + lane * 128 + ((q ^ s128) << 4)) = i4;
      *reinterpret_cast<float4*>(reg + lane * 128 + (((4 + q) ^ s128) << 4)) = f4;
      *reinterpret_cast<float4*>(reg + 4096 + lane * 128 + ((q ^ s128) << 4)) = g4;
      *reinterpret_cast<float4*>(reg + 4096 + lane * 128 + (((4 + q) ^ s128) << 4)) = o4;
      *reinterpret_cast<float4*>(reg + 8192 + lane * 64 + ((q ^ s64) << 4)) = c4;
      *reinterpret_cast<float4*>(reg + 10240 + lane * 64 + ((q ^ s64) << 4)) = h4;
    });
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      const int gx = (cb / kLstmGroup) * 64;  // the group's first column in the gates matrix
      if (gates) {
        tma_store_2d(&map_g, reg, gx, row);
        tma_store_2d(&map_g, reg + 4096, gx + 32, row);
      }
      tma_store_2d(&map_c, reg + 8192, cb, row);
      tma_store_2d(&map_h, reg + 10240, cb, row);
      bulk_commit_group();
    }
  }

  // 16 units: activations and state update for units [cb, cb + 16) of `row`
  // (c_prev already loaded), handed to `put(q, i4, f4, g4, o4, c4, h4)` per 4-unit block
  template <class Put>
  __device__ __forceinline__ void compute16(uint32_t taddr, int c0, int cb, bool valid, const float4 (&cp4)[4],
                                            Put&& put) const {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      uint32_t ri[8], rf[8], rg[8], ro[8];
      tmem_ld8_issue(taddr + c0 + 8 * hh, ri);
      tmem_ld8_issue(taddr + DP + c0 + 8 * hh, rf);
      tmem_ld8_issue(taddr + 2 * DP + c0 + 8 * hh, rg);
      tmem_ld8_issue(taddr + 3 * DP + c0 + 8 * hh, ro);
      tmem_wait_ld4n<8>(ri, rf, rg, ro);
      if (!valid) continue;
#pragma unroll
      for (int qq = 0; qq < 2; ++qq) {
        const int q = 2 * hh + qq;  // 4-unit block inside the group
        // biases: warp-uniform addresses, L1-resident after the first tile
        const float4 bi4 = ldg4(b_i + cb + 4 * q), bf4 = ldg4(b_f + cb + 4 * q);
        const float4 bg4 = ldg4(b_g + cb + 4 * q), bo4 = ldg4(b_o + cb + 4 * q);
        const float cpv[4] = {cp4[q].x, cp4[q].y, cp4[q].z, cp4[q].w};
        const float bi[4] = {bi4.x, bi4.y, bi4.z, bi4.w}, bf[4] = {bf4.x, bf4.y, bf4.z, bf4.w};
        const float bg[4] = {bg4.x, bg4.y, bg4.z, bg4.w}, bo[4] = {bo4.x, bo4.y, bo4.z, bo4.w};
        float iv[4], fv[4], gv[4], ov[4], cn[4], hn[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = 4 * qq + u;
          iv[u] = sigmoid_fast(__uint_as_float(ri[j]) + bi[u]);
          fv[u] = sigmoid_fast(__uint_as_float(rf[j]) + bf[u]);
          gv[u] = tanh_fast(__uint_as_float(rg[j]) + bg[u]);
          ov[u] = sigmoid_fast(__uint_as_float(ro[j]) + bo[u]);
          cn[u] = fv[u] * cpv[u] + iv[u] * gv[u];
          hn[u] = ov[u] * tanh_fast(cn[u]);
        }
        put(q, make_float4(iv[0], iv[1], iv[2], iv[3]), make_float4(fv[0], fv[1], fv[2], fv[3]),
            make_float4(gv[0], gv[1], gv[2], gv[3]), make_float4(ov[0], ov[1], ov[2], ov[3]),
            make_float4(cn[0], cn[1], cn[2], cn[3]), make_float4(hn[0], hn[1], hn[2], hn[3]));
      }
    }
  }

  __device__ __forceinline__ void group(int row, bool valid, int n0, uint32_t taddr, float* ws) const {
    const int u0 = (n0 / (4 * DP)) * DP;
    const int lane = threadIdx.x & 31;
#pragma unroll 1
    for (int c0 = 0; c0 < DP; c0 += 16) {
      const int cb = u0 + c0;
      if (vec && cb + 16 <= H) {
        // whole group of 16 units (warp-uniform branch): the previous cell state of
        // all 16 is in flight before the first TMEM load; the gates come in two
        // halves of 8 units (fewer live registers than one pass of 16)
        const int64_t rb = (int64_t)row * H + cb;
        float4 cp4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          cp4[q] = (valid && c_prev) ? ldg4(c_prev + rb + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (ws == nullptr) {
          float* gr = gates ? gates + lstm_gate_index(row, H, 0, cb) : nullptr;
          compute16(taddr, c0, cb, valid, cp4,
                    [&](int q, float4 i4, float4 f4, float4 g4, float4 o4, float4 c4, float4 h4) {
                      *reinterpret_cast<float4*>(c_out + rb + 4 * q) = c4;
                      *reinterpret_cast<float4*>(h_out + rb + 4 * q) = h4;
                      if (gr) {
                        *reinterpret_cast<float4*>(gr + 4 * q) = i4;
                        *reinterpret_cast<float4*>(gr + 16 + 4 * q) = f4;
                        *reinterpret_cast<float4*>(gr + 32 + 4 * q) = g4;
                        *reinterpret_cast<float4*>(gr + 48 + 4 * q) = o4;
                      }
                    });
          continue;
        }
        float* mine = ws + lane * kStageStride;
        compute16(taddr, c0, cb, valid, cp4,
                  [&](int q, float4 i4, float4 f4, float4 g4, float4 o4, float4 c4, float4 h4) {
                    *reinterpret_cast<float4*>(mine + 4 * q) = i4;
                    *reinterpret_cast<float4*>(mine + 16 + 4 * q) = f4;
                    *reinterpret_cast<float4*>(mine + 32 + 4 * q) = g4;
                    *reinterpret_cast<float4*>(mine + 48 + 4 * q) = o4;
                    *reinterpret_cast<float4*>(mine + 64 + 4 * q) = c4;
                    *reinterpret_cast<float4*>(mine + 80 + 4 * q) = h4;
                  });
        __syncwarp();
        // rows row0 .. row0 + nvalid - 1 of this warp are inside the matrix
        const int64_t row0 = row - lane;
        const int nvalid = __popc(__ballot_sync(0xffffffffu, valid));
        if (gates) {
          // 32 rows x 16 float4: two rows (2 x 256 contiguous bytes) per instruction
          float* gbase = gates + lstm_gate_index(row0, H, 0, cb);
          const int64_t gstride = 64 * ((H + kLstmGroup - 1) / kLstmGroup);
#pragma unroll 4
          for (int k = 0; k < 16; ++k) {
            const int idx = k * 32 + lane, r = idx >> 4, j = idx & 15;
            if (r < nvalid)
              *reinterpret_cast<float4*>(gbase + r * gstride + 4 * j) =
                  *reinterpret_cast<const float4*>(ws + r * kStageStride + 4 * j);
          }
        }
        // c' and h': 32 rows x 4 float4 each, eight rows (64 bytes each) per instruction
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int idx = k * 32 + lane, r = idx >> 2, j = idx & 3;
          if (r < nvalid) {
            const int64_t o = (row0 + r) * H + cb + 4 * j;
            *reinterpret_cast<float4*>(c_out + o) = *reinterpret_cast<const float4*>(ws + r * kStageStride + 64 + 4 * j);
            *reinterpret_cast<float4*>(h_out + o) = *reinterpret_cast<const float4*>(ws + r * kStageStride + 80 + 4 * j);
          }
        }
        __syncwarp();
        continue;
      }
      float gi[16], gf[16], gg[16], go[16];
      tmem_ld16(taddr + c0, gi);
      tmem_ld16(taddr + DP + c0, gf);
      tmem_ld16(taddr + 2 * DP + c0, gg);
      tmem_ld16(taddr + 3 * DP + c0, go);
      if (!valid) continue;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = u0 + c0 + j;
        if (c >= H) break;
        const float i = sigmoid_fast(gi[j] + b_i[c]);
        const float f = sigmoid_fast(gf[j] + b_f[c]);
        const float g = tanh_fast(gg[j] + b_g[c]);
        const float o = sigmoid_fast(go[j] + b_o[c]);
        const float cp = c_prev ? c_prev[(int64_t)row * H + c] : 0.f;
        const float cn = f * cp + i * g;
        c_out[(int64_t)row * H + c] = cn;
        h_out[(int64_t)row * H + c] = o * tanh_fast(cn);
        if (gates) {
          gates[lstm_gate_index(row, H, 0, c)] = i;
          gates[lstm_gate_index(row, H, 1, c)] = f;
          gates[lstm_gate_index(row, H, 2, c)] = g;
          gates[lstm_gate_index(row, H, 3, c)] = o;
        }
      }
    }
  }
#endif
};



// ---------------------------------------------------------------------------
// Reset-gated GRU cell, the recurrence of T-GCN (reference
// backends/dtdg/runtime/models.py:166-178) and of EvolveGCN's MatGRU
// (runtime/modules/rnn_cells.py:38-53):
//   z = sigmoid(W_z [x_z | h] + b_z), r = sigmoid(W_r [x_r | h] + b_r),
//   c = tanh(W_c [x_c | r * h] + b_c), h' = z * h + (1 - z) * c.
// Two GEMMs: the first produces z and r (columns interleaved in groups of 16
// units, [z | r] x 16, so one thread sees both gates of a unit) and writes z, r
// and r * h; the second produces c and writes c and h'.
// ---------------------------------------------------------------------------
constexpr int kRGruGroup = 16;

struct EpiRGruZR {
  static constexpr bool kSplitCols = true;
  static constexpr int kScratchBytes = 0;
  int H = 0;
  const float* bz = nullptr;
  const float* br = nullptr;
  const float* h = nullptr;  // [rows, h_ld] previous state (nullptr -> zeros)
  int h_ld = 0;
  float* z_out = nullptr;    // [rows, H]
  float* r_out = nullptr;    // [rows, H]
  float* rh_out = nullptr;   // [rows, H]: r * h, the second GEMM's input

#ifdef __CUDACC__
  __device__ __forceinline__ void operator()(int row, bool valid, int n0, uint32_t taddr, int tile_cols) const {
#pragma unroll 1
    for (int g0 = 0; g0 < tile_cols; g0 += 2 * kRGruGroup) {
      const int u0 = ((n0 + g0) / (2 * kRGruGroup)) * kRGruGroup;
      float zv[16], rv[16];
      tmem_ld16(taddr + g0, zv);
      tmem_ld16(taddr + g0 + kRGruGroup, rv);
      if (!valid || u0 >= H) continue;
      float hv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) hv[j] = (h != nullptr && u0 + j < H) ? h[(int64_t)row * h_ld + u0 + j] : 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = u0 + j;
        if (c >= H) break;
        const float z = sigmoidf_(zv[j] + bz[c]);
        const float r = sigmoidf_(rv[j] + br[c]);
        const int64_t o = (int64_t)row * H + c;
        z_out[o] = z;
        r_out[o] = r;
        rh_out[o] = r * hv[j];
      }
    }
  }
#endif
};

struct EpiRGruOut {
  static constexpr bool kSplitCols = true;
  static constexpr int kScratchBytes = 0;
  int H = 0;
  const float* bc = nullptr;
  const float* z = nullptr;  // [rows, H] from the first GEMM
  const float* h = nullptr;  // [rows, h_ld] (nullptr -> zeros)
  int h_ld = 0;
  float* c_out = nullptr;    // [rows, H]
  float* h_out = nullptr;    // [rows, H]

#ifdef __CUDACC__
  __device__ __forceinline__ void operator()(int row, bool valid, int n0, uint32_t taddr, int tile_cols) const {
    const int lim = min(H - n0, tile_cols);
    for (int c0 = 0; c0 < lim; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
      if (!valid) continue;
      float zv[16], hv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = n0 + c0 + j;
        zv[j] = c < H ? z[(int64_t)row * H + c] : 0.f;
        hv[j] = (h != nullptr && c < H) ? h[(int64_t)row * h_ld + c] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = n0 + c0 + j;
        if (c >= H) break;
        const float cv = tanhf(v[j] + bc[c]);
        const int64_t o = (int64_t)row * H + c;
        c_out[o] = cv;
        h_out[o] = zv[j] * hv[j] + (1.f - zv[j]) * cv;
      }
    }
  }
#endif
};

}  // namespace su
