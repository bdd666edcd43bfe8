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
  int D = 0, DP = 0;  // DP = gate group width G: tile columns are [r | z | n_i | n_h] x G units
  const float* b_ih = nullptr;   // [3D]
  const float* b_hh = nullptr;   // [3D]
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

#ifdef __CUDACC__
  __device__ __forceinline__ void operator()(int row, bool valid, int n0, uint32_t taddr, int /*tile_cols*/) const {
    const int u0 = (n0 / (4 * DP)) * DP;  // first hidden unit of this tile
    const float* hp = nullptr;
    if (valid && hprev != nullptr) {
      const int64_t hr = hprev_index ? hprev_index[row] : row;
      if (hr >= 0) hp = (hprev_peers ? hprev_peers[hprev_owner[hr]] : hprev) + hr * hprev_ld;
    }
    int64_t srow = -1;
    if (valid && scatter != nullptr) srow = scatter_index[row];
    for (int c0 = 0; c0 < DP; c0 += 16) {
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
        const float rg = sigmoidf_(r[i] + b_ih[c] + b_hh[c]);
        const float zg = sigmoidf_(z[i] + b_ih[D + c] + b_hh[D + c]);
        const float ng = tanhf(ni[i] + b_ih[2 * D + c] + rg * (nh[i] + b_hh[2 * D + c]));
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
    float s1 = 0.f, s2 = 0.f;
    float* xs = xsave + (int64_t)row * Do;
    for (int c0 = 0; c0 < Do; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
      if (!valid) continue;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int c = c0 + i;
        if (c >= Do) break;
        float x = v[i] + bias[c];
        if (drop > 0.f) x = dropout_keep(dseed, (uint64_t)row * Do + c, kStreamOutDrop, drop) ? x / (1.f - drop) : 0.f;
        x = fmaxf(x, 0.f);
        xs[c] = x;
        s1 += x;
        s2 += x * x;
      }
    }
    if (!valid) return;
    if (edge_total != nullptr && *edge_total == 0) {
      float* o = out + (int64_t)row * Do;
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
    float* o = out + (int64_t)row * Do;
    for (int c = 0; c < Do; ++c) o[c] = (xs[c] - mu) * rs * gamma[c] + beta[c];
  }
#endif
};




}  // namespace su

namespace su {

// LSTM cell epilogue (reference runtime/modules/rnn_cells.py:92-116): the accumulator
// holds four blocks of DP columns [x W_i^T + h ... | f | g | o] (one nn.Linear per gate
// over [x || h]). i, f, o = sigmoid, g = tanh, c' = f c + i g, h' = o tanh(c').
// Saves the post-activation gates for the backward pass.
struct EpiLSTM {
  int H = 0, DP = 0;  // DP = gate group width G: tile columns are [i | f | g | o] x G units
  const float* b_i = nullptr;
  const float* b_f = nullptr;
  const float* b_g = nullptr;
  const float* b_o = nullptr;
  const float* c_prev = nullptr;  // [rows, H] (nullptr -> zeros)
  float* h_out = nullptr;         // [rows, H]
  float* c_out = nullptr;         // [rows, H]
  float* gates = nullptr;         // [rows, 4H] (i, f, g, o) post-activation, optional

#ifdef __CUDACC__
  __device__ __forceinline__ void operator()(int row, bool valid, int n0, uint32_t taddr, int /*tc*/) const {
    const int u0 = (n0 / (4 * DP)) * DP;
    for (int c0 = 0; c0 < DP; c0 += 16) {
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
        const float i = sigmoidf_(gi[j] + b_i[c]);
        const float f = sigmoidf_(gf[j] + b_f[c]);
        const float g = tanhf(gg[j] + b_g[c]);
        const float o = sigmoidf_(go[j] + b_o[c]);
        const float cp = c_prev ? c_prev[(int64_t)row * H + c] : 0.f;
        const float cn = f * cp + i * g;
        c_out[(int64_t)row * H + c] = cn;
        h_out[(int64_t)row * H + c] = o * tanhf(cn);
        if (gates) {
          float* gr = gates + (int64_t)row * 4 * H;
          gr[c] = i;
          gr[H + c] = f;
          gr[2 * H + c] = g;
          gr[3 * H + c] = o;
        }
      }
    }
  }
#endif
};

}  // namespace su
