// Torch-side wrappers of the DTDG kernels: CSR SpMM, fused LSTM cell (tcgen05
// GEMM with a gate epilogue) and its backward (elementwise gate gradients, then
// input and weight gradients on the tcgen05 GEMM).
#include "host_common.h"

using namespace su;

at::Tensor spmm_csr(const at::Tensor& rowptr, const at::Tensor& col, const at::Tensor& val, const at::Tensor& x,
                    int64_t n_rows, const c10::optional<at::Tensor>& out_opt, bool accumulate) {
  SU_CHECK_I64(rowptr); SU_CHECK_I32(col); SU_CHECK_F32(val); SU_CHECK_F32(x); SU_CHECK_CONTIG(x);
  const int F = static_cast<int>(x.size(1));
  at::Tensor out = (out_opt.has_value() && out_opt->defined()) ? *out_opt : at::empty({n_rows, F}, x.options());
  TORCH_CHECK(out.is_contiguous() && out.size(1) == F, "bad output buffer");
  if (accumulate == false && n_rows > 0 && rowptr.numel() == n_rows + 1) {
    // every row is written by the kernel
  }
  launch_spmm_csr(cur_stream(), rowptr.data_ptr<int64_t>(), col.data_ptr<int>(), val.data_ptr<float>(),
                  x.data_ptr<float>(), n_rows, F, out.data_ptr<float>(), accumulate ? 1 : 0);
  SU_LAUNCH_CHECK();
  return out;
}

static WeightLayout lstm_layout(const std::vector<at::Tensor>& ws, int in_dim, int H, int DP) {
  WeightLayout L;
  L.nblk = 4;
  L.nseg = 2;
  L.seg_kpad[0] = pad8(in_dim);
  L.seg_kpad[1] = pad8(H);
  for (int i = 0; i < 4; ++i) {
    L.blk_rows[i] = H;
    L.blk_pad[i] = DP;
    L.cell[i][0] = wcell(ws[i], 0, 0, in_dim);
    L.cell[i][1] = wcell(ws[i], 0, in_dim, H);
  }
  return L;
}

// (h', c', gates) = LSTMCell(x, (h, c)); gates: post-activation (i, f, g, o) in groups of
// 16 units per row (lstm_gate_index)
std::vector<at::Tensor> lstm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& h,
                                 const c10::optional<at::Tensor>& c, const at::Tensor& wi, const at::Tensor& bi,
                                 const at::Tensor& wf, const at::Tensor& bf, const at::Tensor& wg,
                                 const at::Tensor& bg, const at::Tensor& wo, const at::Tensor& bo, bool save_gates) {
  SU_CHECK_F32(x); SU_CHECK_CONTIG(x);
  const int rows = static_cast<int>(x.size(0));
  const int in_dim = static_cast<int>(x.size(1));
  const int H = static_cast<int>(wi.size(0));
  constexpr int G = 16;  // gate group: each 64-column half of an N tile holds [i | f | g | o] for 16 units
  auto h_out = at::empty({rows, H}, x.options());
  auto c_out = at::empty({rows, H}, x.options());
  // gates in the epilogue's grouped order (see lstm_gate_index): [rows, 64 * ceil(H / 16)]
  at::Tensor gates = save_gates ? at::empty({rows, 64 * ((H + G - 1) / G)}, x.options()) : at::Tensor();
  if (rows == 0) return {h_out, c_out, gates};
  const bool has_h = h.has_value() && h->defined();
  SegSource a;
  a.nseg = 2;
  a.seg[0] = seg_f32(x, in_dim, pad8(in_dim));
  if (has_h) {
    a.seg[1] = seg_f32(*h, H, pad8(H));
  } else {
    a.seg[1].kind = kSegZero;
    a.seg[1].kpad = pad8(H);
  }
  WeightSource b;
  b.L = lstm_layout({wi, wf, wg, wo}, in_dim, H, H);
  b.gate_group = G;
  EpiLSTM e;
  e.H = H;
  e.DP = G;
  e.b_i = bi.data_ptr<float>();
  e.b_f = bf.data_ptr<float>();
  e.b_g = bg.data_ptr<float>();
  e.b_o = bo.data_ptr<float>();
  e.c_prev = (c.has_value() && c->defined()) ? c->data_ptr<float>() : nullptr;
  e.h_out = h_out.data_ptr<float>();
  e.c_out = c_out.data_ptr<float>();
  e.gates = save_gates ? gates.data_ptr<float>() : nullptr;
  e.vec = (H % 4 == 0 && a16(e.b_i) && a16(e.b_f) && a16(e.b_g) && a16(e.b_o) && a16(e.c_prev) && a16(e.h_out) &&
           a16(e.c_out) && a16(e.gates)) ? 1 : 0;
  GemmShape sh;
  sh.M = rows;
  sh.N = 4 * G * ((H + G - 1) / G);
  sh.K = pad8(in_dim) + pad8(H);
  gemm(a, b, e, sh, cur_stream());
  SU_LAUNCH_CHECK();
  return {h_out, c_out, gates};
}

// Backward of lstm_fwd. Returns (dx, dh_prev, dc_prev) and accumulates weight/bias grads.
std::vector<at::Tensor> lstm_bwd(const at::Tensor& x, const c10::optional<at::Tensor>& h,
                                 const c10::optional<at::Tensor>& c, const at::Tensor& c_new, const at::Tensor& gates,
                                 const c10::optional<at::Tensor>& dh_opt, const c10::optional<at::Tensor>& dc_opt,
                                 const at::Tensor& wi, const at::Tensor& wf, const at::Tensor& wg,
                                 const at::Tensor& wo, at::Tensor& gwi, at::Tensor& gbi, at::Tensor& gwf,
                                 at::Tensor& gbf, at::Tensor& gwg, at::Tensor& gbg, at::Tensor& gwo,
                                 at::Tensor& gbo) {
  const int rows = static_cast<int>(x.size(0));
  const int in_dim = static_cast<int>(x.size(1));
  const int H = static_cast<int>(wi.size(0));
  const bool has_h = h.has_value() && h->defined();
  const bool has_c = c.has_value() && c->defined();
  const float* dh_p = nullptr;
  const float* dc_p = nullptr;
  auto dc_prev = at::empty({rows, H}, x.options());
  auto dxh = at::empty({rows, in_dim + H}, x.options());
  if (rows == 0) return {dxh.narrow(1, 0, in_dim), dxh.narrow(1, in_dim, H), dc_prev};
  // row-strided upstream gradients are read in place (a column view of the next cell's [dx || dh])
  at::Tensor dh_c, dc_c;
  if (dh_opt.has_value() && dh_opt->defined()) dh_c = dh_opt->stride(1) == 1 ? *dh_opt : dh_opt->contiguous();
  if (dc_opt.has_value() && dc_opt->defined()) dc_c = dc_opt->stride(1) == 1 ? *dc_opt : dc_opt->contiguous();
  dh_p = dh_c.defined() ? dh_c.data_ptr<float>() : nullptr;
  dc_p = dc_c.defined() ? dc_c.data_ptr<float>() : nullptr;
  const int dh_ld = dh_c.defined() ? static_cast<int>(dh_c.stride(0)) : H;
  const int dc_ld = dc_c.defined() ? static_cast<int>(dc_c.stride(0)) : H;
  const float* cp_p = has_c ? c->data_ptr<float>() : nullptr;
  const int DP4 = 4 * H;
  // xs = [x || h || 1]: the B operand of the weight-gradient GEMM (the ones column gives the bias gradient)
  SegSource xs;
  xs.nseg = 3;
  xs.seg[0] = seg_f32(x, in_dim, pad8(in_dim));
  if (has_h) xs.seg[1] = seg_f32(*h, H, pad8(H));
  else {
    xs.seg[1].kind = kSegZero;
    xs.seg[1].kpad = pad8(H);
  }
  xs.seg[2] = seg_ones();
  auto wgrad_epi = [&]() {
    EpiWeightGrad e;
    e.L = lstm_layout({gwi, gwf, gwg, gwo}, in_dim, H, H);
    e.L.nseg = 3;
    e.L.seg_kpad[2] = 8;
    float* bgs[4] = {gbi.data_ptr<float>(), gbf.data_ptr<float>(), gbg.data_ptr<float>(), gbo.data_ptr<float>()};
    for (int i = 0; i < 4; ++i) e.bias_grad[i] = bgs[i];
    e.bias_seg = 2;
    e.ncols = pad8(in_dim) + pad8(H) + 8;
    return e;
  };
  auto wgrad_shape = [&](int ncols) {
    GemmShape sh;
    sh.M = DP4;
    sh.N = ncols;
    sh.K = rows;
    const int nchunks = (rows + kBK - 1) / kBK;
    const int tiles = ((DP4 + kBM - 1) / kBM) * ((sh.N + 255) / 256);
    sh.ksplit = wgrad_ksplit(nchunks, tiles);
    return sh;
  };
  // Packed path: the backward kernel writes dpre straight into the two bf16 tile
  // images the GEMMs read (no row-major dpre, no packing pass over it)
  if (H % 32 == 0 && in_dim % 8 == 0 && packed_gemm_enabled() &&
      lstm_bwd_bf16_ok(gates.data_ptr<float>(), cp_p, c_new.data_ptr<float>(), dh_p, dh_ld, dc_p, dc_ld, H, nullptr,
                       dc_prev.data_ptr<float>())) {
    const int64_t tiles_k = (rows + kBM - 1) / kBM, chunks_mn = (rows + kBK - 1) / kBK;
    at::Tensor img_k = at::empty({tiles_k * (DP4 / kBK) * kBM * kBK * 2}, x.options().dtype(at::kByte));
    at::Tensor img_mn = at::empty({(DP4 / kBM) * chunks_mn * kBM * kBK * 2}, x.options().dtype(at::kByte));
    launch_lstm_bwd_pack(cur_stream(), gates.data_ptr<float>(), cp_p, c_new.data_ptr<float>(), dh_p, dh_ld, dc_p,
                         dc_ld, rows, H, img_k.data_ptr<uint8_t>(), img_mn.data_ptr<uint8_t>(),
                         dc_prev.data_ptr<float>());
    Prepacked<false> ak;
    ak.image = img_k.data_ptr<uint8_t>();
    WeightLayout L = lstm_layout({wi, wf, wg, wo}, in_dim, H, H);
    L.blk_pad[3] = DP4 - 3 * H;
    EpiLinear e;
    e.out = dxh.data_ptr<float>();
    e.ldo = in_dim + H;
    e.ncols = in_dim + H;
    GemmShape sh;
    sh.M = rows;
    sh.N = in_dim + pad8(H);
    sh.K = DP4;
    TORCH_CHECK(gemm_prepacked(ak, weight_mn(L, DP4), e, sh, cur_stream()),
                "lstm_bwd: packed GEMM workspace unavailable");
    Prepacked<true> am;
    am.image = img_mn.data_ptr<uint8_t>();
    EpiWeightGrad ew = wgrad_epi();
    TORCH_CHECK(gemm_prepacked(am, seg_mn(xs, rows), ew, wgrad_shape(ew.ncols), cur_stream()),
                "lstm_bwd: packed GEMM workspace unavailable");
    SU_LAUNCH_CHECK();
    return {dxh.narrow(1, 0, in_dim), dxh.narrow(1, in_dim, H), dc_prev};
  }
  // pre-activation gradients in bf16 when the vectorised kernel applies (the GEMMs
  // below read them as bf16 operands either way)
  at::Tensor dpre = at::empty({rows, DP4}, x.options().dtype(at::kBFloat16));
  ASeg dpre_seg;
  if (lstm_bwd_bf16_ok(gates.data_ptr<float>(), cp_p, c_new.data_ptr<float>(), dh_p, dh_ld, dc_p, dc_ld, H,
                       dpre.data_ptr(), dc_prev.data_ptr<float>())) {
    launch_lstm_bwd_bf16(cur_stream(), gates.data_ptr<float>(), cp_p, c_new.data_ptr<float>(), dh_p, dh_ld, dc_p,
                         dc_ld, rows, H, reinterpret_cast<__nv_bfloat16*>(dpre.data_ptr()),
                         dc_prev.data_ptr<float>());
    dpre_seg = seg_bf16(dpre, DP4, pad8(DP4));
  } else {
    dpre = at::empty({rows, DP4}, x.options());
    launch_lstm_bwd(cur_stream(), gates.data_ptr<float>(), cp_p, c_new.data_ptr<float>(), dh_p, dh_ld, dc_p, dc_ld,
                    rows, H, dpre.data_ptr<float>(), dc_prev.data_ptr<float>());
    dpre_seg = seg_f32(dpre, DP4, pad8(DP4));
  }
  // d[x || h] = dpre [W_i; W_f; W_g; W_o]
  {
    SegSource a;
    a.nseg = 1;
    a.seg[0] = dpre_seg;
    WeightLayout L = lstm_layout({wi, wf, wg, wo}, in_dim, H, H);
    L.blk_pad[3] = pad8(DP4) - 3 * H;
    WeightMN b = weight_mn(L, pad8(DP4));
    EpiLinear e;
    e.out = dxh.data_ptr<float>();
    e.ldo = in_dim + H;
    e.ncols = in_dim + H;
    // B rows follow the padded K space of the forward (x then h segments)
    GemmShape sh;
    sh.M = rows;
    sh.N = pad8(in_dim) + pad8(H);
    sh.K = pad8(DP4);
    // write into a padded buffer then compact (segment padding shifts the h columns)
    if (pad8(in_dim) != in_dim) {
      auto tmp = at::empty({rows, pad8(in_dim) + pad8(H)}, x.options());
      e.out = tmp.data_ptr<float>();
      e.ldo = pad8(in_dim) + pad8(H);
      e.ncols = pad8(in_dim) + pad8(H);
      gemm(a, b, e, sh, cur_stream());
      dxh.narrow(1, 0, in_dim).copy_(tmp.narrow(1, 0, in_dim));
      dxh.narrow(1, in_dim, H).copy_(tmp.narrow(1, pad8(in_dim), H));
    } else {
      gemm(a, b, e, sh, cur_stream());
    }
  }
  // weight / bias gradients: dW_gate += dpre_gate^T [x || h]
  {
    SegSource dy;
    dy.nseg = 1;
    dy.seg[0] = dpre_seg;
    EpiWeightGrad e = wgrad_epi();
    gemm(seg_mn(dy, rows), seg_mn(xs, rows), e, wgrad_shape(e.ncols), cur_stream());
  }
  SU_LAUNCH_CHECK();
  return {dxh.narrow(1, 0, in_dim), dxh.narrow(1, in_dim, H), dc_prev};
}

// ---------------------------------------------------------------------------
// NVLink halo path (see starry_unigraph/parallel/halo.py): aggregation whose
// source rows are read from the owners' staging buffers, and its backward
// pushing source-row gradients into the owners' gradient buffers.
// ---------------------------------------------------------------------------
at::Tensor spmm_peer_gather(const at::Tensor& rowptr, const at::Tensor& col, const at::Tensor& val,
                            const at::Tensor& peers, const at::Tensor& src_owner, const at::Tensor& src_row,
                            int64_t n_rows, int64_t F) {
  SU_CHECK_I64(rowptr); SU_CHECK_I32(col); SU_CHECK_F32(val); SU_CHECK_I32(src_owner); SU_CHECK_I32(src_row);
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong, "peer table must be cuda int64");
  at::Tensor out = at::empty({n_rows, F}, val.options());
  launch_spmm_peer_gather(cur_stream(), rowptr.data_ptr<int64_t>(), col.data_ptr<int>(), val.data_ptr<float>(),
                          reinterpret_cast<const float* const*>(peers.data_ptr<int64_t>()),
                          src_owner.data_ptr<int>(), src_row.data_ptr<int>(), n_rows, static_cast<int>(F),
                          out.data_ptr<float>());
  SU_LAUNCH_CHECK();
  return out;
}

at::Tensor halo_pull(const at::Tensor& peers, const at::Tensor& src_owner, const at::Tensor& src_row,
                     const at::Tensor& halo_src, int64_t F) {
  SU_CHECK_I32(src_owner); SU_CHECK_I32(src_row); SU_CHECK_I32(halo_src);
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong, "peer table must be cuda int64");
  TORCH_CHECK(F % 4 == 0, "halo rows are pulled in 16-byte vectors: F must be a multiple of 4");
  at::Tensor out = at::empty({halo_src.numel(), F}, src_owner.options().dtype(at::kFloat));
  launch_halo_pull(cur_stream(), reinterpret_cast<const float* const*>(peers.data_ptr<int64_t>()),
                   src_owner.data_ptr<int>(), src_row.data_ptr<int>(), halo_src.data_ptr<int>(), halo_src.numel(),
                   static_cast<int>(F), out.data_ptr<float>());
  SU_LAUNCH_CHECK();
  return out;
}

at::Tensor spmm_two_tables(const at::Tensor& rowptr, const at::Tensor& col, const at::Tensor& val,
                           const at::Tensor& x, const at::Tensor& halo, int64_t n_rows) {
  SU_CHECK_I64(rowptr); SU_CHECK_I32(col); SU_CHECK_F32(val); SU_CHECK_F32(x); SU_CHECK_CONTIG(x);
  SU_CHECK_F32(halo); SU_CHECK_CONTIG(halo);
  const int F = static_cast<int>(x.size(1));
  TORCH_CHECK(halo.numel() == 0 || halo.size(1) == F, "halo rows must have the width of x");
  at::Tensor out = at::empty({n_rows, F}, x.options());
  launch_spmm_two_tables(cur_stream(), rowptr.data_ptr<int64_t>(), col.data_ptr<int>(), val.data_ptr<float>(),
                         x.data_ptr<float>(), halo.numel() ? halo.data_ptr<float>() : nullptr,
                         static_cast<int>(x.size(0)), n_rows, F, out.data_ptr<float>());
  SU_LAUNCH_CHECK();
  return out;
}

void spmm_peer_push(const at::Tensor& rowptr_t, const at::Tensor& col_t, const at::Tensor& val_t,
                    const at::Tensor& grad_dst, int64_t n_src, const at::Tensor& peers, const at::Tensor& src_owner,
                    const at::Tensor& src_row) {
  SU_CHECK_F32(grad_dst); SU_CHECK_CONTIG(grad_dst);
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong, "peer table must be cuda int64");
  launch_spmm_peer_push(cur_stream(), rowptr_t.data_ptr<int64_t>(), col_t.data_ptr<int>(), val_t.data_ptr<float>(),
                        grad_dst.data_ptr<float>(), n_src, static_cast<int>(grad_dst.size(1)),
                        reinterpret_cast<float* const*>(peers.data_ptr<int64_t>()), src_owner.data_ptr<int>(),
                        src_row.data_ptr<int>());
  SU_LAUNCH_CHECK();
}
