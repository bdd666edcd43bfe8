// Torch-side wrappers of the DTDG kernels: CSR SpMM, fused LSTM cell (tcgen05
// GEMM with a gate epilogue) and its backward (elementwise gate gradients, then
// input and weight gradients on the tcgen05 GEMM).
#include "host_common.h"

using namespace su;

int64_t spmm_plan_warps_op() { return spmm_plan_warps(at::cuda::current_device()); }

at::Tensor spmm_csr(const at::Tensor& rowptr, const at::Tensor& col, const at::Tensor& val, const at::Tensor& x,
                    int64_t n_rows, const c10::optional<at::Tensor>& out_opt, bool accumulate,
                    const c10::optional<std::vector<at::Tensor>>& plan_t) {
  SU_CHECK_I64(rowptr); SU_CHECK_I32(col); SU_CHECK_F32(val); SU_CHECK_F32(x); SU_CHECK_CONTIG(x);
  const int F = static_cast<int>(x.size(1));
  at::Tensor out = (out_opt.has_value() && out_opt->defined()) ? *out_opt : at::empty({n_rows, F}, x.options());
  TORCH_CHECK(out.is_contiguous() && out.size(1) == F, "bad output buffer");
  SpmmPlan plan;
  const bool planned = spmm_plan_from(plan_t, &plan).items != nullptr;
  launch_spmm_csr(cur_stream(), rowptr.data_ptr<int64_t>(), col.data_ptr<int>(), val.data_ptr<float>(),
                  x.data_ptr<float>(), n_rows, F, out.data_ptr<float>(), accumulate ? 1 : 0,
                  planned ? &plan : nullptr);
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
  // (bf16 images: the tf32 precision takes the fp32 path below)
  if (H % 32 == 0 && in_dim % 8 == 0 && packed_gemm_enabled() && !gemm_precision_tf32() &&
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
  if (!gemm_precision_tf32() && lstm_bwd_bf16_ok(gates.data_ptr<float>(), cp_p, c_new.data_ptr<float>(), dh_p, dh_ld, dc_p, dc_ld, H,
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

// `ld`: row stride of the peers' staging buffers (-1: F)
at::Tensor halo_pull(const at::Tensor& peers, const at::Tensor& src_owner, const at::Tensor& src_row,
                     const at::Tensor& halo_src, int64_t F, int64_t ld) {
  SU_CHECK_I32(src_owner); SU_CHECK_I32(src_row); SU_CHECK_I32(halo_src);
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong, "peer table must be cuda int64");
  if (ld < 0) ld = F;
  TORCH_CHECK(F % 4 == 0 && ld % 4 == 0 && ld >= F,
              "halo rows are pulled in 16-byte vectors: F and the row stride must be multiples of 4, stride >= F");
  at::Tensor out = at::empty({halo_src.numel(), F}, src_owner.options().dtype(at::kFloat));
  launch_halo_pull(cur_stream(), reinterpret_cast<const float* const*>(peers.data_ptr<int64_t>()),
                   src_owner.data_ptr<int>(), src_row.data_ptr<int>(), halo_src.data_ptr<int>(), halo_src.numel(),
                   static_cast<int>(F), static_cast<int>(ld), out.data_ptr<float>());
  SU_LAUNCH_CHECK();
  return out;
}

at::Tensor spmm_two_tables(const at::Tensor& rowptr, const at::Tensor& col, const at::Tensor& val,
                           const at::Tensor& x, const at::Tensor& halo, int64_t n_rows,
                           const c10::optional<std::vector<at::Tensor>>& plan_t) {
  SU_CHECK_I64(rowptr); SU_CHECK_I32(col); SU_CHECK_F32(val); SU_CHECK_F32(x);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be a row-major matrix (any row stride)");
  SU_CHECK_F32(halo); SU_CHECK_CONTIG(halo);
  const int F = static_cast<int>(x.size(1));
  TORCH_CHECK(halo.numel() == 0 || halo.size(1) == F, "halo rows must have the width of x");
  TORCH_CHECK(F % 4 != 0 || (x.stride(0) % 4 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0),
              "row-strided x needs 16-byte aligned rows");
  at::Tensor out = at::empty({n_rows, F}, x.options());
  SpmmPlan plan;
  launch_spmm_two_tables(cur_stream(), rowptr.data_ptr<int64_t>(), col.data_ptr<int>(), val.data_ptr<float>(),
                         x.data_ptr<float>(), static_cast<int>(x.stride(0)), halo.numel() ? halo.data_ptr<float>() : nullptr,
                         static_cast<int>(x.size(0)), n_rows, F, out.data_ptr<float>(),
                         spmm_plan_from(plan_t, &plan).items != nullptr ? &plan : nullptr);
  SU_LAUNCH_CHECK();
  return out;
}

// `ld`: row stride of the owners' gradient buffers (-1: the gradient width)
void spmm_peer_push(const at::Tensor& rowptr_t, const at::Tensor& col_t, const at::Tensor& val_t,
                    const at::Tensor& grad_dst, int64_t n_src, const at::Tensor& peers, const at::Tensor& src_owner,
                    const at::Tensor& src_row, int64_t ld, const c10::optional<std::vector<at::Tensor>>& plan_t) {
  SU_CHECK_F32(grad_dst); SU_CHECK_CONTIG(grad_dst);
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong, "peer table must be cuda int64");
  const int F = static_cast<int>(grad_dst.size(1));
  if (ld < 0) ld = F;
  TORCH_CHECK(ld >= F, "gradient buffer rows narrower than the gradient");
  SpmmPlan plan;
  launch_spmm_peer_push(cur_stream(), rowptr_t.data_ptr<int64_t>(), col_t.data_ptr<int>(), val_t.data_ptr<float>(),
                        grad_dst.data_ptr<float>(), n_src, F, static_cast<int>(ld),
                        reinterpret_cast<float* const*>(peers.data_ptr<int64_t>()), src_owner.data_ptr<int>(),
                        src_row.data_ptr<int>(), spmm_plan_from(plan_t, &plan).items != nullptr ? &plan : nullptr);
  SU_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// Reset-gated GRU cell (T-GCN, EvolveGCN MatGRU); see EpiRGruZR.
//   w_z, w_r, w_c: [H, Fx + H] over [x | h] (w_c over [x_c | r * h]).
// Forward returns (h', z, r, c, rh); the last four are saved for the backward.
// ---------------------------------------------------------------------------
static int rgru_check(const at::Tensor& xz, const at::Tensor& xr, const at::Tensor& xc, const at::Tensor& wz) {
  SU_CHECK_F32(xz); SU_CHECK_F32(xr); SU_CHECK_F32(xc); SU_CHECK_F32(wz);
  TORCH_CHECK(xz.stride(1) == 1 && xr.stride(1) == 1 && xc.stride(1) == 1, "gate inputs need unit column stride");
  const int H = static_cast<int>(wz.size(0));
  TORCH_CHECK(H % 8 == 0, "reset-gated GRU cell: hidden size must be a multiple of 8");
  return H;
}

std::vector<at::Tensor> rgru_fwd(const at::Tensor& xz, const at::Tensor& xr, const at::Tensor& xc,
                                 const c10::optional<at::Tensor>& h, const at::Tensor& wz, const at::Tensor& bz,
                                 const at::Tensor& wr, const at::Tensor& br, const at::Tensor& wc,
                                 const at::Tensor& bc) {
  const int H = rgru_check(xz, xr, xc, wz);
  const int rows = static_cast<int>(xz.size(0));
  const int Fx = static_cast<int>(xz.size(1));
  const int pF = pad8(Fx);
  const bool has_h = h.has_value() && h->defined();
  if (has_h) { SU_CHECK_F32(*h); TORCH_CHECK(h->stride(1) == 1, "h needs unit column stride"); }
  auto opt = xz.options();
  at::Tensor z = at::empty({rows, H}, opt), r = at::empty({rows, H}, opt), rh = at::empty({rows, H}, opt);
  at::Tensor c = at::empty({rows, H}, opt), hn = at::empty({rows, H}, opt);
  if (rows == 0) return {hn, z, r, c, rh};
  // z, r = sigmoid([x_z | x_r | h] [[W_zx, 0, W_zh], [0, W_rx, W_rh]]^T + b)
  {
    SegSource a;
    a.nseg = 3;
    a.seg[0] = seg_f32(xz, Fx, pF);
    a.seg[1] = seg_f32(xr, Fx, pF);
    if (has_h) a.seg[2] = seg_f32(*h, H, H);
    else { a.seg[2].kind = kSegZero; a.seg[2].kpad = H; }
    WeightSource b;
    b.gate_group = kRGruGroup;
    b.L.nblk = 2;
    b.L.nseg = 3;
    b.L.seg_kpad[0] = pF;
    b.L.seg_kpad[1] = pF;
    b.L.seg_kpad[2] = H;
    for (int i = 0; i < 2; ++i) {
      b.L.blk_rows[i] = H;
      b.L.blk_pad[i] = H;
    }
    b.L.cell[0][0] = wcell(wz, 0, 0, Fx);
    b.L.cell[0][2] = wcell(wz, 0, Fx, H);
    b.L.cell[1][1] = wcell(wr, 0, 0, Fx);
    b.L.cell[1][2] = wcell(wr, 0, Fx, H);
    EpiRGruZR e;
    e.H = H;
    e.bz = bz.data_ptr<float>();
    e.br = br.data_ptr<float>();
    e.h = has_h ? h->data_ptr<float>() : nullptr;
    e.h_ld = has_h ? static_cast<int>(h->stride(0)) : H;
    e.z_out = z.data_ptr<float>();
    e.r_out = r.data_ptr<float>();
    e.rh_out = rh.data_ptr<float>();
    GemmShape sh;
    sh.M = rows;
    sh.N = 2 * kRGruGroup * ((H + kRGruGroup - 1) / kRGruGroup);
    sh.K = 2 * pF + H;
    gemm(a, b, e, sh, cur_stream());
  }
  // c = tanh([x_c | r h] W_c^T + b_c), h' = z h + (1 - z) c
  {
    SegSource a;
    a.nseg = 2;
    a.seg[0] = seg_f32(xc, Fx, pF);
    a.seg[1] = seg_f32(rh, H, H);
    WeightSource b;
    b.L.nblk = 1;
    b.L.nseg = 2;
    b.L.seg_kpad[0] = pF;
    b.L.seg_kpad[1] = H;
    b.L.blk_rows[0] = H;
    b.L.blk_pad[0] = H;
    b.L.cell[0][0] = wcell(wc, 0, 0, Fx);
    b.L.cell[0][1] = wcell(wc, 0, Fx, H);
    EpiRGruOut e;
    e.H = H;
    e.bc = bc.data_ptr<float>();
    e.z = z.data_ptr<float>();
    e.h = has_h ? h->data_ptr<float>() : nullptr;
    e.h_ld = has_h ? static_cast<int>(h->stride(0)) : H;
    e.c_out = c.data_ptr<float>();
    e.h_out = hn.data_ptr<float>();
    GemmShape sh;
    sh.M = rows;
    sh.N = H;
    sh.K = pF + H;
    gemm(a, b, e, sh, cur_stream());
  }
  SU_LAUNCH_CHECK();
  return {hn, z, r, c, rh};
}

// Backward of rgru_fwd: returns (dx_z, dx_r, dx_c, dh) and accumulates the weight
// and bias gradients (gw_*, gb_*).
std::vector<at::Tensor> rgru_bwd(const at::Tensor& xz, const at::Tensor& xr, const at::Tensor& xc,
                                 const c10::optional<at::Tensor>& h, const at::Tensor& z, const at::Tensor& r,
                                 const at::Tensor& c, const at::Tensor& rh, const at::Tensor& dhn,
                                 const at::Tensor& wz, const at::Tensor& wr, const at::Tensor& wc, at::Tensor& gwz,
                                 at::Tensor& gbz, at::Tensor& gwr, at::Tensor& gbr, at::Tensor& gwc,
                                 at::Tensor& gbc) {
  const int H = rgru_check(xz, xr, xc, wz);
  const int rows = static_cast<int>(xz.size(0));
  const int Fx = static_cast<int>(xz.size(1));
  const int pF = pad8(Fx);
  const bool has_h = h.has_value() && h->defined();
  SU_CHECK_F32(dhn);
  TORCH_CHECK(dhn.stride(1) == 1, "dh' needs unit column stride");
  auto opt = xz.options();
  at::Tensor dzr = at::empty({rows, 2 * H}, opt);  // [dz_pre | dr_pre]
  at::Tensor dcp = at::empty({rows, H}, opt);
  at::Tensor dh_acc = has_h ? at::empty({rows, H}, opt) : at::Tensor();
  at::Tensor t2 = at::empty({rows, pF + H}, opt);        // d[x_c | r h]
  at::Tensor t1 = at::empty({rows, 2 * pF + H}, opt);    // d[x_z | x_r | h] through the z, r GEMM
  at::Tensor dh = has_h ? at::empty({rows, H}, opt) : at::Tensor();
  auto ret = [&]() {
    return std::vector<at::Tensor>{t1.narrow(1, 0, Fx), t1.narrow(1, pF, Fx), t2.narrow(1, 0, Fx), dh};
  };
  if (rows == 0) return ret();
  const float* hp = has_h ? h->data_ptr<float>() : nullptr;
  const int h_ld = has_h ? static_cast<int>(h->stride(0)) : H;
  launch_rgru_bwd1(cur_stream(), dhn.data_ptr<float>(), static_cast<int>(dhn.stride(0)), hp, h_ld, z.data_ptr<float>(),
                   c.data_ptr<float>(), rows, H, dzr.data_ptr<float>(), dcp.data_ptr<float>(),
                   has_h ? dh_acc.data_ptr<float>() : nullptr);
  auto ksplit_for = [&](int M, int N) {
    const int nchunks = (rows + kBK - 1) / kBK;
    const int tiles = ((M + kBM - 1) / kBM) * ((N + 255) / 256);
    return wgrad_ksplit(nchunks, tiles);
  };
  // --- candidate GEMM: d[x_c | r h] = dc_pre W_c; dW_c += dc_pre^T [x_c | r h | 1]
  WeightLayout Lc;
  Lc.nblk = 1;
  Lc.nseg = 2;
  Lc.seg_kpad[0] = pF;
  Lc.seg_kpad[1] = H;
  Lc.blk_rows[0] = H;
  Lc.blk_pad[0] = H;
  Lc.cell[0][0] = wcell(wc, 0, 0, Fx);
  Lc.cell[0][1] = wcell(wc, 0, Fx, H);
  {
    SegSource a;
    a.nseg = 1;
    a.seg[0] = seg_f32(dcp, H, H);
    EpiLinear e;
    e.out = t2.data_ptr<float>();
    e.ldo = pF + H;
    e.ncols = pF + H;
    GemmShape sh;
    sh.M = rows;
    sh.N = pF + H;
    sh.K = H;
    gemm(a, weight_mn(Lc, H), e, sh, cur_stream());
  }
  {
    SegSource dy;
    dy.nseg = 1;
    dy.seg[0] = seg_f32(dcp, H, H);
    SegSource xs;
    xs.nseg = 3;
    xs.seg[0] = seg_f32(xc, Fx, pF);
    xs.seg[1] = seg_f32(rh, H, H);
    xs.seg[2] = seg_ones();
    EpiWeightGrad e;
    e.L = Lc;
    e.L.nseg = 3;
    e.L.seg_kpad[2] = 8;
    e.L.cell[0][0] = wcell(gwc, 0, 0, Fx);
    e.L.cell[0][1] = wcell(gwc, 0, Fx, H);
    e.bias_grad[0] = gbc.data_ptr<float>();
    e.bias_seg = 2;
    e.ncols = pF + H + 8;
    GemmShape sh;
    sh.M = H;
    sh.N = e.ncols;
    sh.K = rows;
    sh.ksplit = ksplit_for(sh.M, sh.N);
    gemm(seg_mn(dy, rows), seg_mn(xs, rows), e, sh, cur_stream());
  }
  // dr_pre = d(r h) h r (1 - r); dh += d(r h) r
  launch_rgru_bwd2(cur_stream(), t2.data_ptr<float>() + pF, pF + H, hp, h_ld, r.data_ptr<float>(), rows, H,
                   dzr.data_ptr<float>(), has_h ? dh_acc.data_ptr<float>() : nullptr);
  // --- gate GEMM: d[x_z | x_r | h] = [dz_pre | dr_pre] [[W_zx, 0, W_zh], [0, W_rx, W_rh]]
  WeightLayout Lg;
  Lg.nblk = 2;
  Lg.nseg = 3;
  Lg.seg_kpad[0] = pF;
  Lg.seg_kpad[1] = pF;
  Lg.seg_kpad[2] = H;
  for (int i = 0; i < 2; ++i) {
    Lg.blk_rows[i] = H;
    Lg.blk_pad[i] = H;
  }
  Lg.cell[0][0] = wcell(wz, 0, 0, Fx);
  Lg.cell[0][2] = wcell(wz, 0, Fx, H);
  Lg.cell[1][1] = wcell(wr, 0, 0, Fx);
  Lg.cell[1][2] = wcell(wr, 0, Fx, H);
  {
    SegSource a;
    a.nseg = 1;
    a.seg[0] = seg_f32(dzr, 2 * H, 2 * H);
    EpiLinear e;
    e.out = t1.data_ptr<float>();
    e.ldo = 2 * pF + H;
    e.ncols = 2 * pF + H;
    GemmShape sh;
    sh.M = rows;
    sh.N = 2 * pF + H;
    sh.K = 2 * H;
    gemm(a, weight_mn(Lg, 2 * H), e, sh, cur_stream());
  }
  {
    SegSource dy;
    dy.nseg = 1;
    dy.seg[0] = seg_f32(dzr, 2 * H, 2 * H);
    SegSource xs;
    xs.nseg = 4;
    xs.seg[0] = seg_f32(xz, Fx, pF);
    xs.seg[1] = seg_f32(xr, Fx, pF);
    if (has_h) xs.seg[2] = seg_f32(*h, H, H);
    else { xs.seg[2].kind = kSegZero; xs.seg[2].kpad = H; }
    xs.seg[3] = seg_ones();
    EpiWeightGrad e;
    e.L = Lg;
    e.L.nseg = 4;
    e.L.seg_kpad[3] = 8;
    e.L.cell[0][0] = wcell(gwz, 0, 0, Fx);
    e.L.cell[0][2] = wcell(gwz, 0, Fx, H);
    e.L.cell[1][1] = wcell(gwr, 0, 0, Fx);
    e.L.cell[1][2] = wcell(gwr, 0, Fx, H);
    e.bias_grad[0] = gbz.data_ptr<float>();
    e.bias_grad[1] = gbr.data_ptr<float>();
    e.bias_seg = 3;
    e.ncols = 2 * pF + H + 8;
    GemmShape sh;
    sh.M = 2 * H;
    sh.N = e.ncols;
    sh.K = rows;
    sh.ksplit = ksplit_for(sh.M, sh.N);
    gemm(seg_mn(dy, rows), seg_mn(xs, rows), e, sh, cur_stream());
  }
  if (has_h)
    launch_add_rows(cur_stream(), dh_acc.data_ptr<float>(), t1.data_ptr<float>() + 2 * pF, 2 * pF + H, rows, H,
                    dh.data_ptr<float>());
  SU_LAUNCH_CHECK();
  return ret();
}
