#include "host_common.h"

using namespace su;

// ===========================================================================
// host entry points
// ===========================================================================
void tgn_prep(const at::Tensor& src, const at::Tensor& dst, const at::Tensor& ts, const at::Tensor& n_ev,
              const at::Tensor& neg_pool, at::Tensor& stamp, at::Tensor& node2root, at::Tensor& step_ctr, int64_t seed,
              at::Tensor& roots, at::Tensor& n_roots, at::Tensor& src_idx, at::Tensor& dst_idx, at::Tensor& neg,
              at::Tensor& neg_idx, at::Tensor& ts_max, at::Tensor& root_ts, at::Tensor& win_key, at::Tensor& win,
              at::Tensor& cnt) {
  SU_CHECK_I64(src); SU_CHECK_I64(dst); SU_CHECK_F32(ts); SU_CHECK_I32(n_ev);
  PrepArgs a;
  a.src = src.data_ptr<int64_t>();
  a.dst = dst.data_ptr<int64_t>();
  a.ts = ts.data_ptr<float>();
  a.n_ev = n_ev.data_ptr<int>();
  a.bmax = static_cast<int>(src.numel());
  a.rmax = static_cast<int>(roots.numel());
  TORCH_CHECK(a.rmax >= 2 * a.bmax, "roots buffer must hold 2 * bmax entries");
  a.neg_pool = neg_pool.data_ptr<int64_t>();
  a.pool_size = neg_pool.numel();
  TORCH_CHECK(a.pool_size > 0, "empty negative pool");
  a.stamp = stamp.data_ptr<int>();
  a.node2root = node2root.data_ptr<int>();
  a.step_ctr = step_ctr.data_ptr<int64_t>();
  a.seed = static_cast<uint64_t>(seed);
  a.roots = roots.data_ptr<int64_t>();
  a.n_roots = n_roots.data_ptr<int>();
  a.src_idx = src_idx.data_ptr<int>();
  a.dst_idx = dst_idx.data_ptr<int>();
  a.neg = neg.data_ptr<int64_t>();
  a.neg_idx = neg_idx.data_ptr<int>();
  a.ts_max = ts_max.data_ptr<float>();
  a.root_ts = root_ts.data_ptr<int64_t>();
  a.win_key = reinterpret_cast<unsigned long long*>(win_key.data_ptr<int64_t>());
  a.win = win.data_ptr<int>();
  a.cnt = cnt.data_ptr<int>();
  a.status = device_status_ptr(at::cuda::current_device());
  launch_tgn_prep(dim3(1), dim3(1024), cur_stream(), a);
  SU_LAUNCH_CHECK();
}

void tgn_sample(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& root_ts,
                const at::Tensor& rowptr, const at::Tensor& nbr, const at::Tensor& eid, const at::Tensor& ets,
                int64_t k, int64_t policy, int64_t seed, const at::Tensor& step_ctr, at::Tensor& out_nbr,
                at::Tensor& out_eid, at::Tensor& out_dt, at::Tensor& out_cnt, at::Tensor& edge_total) {
  C10_CUDA_CHECK(cudaMemsetAsync(edge_total.data_ptr<int>(), 0, sizeof(int), cur_stream()));
  const int rmax = static_cast<int>(roots.numel());
  TORCH_CHECK(k >= 1 && k <= 1024, "fanout out of range");
  const bool per_root = root_ts.numel() == roots.numel() && roots.numel() > 1;
  const int threads = 256;
  const int blocks = (rmax * 32 + threads - 1) / threads;
  launch_tgn_sample(dim3(blocks), dim3(threads), cur_stream(), 
      roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(), rmax, root_ts.data_ptr<int64_t>(),
      per_root ? root_ts.data_ptr<int64_t>() : nullptr, rowptr.data_ptr<int64_t>(), nbr.data_ptr<int64_t>(),
      eid.data_ptr<int64_t>(), ets.data_ptr<int64_t>(), static_cast<int>(k), static_cast<int>(policy),
      static_cast<uint64_t>(seed), step_ctr.data_ptr<int64_t>(), out_nbr.data_ptr<int64_t>(),
      out_eid.data_ptr<int64_t>(), out_dt.data_ptr<float>(), out_cnt.data_ptr<int>(),
      edge_total.data_ptr<int>());
  SU_LAUNCH_CHECK();
}

// One GRU step over rows `index` of `x_src` (gathered, column block col0..col0+width)
// with previous hidden rows (or zeros); see EpiGRU for outputs.
// hidden units per gate group: a 128-column tile holds two groups [r | z | n_i | n_h] x 16, one per
// epilogue column half
static constexpr int kGateGroup = 16;

static void gru_step(const SegSource& a, int kx, int kh, const at::Tensor& w_ih, const at::Tensor& w_hh,
                     const at::Tensor& b_ih, const at::Tensor& b_hh, EpiGRU e, int rmax, const int* m_dev) {
  const int D = static_cast<int>(w_hh.size(1));
  const int KX = static_cast<int>(w_ih.size(1));
  WeightSource b;
  b.gate_group = kGateGroup;
  b.L.nblk = 4;
  b.L.nseg = kh > 0 ? 2 : 1;
  for (int i = 0; i < 4; ++i) {
    b.L.blk_rows[i] = D;
    b.L.blk_pad[i] = D;
  }
  b.L.seg_kpad[0] = kx;
  b.L.seg_kpad[1] = kh;
  // r: [W_ir | W_hr], z: [W_iz | W_hz], n_i: [W_in | 0], n_h: [0 | W_hn]
  b.L.cell[0][0] = wcell(w_ih, 0, 0, KX);
  b.L.cell[1][0] = wcell(w_ih, D, 0, KX);
  b.L.cell[2][0] = wcell(w_ih, 2 * D, 0, KX);
  if (kh > 0) {
    b.L.cell[0][1] = wcell(w_hh, 0, 0, D);
    b.L.cell[1][1] = wcell(w_hh, D, 0, D);
    b.L.cell[3][1] = wcell(w_hh, 2 * D, 0, D);
  }
  e.D = D;
  e.DP = kGateGroup;
  e.b_ih = b_ih.data_ptr<float>();
  e.b_hh = b_hh.data_ptr<float>();
  GemmShape sh;
  sh.M = rmax;
  sh.m_dev = m_dev;
  sh.N = 4 * kGateGroup * ((D + kGateGroup - 1) / kGateGroup);
  sh.K = kx + kh;
  e.vec = gru_vec(e);
  gemm(a, b, e, sh, cur_stream());
}

// Memory updater: GRU over the K mailbox slots (h0 = 0) then GRUCell(agg, mem),
// writing the new memory into `memory` rows `roots` (and memory_ts = ts_max) and
// saving the previous memory rows into `mem_prev`.
void tgn_memory_update(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& mailbox, int64_t K,
                       at::Tensor& memory, at::Tensor& memory_ts, const at::Tensor& ts_max, const at::Tensor& gru_w_ih,
                       const at::Tensor& gru_w_hh, const at::Tensor& gru_b_ih, const at::Tensor& gru_b_hh,
                       const at::Tensor& cell_w_ih, const at::Tensor& cell_w_hh, const at::Tensor& cell_b_ih,
                       const at::Tensor& cell_b_hh, at::Tensor& agg_buf, at::Tensor& agg_buf2, at::Tensor& mem_prev,
                       const c10::optional<at::Tensor>& peer) {
  const PeerDesc pd = peer_desc(peer);
  const int rmax = static_cast<int>(roots.numel());
  const int D = static_cast<int>(memory.size(1));
  const int SW = static_cast<int>(gru_w_ih.size(1));
  const int* m_dev = n_roots.data_ptr<int>();
  const int64_t* ridx = roots.data_ptr<int64_t>();
  at::Tensor cur = agg_buf, nxt = agg_buf2;
  for (int s = 0; s < K; ++s) {
    SegSource a;
    a.nrows_dev = m_dev;
    a.nseg = s == 0 ? 1 : 2;
    a.seg[0] = seg_f32(mailbox.view({mailbox.size(0), -1}), SW, pad8(SW), ridx, s * SW);
    if (pd.on) {  // mailbox rows of the owner rank
      a.seg[0].kind = kSegSharded;
      a.seg[0].peers = pd.mail_peers;
      a.seg[0].owner = pd.owner;
      a.seg[0].vec = (a.seg[0].ld % 4 == 0 && (s * SW) % 4 == 0) ? 1 : 0;
    }
    if (s > 0) a.seg[1] = seg_f32(cur, D, pad8(D));
    EpiGRU e;
    e.hprev = s == 0 ? nullptr : cur.data_ptr<float>();
    e.hprev_ld = D;
    e.hout = nxt.data_ptr<float>();
    e.hout_ld = D;
    gru_step(a, pad8(SW), s == 0 ? 0 : pad8(D), gru_w_ih, gru_w_hh, gru_b_ih, gru_b_hh, e, rmax, m_dev);
    std::swap(cur, nxt);
  }
  // GRUCell(agg, memory[roots]) -> memory[roots]
  SegSource a;
  a.nrows_dev = m_dev;
  a.nseg = 2;
  a.seg[0] = seg_f32(cur, D, pad8(D));
  a.seg[1] = seg_memory(memory, D, ridx, pd, false);
  EpiGRU e;
  e.hprev = memory.data_ptr<float>();
  e.hprev_index = ridx;
  e.hprev_ld = D;
  e.save_prev = mem_prev.data_ptr<float>();
  if (pd.on) {
    // tables stay read-only during the step: new rows go to mem_new and are
    // written back to the owners after the ranks' barrier
    e.hprev_peers = pd.mem_peers;
    e.hprev_owner = pd.owner;
    e.hout = pd.mem_new;
    e.hout_ld = D;
  } else {
    e.scatter = memory.data_ptr<float>();
    e.scatter_index = ridx;
    e.scatter_ld = D;
    e.scatter_ts = memory_ts.data_ptr<float>();
    e.ts_value = ts_max.data_ptr<float>();
  }
  gru_step(a, pad8(D), pad8(D), cell_w_ih, cell_w_hh, cell_b_ih, cell_b_hh, e, rmax, m_dev);
}

// JODIE memory updater: tanh RNN cell over the (single) newest mailbox slot,
//   h' = tanh(W_ih m + b_ih + W_hh h + b_hh),
// with the same outputs as tgn_memory_update (memory rows, memory_ts, mem_prev),
// after recording the roots' memory_ts before the update (prev_ts) for the
// time projection.
void tgn_rnn_memory_update(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& mailbox,
                           at::Tensor& memory, at::Tensor& memory_ts, const at::Tensor& ts_max,
                           const at::Tensor& w_ih, const at::Tensor& w_hh, const at::Tensor& b_ih,
                           const at::Tensor& b_hh, at::Tensor& mem_prev, at::Tensor& prev_ts,
                           const c10::optional<at::Tensor>& peer) {
  const PeerDesc pd = peer_desc(peer);
  const int rmax = static_cast<int>(roots.numel());
  const int D = static_cast<int>(memory.size(1));
  const int SW = static_cast<int>(w_ih.size(1));
  const int* m_dev = n_roots.data_ptr<int>();
  const int64_t* ridx = roots.data_ptr<int64_t>();
  TORCH_CHECK(!pd.on || pd.ts_peers != nullptr, "peer descriptor without memory_ts tables");
  launch_jodie_prev_ts(cur_stream(), ridx, m_dev, rmax, memory_ts.data_ptr<float>(), pd.on ? pd.ts_peers : nullptr,
                       pd.owner, prev_ts.data_ptr<float>());
  SegSource a;
  a.nrows_dev = m_dev;
  a.nseg = 2;
  a.seg[0] = seg_f32(mailbox.view({mailbox.size(0), -1}), SW, pad8(SW), ridx, 0);
  if (pd.on) {
    a.seg[0].kind = kSegSharded;
    a.seg[0].peers = pd.mail_peers;
    a.seg[0].owner = pd.owner;
  }
  a.seg[1] = seg_memory(memory, D, ridx, pd, false);
  WeightSource b;
  b.gate_group = kGateGroup;
  b.L.nblk = 1;
  b.L.nseg = 2;
  b.L.blk_rows[0] = D;
  b.L.blk_pad[0] = D;
  b.L.seg_kpad[0] = pad8(SW);
  b.L.seg_kpad[1] = pad8(D);
  b.L.cell[0][0] = wcell(w_ih, 0, 0, SW);
  b.L.cell[0][1] = wcell(w_hh, 0, 0, D);
  EpiGRU e;
  e.D = D;
  e.DP = kGateGroup;
  e.ngates = 1;
  e.b_ih = b_ih.data_ptr<float>();
  e.b_hh = b_hh.data_ptr<float>();
  e.hprev = memory.data_ptr<float>();
  e.hprev_index = ridx;
  e.hprev_ld = D;
  e.save_prev = mem_prev.data_ptr<float>();
  if (pd.on) {
    e.hprev_peers = pd.mem_peers;
    e.hprev_owner = pd.owner;
    e.hout = pd.mem_new;
    e.hout_ld = D;
  } else {
    e.scatter = memory.data_ptr<float>();
    e.scatter_index = ridx;
    e.scatter_ld = D;
    e.scatter_ts = memory_ts.data_ptr<float>();
    e.ts_value = ts_max.data_ptr<float>();
  }
  GemmShape sh;
  sh.M = rmax;
  sh.m_dev = m_dev;
  sh.N = kGateGroup * ((D + kGateGroup - 1) / kGateGroup);
  sh.K = pad8(SW) + pad8(D);
  e.vec = gru_vec(e);
  gemm(a, b, e, sh, cur_stream());
  SU_LAUNCH_CHECK();
}

// z = memory(roots) * (1 + w dt + b)  (JODIE time projection), dt saved for the backward
void jodie_project(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& memory,
                   const at::Tensor& prev_ts, const at::Tensor& root_ts, double dt_scale, const at::Tensor& w,
                   const at::Tensor& b, at::Tensor& out, at::Tensor& dt, const c10::optional<at::Tensor>& peer) {
  const PeerDesc pd = peer_desc(peer);
  launch_jodie_project(cur_stream(), roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(),
                       static_cast<int>(roots.numel()), memory.data_ptr<float>(), pd.on ? pd.mem_new : nullptr,
                       static_cast<int>(memory.size(1)), prev_ts.data_ptr<float>(), root_ts.data_ptr<int64_t>(),
                       static_cast<float>(dt_scale), w.data_ptr<float>(), b.data_ptr<float>(), out.data_ptr<float>(),
                       dt.data_ptr<float>());
  SU_LAUNCH_CHECK();
}

void jodie_project_bwd(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& memory,
                       const at::Tensor& dt, const at::Tensor& dz, at::Tensor& dw, at::Tensor& db,
                       const c10::optional<at::Tensor>& peer) {
  const PeerDesc pd = peer_desc(peer);
  launch_jodie_project_bwd(cur_stream(), roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(),
                           static_cast<int>(roots.numel()), memory.data_ptr<float>(), pd.on ? pd.mem_new : nullptr,
                           static_cast<int>(memory.size(1)), dt.data_ptr<float>(), dz.data_ptr<float>(),
                           dw.data_ptr<float>(), db.data_ptr<float>());
  SU_LAUNCH_CHECK();
}

void tgn_mailbox_write(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& win,
                       const at::Tensor& cnt, const at::Tensor& src_idx, const at::Tensor& dst_idx,
                       const at::Tensor& ev_eid, const at::Tensor& ev_ts, const at::Tensor& mem_prev,
                       const at::Tensor& efeat, int64_t E, at::Tensor& mailbox, at::Tensor& mailbox_ts,
                       at::Tensor& next_pos) {
  const int rmax = static_cast<int>(roots.numel());
  const int D = static_cast<int>(mem_prev.size(1));
  const int K = static_cast<int>(mailbox.size(1));
  launch_tgn_mailbox(dim3(rmax), dim3(128), cur_stream(), 
      roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(), rmax, win.data_ptr<int>(), cnt.data_ptr<int>(),
      src_idx.data_ptr<int>(), dst_idx.data_ptr<int>(), ev_eid.data_ptr<int64_t>(), ev_ts.data_ptr<float>(),
      mem_prev.data_ptr<float>(), D, efeat.data_ptr(), efeat.scalar_type() == at::kBFloat16 ? 1 : 0,
      static_cast<int>(efeat.stride(0)),
      static_cast<int>(efeat.size(1)), static_cast<int>(E), mailbox.data_ptr<float>(), mailbox_ts.data_ptr<float>(),
      next_pos.data_ptr<int64_t>(), K);
  SU_LAUNCH_CHECK();
}

// Q = W_q [h(roots) || cos(b_t)] + b_q ;  KV = [W_k; W_v] [h(nbr) || e(eid) || cos(w_t dt + b_t)] + [b_k; b_v]
void tgn_attn_proj(const at::Tensor& memory, const at::Tensor& roots, const at::Tensor& n_roots,
                   const at::Tensor& nbr, const at::Tensor& nbr_eid, const at::Tensor& nbr_dt,
                   const at::Tensor& nbr_cnt, const at::Tensor& efeat, int64_t E, const at::Tensor& te_w,
                   const at::Tensor& te_b, const at::Tensor& wq, const at::Tensor& bq, const at::Tensor& wk,
                   const at::Tensor& bk, const at::Tensor& wv, const at::Tensor& bv, at::Tensor& Q, at::Tensor& KV,
    const c10::optional<at::Tensor>& peer) {
  const PeerDesc pd = peer_desc(peer);
  const int rmax = static_cast<int>(roots.numel());
  const int k = static_cast<int>(nbr.numel() / rmax);
  const int D = static_cast<int>(memory.size(1));
  const int T = static_cast<int>(te_b.numel());
  const int Do = static_cast<int>(wq.size(0));
  const int ER = static_cast<int>(efeat.size(1));
  const int Ew = std::min<int>(static_cast<int>(E), ER);
  // --- Q over roots
  {
    SegSource a;
    a.nrows_dev = n_roots.data_ptr<int>();
    a.nseg = 2;
    a.seg[0] = seg_memory(memory, D, roots.data_ptr<int64_t>(), pd, true);
    a.seg[1] = seg_time(nullptr, te_w, te_b, pad8(T));
    WeightSource b;
    b.L.nblk = 1;
    b.L.nseg = 2;
    b.L.blk_rows[0] = Do;
    b.L.blk_pad[0] = Do;
    b.L.seg_kpad[0] = pad8(D);
    b.L.seg_kpad[1] = pad8(T);
    b.L.cell[0][0] = wcell(wq, 0, 0, D);
    b.L.cell[0][1] = wcell(wq, 0, D, T);
    EpiLinear e;
    e.out = Q.data_ptr<float>();
    e.ldo = Do;
    e.ncols = Do;
    e.bias = bq.data_ptr<float>();
    GemmShape sh;
    sh.M = rmax;
    sh.m_dev = n_roots.data_ptr<int>();
    sh.N = Do;
    sh.K = pad8(D) + pad8(T);
    gemm(a, b, e, sh, cur_stream());
  }
  // --- K, V over edges
  {
    SegSource a;
    a.group = k;
    a.gcount = nbr_cnt.data_ptr<int>();
    a.nseg = 3;
    a.seg[0] = seg_memory(memory, D, nbr.data_ptr<int64_t>(), pd, true);
    a.seg[1] = seg_feat(efeat, Ew, pad8(static_cast<int>(E)), nbr_eid.data_ptr<int64_t>());
    a.seg[2] = seg_time(nbr_dt.data_ptr<float>(), te_w, te_b, pad8(T));
    WeightSource b;
    b.L.nblk = 2;
    b.L.nseg = 3;
    b.L.blk_rows[0] = Do;
    b.L.blk_pad[0] = Do;
    b.L.blk_rows[1] = Do;
    b.L.blk_pad[1] = Do;
    b.L.seg_kpad[0] = pad8(D);
    b.L.seg_kpad[1] = pad8(static_cast<int>(E));
    b.L.seg_kpad[2] = pad8(T);
    const at::Tensor* ws[2] = {&wk, &wv};
    for (int i = 0; i < 2; ++i) {
      b.L.cell[i][0] = wcell(*ws[i], 0, 0, D);
      b.L.cell[i][1] = wcell(*ws[i], 0, D, static_cast<int>(E));
      b.L.cell[i][2] = wcell(*ws[i], 0, D + static_cast<int>(E), T);
    }
    EpiLinear e;
    e.out = KV.data_ptr<float>();
    e.ldo = 2 * Do;
    e.ncols = 2 * Do;
    e.bias = bk.data_ptr<float>();
    e.bias2 = bv.data_ptr<float>();
    e.bias_split = Do;
    GemmShape sh;
    sh.M = rmax * k;
    sh.N = 2 * Do;
    sh.K = pad8(D) + pad8(static_cast<int>(E)) + pad8(T);
    gemm(a, b, e, sh, cur_stream());
  }
}

void tgn_attn_fwd(const at::Tensor& Q, const at::Tensor& KV, const at::Tensor& nbr_cnt, const at::Tensor& n_roots,
                  int64_t H, double att_drop, int64_t seed, const at::Tensor& step_ctr, at::Tensor& att_p,
                  at::Tensor& agg) {
  const int rmax = static_cast<int>(Q.size(0));
  const int Do = static_cast<int>(Q.size(1));
  const int k = static_cast<int>(KV.size(0) / rmax);
  TORCH_CHECK(k <= 32, "fused attention supports fanout <= 32");
  TORCH_CHECK(H <= 4 && Do % H == 0, "heads must divide the output dim (<= 4 heads)");
  TORCH_CHECK(Do <= 256, "fused attention supports output dims up to 256");
  const int threads = 256;
  launch_tgn_attn_fwd(dim3((rmax * 32 + threads - 1) / threads), dim3(threads), cur_stream(), 
      Q.data_ptr<float>(), KV.data_ptr<float>(), nbr_cnt.data_ptr<int>(), n_roots.data_ptr<int>(), rmax, k, Do,
      static_cast<int>(H), static_cast<float>(att_drop), static_cast<uint64_t>(seed), step_ctr.data_ptr<int64_t>(),
      att_p.data_ptr<float>(), agg.data_ptr<float>());
  SU_LAUNCH_CHECK();
}

void tgn_attn_bwd(const at::Tensor& Q, const at::Tensor& KV, const at::Tensor& att_p, const at::Tensor& dagg,
                  const at::Tensor& nbr_cnt, const at::Tensor& n_roots, int64_t H, double att_drop, int64_t seed,
                  const at::Tensor& step_ctr, at::Tensor& dKV, at::Tensor& dQ) {
  const int rmax = static_cast<int>(Q.size(0));
  const int Do = static_cast<int>(Q.size(1));
  const int k = static_cast<int>(KV.size(0) / rmax);
  TORCH_CHECK(k <= 32 && H <= 4 && Do % H == 0 && Do <= 256, "fused attention: fanout <= 32, <= 4 heads, dim <= 256");
  const int threads = 256;
  launch_tgn_attn_bwd(dim3((rmax * 32 + threads - 1) / threads), dim3(threads), cur_stream(), 
      Q.data_ptr<float>(), KV.data_ptr<float>(), att_p.data_ptr<float>(), dagg.data_ptr<float>(),
      nbr_cnt.data_ptr<int>(), n_roots.data_ptr<int>(), rmax, k, Do, static_cast<int>(H), static_cast<float>(att_drop),
      static_cast<uint64_t>(seed), step_ctr.data_ptr<int64_t>(), dKV.data_ptr<float>(), dQ.data_ptr<float>());
  SU_LAUNCH_CHECK();
}

// out = LayerNorm(ReLU(Dropout(W_out [agg || h(roots)] + b_out)))
void tgn_out_fwd(const at::Tensor& agg, const at::Tensor& memory, const at::Tensor& roots, const at::Tensor& n_roots,
                 const at::Tensor& w_out, const at::Tensor& b_out, const at::Tensor& gamma, const at::Tensor& beta,
                 double drop, int64_t seed, const at::Tensor& step_ctr, const at::Tensor& edge_total, at::Tensor& out,
                 at::Tensor& xsave, at::Tensor& mean, at::Tensor& rstd,
    const c10::optional<at::Tensor>& peer) {
  const PeerDesc pd = peer_desc(peer);
  const int rmax = static_cast<int>(roots.numel());
  const int Do = static_cast<int>(w_out.size(0));
  const int D = static_cast<int>(memory.size(1));
  SegSource a;
  a.nrows_dev = n_roots.data_ptr<int>();
  a.nseg = 2;
  a.seg[0] = seg_f32(agg, Do, pad8(Do));
  a.seg[1] = seg_memory(memory, D, roots.data_ptr<int64_t>(), pd, true);
  WeightSource b;
  b.L.nblk = 1;
  b.L.nseg = 2;
  b.L.blk_rows[0] = Do;
  b.L.blk_pad[0] = Do;
  b.L.seg_kpad[0] = pad8(Do);
  b.L.seg_kpad[1] = pad8(D);
  b.L.cell[0][0] = wcell(w_out, 0, 0, Do);
  b.L.cell[0][1] = wcell(w_out, 0, Do, D);
  EpiOutLN e;
  e.Do = Do;
  e.bias = b_out.data_ptr<float>();
  e.gamma = gamma.data_ptr<float>();
  e.beta = beta.data_ptr<float>();
  e.drop = static_cast<float>(drop);
  e.seed = static_cast<uint64_t>(seed);
  e.step_ctr = step_ctr.data_ptr<int64_t>();
  e.edge_total = edge_total.data_ptr<int>();
  e.out = out.data_ptr<float>();
  e.xsave = xsave.data_ptr<float>();
  e.mean = mean.data_ptr<float>();
  e.rstd = rstd.data_ptr<float>();
  GemmShape sh;
  sh.M = rmax;
  sh.m_dev = n_roots.data_ptr<int>();
  sh.N = Do;
  sh.K = pad8(Do) + pad8(D);
  TORCH_CHECK(Do <= 256, "output dim must be <= 256");
  gemm(a, b, e, sh, cur_stream());
}

void tgn_out_bwd(const at::Tensor& dout, const at::Tensor& xsave, const at::Tensor& mean, const at::Tensor& rstd,
                 const at::Tensor& gamma, const at::Tensor& n_roots, double drop, int64_t seed,
                 const at::Tensor& step_ctr, const at::Tensor& edge_total, at::Tensor& dpre, at::Tensor& dgamma,
                 at::Tensor& dbeta) {
  const int rmax = static_cast<int>(dout.size(0));
  const int Do = static_cast<int>(dout.size(1));
  const int threads = 256;
  launch_tgn_out_bwd(dim3((rmax * 32 + threads - 1) / threads), dim3(threads), cur_stream(), 
      dout.data_ptr<float>(), xsave.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(),
      gamma.data_ptr<float>(), n_roots.data_ptr<int>(), rmax, Do, static_cast<float>(drop),
      static_cast<uint64_t>(seed), step_ctr.data_ptr<int64_t>(), edge_total.data_ptr<int>(), dpre.data_ptr<float>(),
      dgamma.data_ptr<float>(),
      dbeta.data_ptr<float>());
  SU_LAUNCH_CHECK();
}

// Weight gradients of a projection whose input is regenerated by a SegSource.
static void proj_wgrad(const SegSource& dy_src, int dy_cols, const SegSource& x_src_with_ones, int x_kspace,
                       int rows_static, const WeightLayout& grad_layout, float* const* bias_grads, int bias_seg) {
  SegMN a = seg_mn(dy_src, rows_static);
  SegMN b = seg_mn(x_src_with_ones, rows_static);
  EpiWeightGrad e;
  e.L = grad_layout;
  for (int i = 0; i < kMaxBlk; ++i) e.bias_grad[i] = bias_grads ? bias_grads[i] : nullptr;
  e.bias_seg = bias_seg;
  e.ncols = x_kspace;
  GemmShape sh;
  sh.M = dy_cols;
  sh.N = x_kspace;
  sh.K = rows_static;
  const int nchunks = (rows_static + kBK - 1) / kBK;
  const int tiles = ((dy_cols + kBM - 1) / kBM) * ((x_kspace + 255) / 256);
  sh.ksplit = wgrad_ksplit(nchunks, tiles);
  gemm(a, b, e, sh, cur_stream());
}

// Backward of the attention projections: grads of W_q,b_q,W_k,b_k,W_v,b_v and of
// the time encoder (w_t, b_t). Memory rows and edge features are detached.
void tgn_attn_proj_bwd(const at::Tensor& memory, const at::Tensor& roots, const at::Tensor& n_roots,
                       const at::Tensor& nbr, const at::Tensor& nbr_eid, const at::Tensor& nbr_dt,
                       const at::Tensor& nbr_cnt, const at::Tensor& efeat, int64_t E, const at::Tensor& te_w,
                       const at::Tensor& te_b, const at::Tensor& wq, const at::Tensor& wk, const at::Tensor& wv,
                       const at::Tensor& dQ, const at::Tensor& dKV, at::Tensor& g_wq, at::Tensor& g_bq,
                       at::Tensor& g_wk, at::Tensor& g_bk, at::Tensor& g_wv, at::Tensor& g_bv, at::Tensor& g_tw,
                       at::Tensor& g_tb, at::Tensor& M_t, at::Tensor& M_1,
    const c10::optional<at::Tensor>& peer, int64_t part) {
  // part 0: all; 1: W_q / b_q gradients; 2: W_k, W_v gradients and the encoder products M_t, M_1
  // ([2*Do, T] buffers of the caller); 3: the encoder gradient from M_t, M_1 and g_bq
  const PeerDesc pd = peer_desc(peer);
  const int rmax = static_cast<int>(roots.numel());
  const int k = static_cast<int>(nbr.numel() / rmax);
  const int D = static_cast<int>(memory.size(1));
  const int T = static_cast<int>(te_b.numel());
  const int Do = static_cast<int>(wq.size(0));
  const int Ei = static_cast<int>(E);
  const int Ew = std::min<int>(Ei, static_cast<int>(efeat.size(1)));
  // ---------------- W_q, b_q
  if (part == 0 || part == 1) {
    SegSource dy;
    dy.nrows_dev = n_roots.data_ptr<int>();
    dy.nseg = 1;
    dy.seg[0] = seg_f32(dQ, Do, pad8(Do));
    SegSource x;
    x.nrows_dev = n_roots.data_ptr<int>();
    x.nseg = 3;
    x.seg[0] = seg_memory(memory, D, roots.data_ptr<int64_t>(), pd, true);
    x.seg[1] = seg_time(nullptr, te_w, te_b, pad8(T));
    x.seg[2] = seg_ones();
    WeightLayout L;
    L.nblk = 1;
    L.nseg = 3;
    L.blk_rows[0] = Do;
    L.blk_pad[0] = Do;
    L.seg_kpad[0] = pad8(D);
    L.seg_kpad[1] = pad8(T);
    L.seg_kpad[2] = 8;
    L.cell[0][0] = wcell(g_wq, 0, 0, D);
    L.cell[0][1] = wcell(g_wq, 0, D, T);
    float* bg[4] = {g_bq.data_ptr<float>(), nullptr, nullptr, nullptr};
    proj_wgrad(dy, Do, x, pad8(D) + pad8(T) + 8, rmax, L, bg, 2);
  }
  // ---------------- W_k, b_k, W_v, b_v (reduction over edges), plus the time-encoder terms
  // The encoder gradient is  dw[c] = sum_r dT[r,c] (-sin(w_c t_r + b_c)) t_r  with  dT = dKV W_kv[:, time],
  // i.e.  dw[c] = sum_o W_kv[o, time c] * M_t[o, c],  M_t = dKV^T (-sin(..) t)  (and M_1 without t for db):
  // two extra column segments of this weight-gradient GEMM, then a T-wide finishing kernel.
  TORCH_CHECK(M_t.numel() == 2 * Do * T && M_1.numel() == 2 * Do * T, "encoder product buffers must be [2*Do, T]");
  if (part == 0 || part == 2) {
    M_t.zero_();
    M_1.zero_();
    SegSource dy;
    dy.group = k;
    dy.gcount = nbr_cnt.data_ptr<int>();
    dy.nseg = 1;
    dy.seg[0] = seg_f32(dKV, 2 * Do, pad8(2 * Do));
    SegSource x;
    x.group = k;
    x.gcount = nbr_cnt.data_ptr<int>();
    x.nseg = 6;
    x.seg[0] = seg_memory(memory, D, nbr.data_ptr<int64_t>(), pd, true);
    x.seg[1] = seg_feat(efeat, Ew, pad8(Ei), nbr_eid.data_ptr<int64_t>());
    x.seg[2] = seg_time(nbr_dt.data_ptr<float>(), te_w, te_b, pad8(T));
    x.seg[3] = seg_ones();
    x.seg[4] = seg_time(nbr_dt.data_ptr<float>(), te_w, te_b, pad8(T));
    x.seg[4].kind = kSegTimeSin;
    x.seg[4].tmul = 1;
    x.seg[5] = seg_time(nbr_dt.data_ptr<float>(), te_w, te_b, pad8(T));
    x.seg[5].kind = kSegTimeSin;
    WeightLayout L;
    L.nblk = 2;
    L.nseg = 6;
    L.blk_rows[0] = Do;
    L.blk_pad[0] = Do;
    L.blk_rows[1] = Do;
    L.blk_pad[1] = Do;
    L.seg_kpad[0] = pad8(D);
    L.seg_kpad[1] = pad8(Ei);
    L.seg_kpad[2] = pad8(T);
    L.seg_kpad[3] = 8;
    L.seg_kpad[4] = pad8(T);
    L.seg_kpad[5] = pad8(T);
    at::Tensor* gs[2] = {&g_wk, &g_wv};
    for (int i = 0; i < 2; ++i) {
      L.cell[i][0] = wcell(*gs[i], 0, 0, D);
      L.cell[i][1] = wcell(*gs[i], 0, D, Ei);
      L.cell[i][2] = wcell(*gs[i], 0, D + Ei, T);
      L.cell[i][4] = wcell(M_t, i * Do, 0, T);
      L.cell[i][5] = wcell(M_1, i * Do, 0, T);
    }
    float* bg[4] = {g_bk.data_ptr<float>(), g_bv.data_ptr<float>(), nullptr, nullptr};
    proj_wgrad(dy, 2 * Do, x, pad8(D) + pad8(Ei) + pad8(T) + 8 + 2 * pad8(T), rmax * k, L, bg, 3);
  }
  if (part == 0 || part == 3) {
    // Q side: roots encode t = 0, so only db gets  -sin(b_c) sum_o W_q[o, time c] * (sum_rows dQ[r, o]);
    // the row sum of dQ is this step's b_q gradient (computed above)
    launch_time_grad_finish(cur_stream(), wk.data_ptr<float>(), wv.data_ptr<float>(), static_cast<int>(wk.stride(0)),
                            D + Ei, wq.data_ptr<float>(), static_cast<int>(wq.stride(0)), D, Do, T,
                            M_t.data_ptr<float>(), M_1.data_ptr<float>(), g_bq.data_ptr<float>(),
                            te_b.data_ptr<float>(), g_tw.data_ptr<float>(), g_tb.data_ptr<float>());
  }
  SU_LAUNCH_CHECK();
}

// Output projection backward: dW_out, db_out and d(agg) from dpre.
void tgn_out_proj_bwd(const at::Tensor& dpre, const at::Tensor& agg, const at::Tensor& memory,
                      const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& w_out, at::Tensor& g_wout,
                      at::Tensor& g_bout, at::Tensor& dagg,
    const c10::optional<at::Tensor>& peer, int64_t part) {
  // part 0: both; 1: weight gradients only; 2: data gradient only
  const PeerDesc pd = peer_desc(peer);
  const int rmax = static_cast<int>(roots.numel());
  const int Do = static_cast<int>(w_out.size(0));
  const int D = static_cast<int>(memory.size(1));
  if (part != 2) {
    SegSource dy;
    dy.nrows_dev = n_roots.data_ptr<int>();
    dy.nseg = 1;
    dy.seg[0] = seg_f32(dpre, Do, pad8(Do));
    SegSource x;
    x.nrows_dev = n_roots.data_ptr<int>();
    x.nseg = 3;
    x.seg[0] = seg_f32(agg, Do, pad8(Do));
    x.seg[1] = seg_memory(memory, D, roots.data_ptr<int64_t>(), pd, true);
    x.seg[2] = seg_ones();
    WeightLayout L;
    L.nblk = 1;
    L.nseg = 3;
    L.blk_rows[0] = Do;
    L.blk_pad[0] = Do;
    L.seg_kpad[0] = pad8(Do);
    L.seg_kpad[1] = pad8(D);
    L.seg_kpad[2] = 8;
    L.cell[0][0] = wcell(g_wout, 0, 0, Do);
    L.cell[0][1] = wcell(g_wout, 0, Do, D);
    float* bg[4] = {g_bout.data_ptr<float>(), nullptr, nullptr, nullptr};
    proj_wgrad(dy, Do, x, pad8(Do) + pad8(D) + 8, rmax, L, bg, 2);
  }
  if (part != 1) {
    SegSource a;
    a.nrows_dev = n_roots.data_ptr<int>();
    a.nseg = 1;
    a.seg[0] = seg_f32(dpre, Do, pad8(Do));
    WeightLayout L;  // B[n = agg col, k = out feature] = W_out[k, n]
    L.nblk = 1;
    L.nseg = 1;
    L.blk_rows[0] = Do;
    L.blk_pad[0] = pad8(Do);
    L.seg_kpad[0] = pad8(Do);
    L.cell[0][0] = wcell(w_out, 0, 0, Do);
    WeightMN b = weight_mn(L, pad8(Do));
    EpiLinear e;
    e.out = dagg.data_ptr<float>();
    e.ldo = Do;
    e.ncols = Do;
    GemmShape sh;
    sh.M = rmax;
    sh.m_dev = n_roots.data_ptr<int>();
    sh.N = Do;
    sh.K = pad8(Do);
    gemm(a, b, e, sh, cur_stream());
  }
}

// P = out [W_src; W_dst]^T + [b_src; b_dst] (per-root projections of the link predictor)
void tgn_link_proj(const at::Tensor& out, const at::Tensor& n_roots, const at::Tensor& w_src, const at::Tensor& b_src,
                   const at::Tensor& w_dst, const at::Tensor& b_dst, at::Tensor& P) {
  const int rmax = static_cast<int>(out.size(0));
  const int D = static_cast<int>(out.size(1));
  const int Dp = static_cast<int>(w_src.size(0));
  SegSource a;
  a.nrows_dev = n_roots.data_ptr<int>();
  a.nseg = 1;
  a.seg[0] = seg_f32(out, D, pad8(D));
  WeightSource b;
  b.L.nblk = 2;
  b.L.nseg = 1;
  b.L.blk_rows[0] = Dp;
  b.L.blk_pad[0] = Dp;
  b.L.blk_rows[1] = Dp;
  b.L.blk_pad[1] = Dp;
  b.L.seg_kpad[0] = pad8(D);
  b.L.cell[0][0] = wcell(w_src, 0, 0, D);
  b.L.cell[1][0] = wcell(w_dst, 0, 0, D);
  EpiLinear e;
  e.out = P.data_ptr<float>();
  e.ldo = 2 * Dp;
  e.ncols = 2 * Dp;
  e.bias = b_src.data_ptr<float>();
  e.bias2 = b_dst.data_ptr<float>();
  e.bias_split = Dp;
  GemmShape sh;
  sh.M = rmax;
  sh.m_dev = n_roots.data_ptr<int>();
  sh.N = 2 * Dp;
  sh.K = pad8(D);
  gemm(a, b, e, sh, cur_stream());
}

void tgn_link_loss(const at::Tensor& P, const at::Tensor& src_idx, const at::Tensor& dst_idx,
                   const at::Tensor& neg_idx, const at::Tensor& n_ev, const at::Tensor& b_dst,
                   const at::Tensor& w_out, const at::Tensor& b_out, bool need_grad, at::Tensor& scores,
                   at::Tensor& loss, at::Tensor& dP, at::Tensor& g_w_out, at::Tensor& g_b_out, at::Tensor& g_b_dst) {
  const int bmax = static_cast<int>(src_idx.numel());
  const int D = static_cast<int>(w_out.numel());
  const int threads = 256;
  launch_tgn_link(dim3((bmax * 32 + threads - 1) / threads), dim3(threads), cur_stream(), 
      P.data_ptr<float>(), src_idx.data_ptr<int>(), dst_idx.data_ptr<int>(), neg_idx.data_ptr<int>(),
      n_ev.data_ptr<int>(), bmax, D, b_dst.data_ptr<float>(), w_out.data_ptr<float>(), b_out.data_ptr<float>(),
      need_grad ? 1 : 0, scores.data_ptr<float>(), loss.data_ptr<float>(), need_grad ? dP.data_ptr<float>() : nullptr,
      need_grad ? g_w_out.data_ptr<float>() : nullptr, need_grad ? g_b_out.data_ptr<float>() : nullptr,
      need_grad ? g_b_dst.data_ptr<float>() : nullptr);
  SU_LAUNCH_CHECK();
}

void tgn_metrics(const at::Tensor& scores, const at::Tensor& n_ev, at::Tensor& out) {
  const int bmax = static_cast<int>(scores.numel() / 2);
  launch_tgn_metrics(dim3(1), dim3(1024), cur_stream(), scores.data_ptr<float>(), n_ev.data_ptr<int>(), bmax,
                                                   out.data_ptr<float>());
  SU_LAUNCH_CHECK();
}

// Link-predictor backward through the per-root projections: dW_src/dW_dst (+biases)
// and d(out) = dP [W_src; W_dst].
void tgn_link_proj_bwd(const at::Tensor& dP, const at::Tensor& out, const at::Tensor& n_roots,
                       const at::Tensor& w_src, const at::Tensor& w_dst, at::Tensor& g_wsrc, at::Tensor& g_bsrc,
                       at::Tensor& g_wdst, at::Tensor& g_bdst, at::Tensor& dout, int64_t part) {
  // part 0: both; 1: weight gradients only; 2: data gradient only (callers overlap the two on two streams)
  const int rmax = static_cast<int>(out.size(0));
  const int D = static_cast<int>(out.size(1));
  const int Dp = static_cast<int>(w_src.size(0));
  if (part != 2) {
    SegSource dy;
    dy.nrows_dev = n_roots.data_ptr<int>();
    dy.nseg = 1;
    dy.seg[0] = seg_f32(dP, 2 * Dp, pad8(2 * Dp));
    SegSource x;
    x.nrows_dev = n_roots.data_ptr<int>();
    x.nseg = 2;
    x.seg[0] = seg_f32(out, D, pad8(D));
    x.seg[1] = seg_ones();
    WeightLayout L;
    L.nblk = 2;
    L.nseg = 2;
    L.blk_rows[0] = Dp;
    L.blk_pad[0] = Dp;
    L.blk_rows[1] = Dp;
    L.blk_pad[1] = Dp;
    L.seg_kpad[0] = pad8(D);
    L.seg_kpad[1] = 8;
    L.cell[0][0] = wcell(g_wsrc, 0, 0, D);
    L.cell[1][0] = wcell(g_wdst, 0, 0, D);
    float* bg[4] = {g_bsrc.data_ptr<float>(), g_bdst.data_ptr<float>(), nullptr, nullptr};
    proj_wgrad(dy, 2 * Dp, x, pad8(D) + 8, rmax, L, bg, 1);
  }
  if (part != 1) {
    SegSource a;
    a.nrows_dev = n_roots.data_ptr<int>();
    a.nseg = 1;
    a.seg[0] = seg_f32(dP, 2 * Dp, pad8(2 * Dp));
    WeightLayout L;
    L.nblk = 2;
    L.nseg = 1;
    L.blk_rows[0] = Dp;
    L.blk_pad[0] = Dp;
    L.blk_rows[1] = Dp;
    L.blk_pad[1] = pad8(2 * Dp) - Dp;
    L.seg_kpad[0] = pad8(D);
    L.cell[0][0] = wcell(w_src, 0, 0, D);
    L.cell[1][0] = wcell(w_dst, 0, 0, D);
    WeightMN b = weight_mn(L, pad8(2 * Dp));
    EpiLinear e;
    e.out = dout.data_ptr<float>();
    e.ldo = D;
    e.ncols = D;
    GemmShape sh;
    sh.M = rmax;
    sh.m_dev = n_roots.data_ptr<int>();
    sh.N = D;
    sh.K = pad8(2 * Dp);
    gemm(a, b, e, sh, cur_stream());
  }
}
