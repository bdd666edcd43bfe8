// Python bindings of the sm_100a kernels (module starry_unigraph._C).
#include <torch/extension.h>

int64_t status_read(bool clear);
#include <c10/cuda/CUDACachingAllocator.h>
#include <cuda_runtime.h>
namespace su {
long long launch_count();
void set_gemm_precision(bool tf32);
bool gemm_precision_tf32();
void set_tma_store_min_rows(int rows);
int tma_store_min_rows();
using WorkspaceAlloc = void* (*)(size_t bytes, cudaStream_t stream);
using WorkspaceFree = void (*)(void* ptr);
void set_workspace_allocator(WorkspaceAlloc alloc, WorkspaceFree free_fn);
}
// GEMM operand images come from the caching allocator: stream-ordered reuse, and
// the CUDA graph's private pool during capture
static void* su_ws_alloc(size_t bytes, cudaStream_t st) {
  return c10::cuda::CUDACachingAllocator::raw_alloc_with_stream(bytes, st);
}
static void su_ws_free(void* p) { c10::cuda::CUDACachingAllocator::raw_delete(p); }
at::Tensor linear_fwd(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, int64_t act);
void linear_fwd_into(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, int64_t act,
                     at::Tensor& out);
at::Tensor linear_dgrad(const at::Tensor& dy, const at::Tensor& w, const c10::optional<at::Tensor>& mask);
void linear_wgrad(const at::Tensor& dy, const at::Tensor& x, at::Tensor& dw, const c10::optional<at::Tensor>& db,
                  const c10::optional<at::Tensor>& mask);

void tgn_prep(const at::Tensor& src, const at::Tensor& dst, const at::Tensor& ts, const at::Tensor& n_ev,
              const at::Tensor& neg_pool, at::Tensor& stamp, at::Tensor& node2root, at::Tensor& step_ctr, int64_t seed,
              at::Tensor& roots, at::Tensor& n_roots, at::Tensor& src_idx, at::Tensor& dst_idx, at::Tensor& neg,
              at::Tensor& neg_idx, at::Tensor& ts_max, at::Tensor& root_ts, at::Tensor& win_key, at::Tensor& win,
              at::Tensor& cnt);
void tgn_sample(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& root_ts,
                const at::Tensor& rowptr, const at::Tensor& nbr, const at::Tensor& eid, const at::Tensor& ets,
                int64_t k, int64_t policy, int64_t seed, const at::Tensor& step_ctr, at::Tensor& out_nbr,
                at::Tensor& out_eid, at::Tensor& out_dt, at::Tensor& out_cnt, at::Tensor& edge_total);
void tgn_memory_update(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& mailbox, int64_t K,
                       at::Tensor& memory, at::Tensor& memory_ts, const at::Tensor& ts_max, const at::Tensor& gru_w_ih,
                       const at::Tensor& gru_w_hh, const at::Tensor& gru_b_ih, const at::Tensor& gru_b_hh,
                       const at::Tensor& cell_w_ih, const at::Tensor& cell_w_hh, const at::Tensor& cell_b_ih,
                       const at::Tensor& cell_b_hh, at::Tensor& agg_buf, at::Tensor& agg_buf2, at::Tensor& mem_prev,
                       const c10::optional<at::Tensor>& peer);
void tgn_mailbox_write(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& win,
                       const at::Tensor& cnt, const at::Tensor& src_idx, const at::Tensor& dst_idx,
                       const at::Tensor& ev_eid, const at::Tensor& ev_ts, const at::Tensor& mem_prev,
                       const at::Tensor& efeat, int64_t E, at::Tensor& mailbox, at::Tensor& mailbox_ts,
                       at::Tensor& next_pos);
void tgn_attn_proj(const at::Tensor& memory, const at::Tensor& roots, const at::Tensor& n_roots,
                   const at::Tensor& nbr, const at::Tensor& nbr_eid, const at::Tensor& nbr_dt,
                   const at::Tensor& nbr_cnt, const at::Tensor& efeat, int64_t E, const at::Tensor& te_w,
                   const at::Tensor& te_b, const at::Tensor& wq, const at::Tensor& bq, const at::Tensor& wk,
                   const at::Tensor& bk, const at::Tensor& wv, const at::Tensor& bv, at::Tensor& Q, at::Tensor& KV,
                   const c10::optional<at::Tensor>& peer);
void tgn_attn_fwd(const at::Tensor& Q, const at::Tensor& KV, const at::Tensor& nbr_cnt, const at::Tensor& n_roots,
                  int64_t H, double att_drop, int64_t seed, const at::Tensor& step_ctr, at::Tensor& att_p,
                  at::Tensor& agg);
void tgn_attn_bwd(const at::Tensor& Q, const at::Tensor& KV, const at::Tensor& att_p, const at::Tensor& dagg,
                  const at::Tensor& nbr_cnt, const at::Tensor& n_roots, int64_t H, double att_drop, int64_t seed,
                  const at::Tensor& step_ctr, at::Tensor& dKV, at::Tensor& dQ);
void tgn_out_fwd(const at::Tensor& agg, const at::Tensor& memory, const at::Tensor& roots, const at::Tensor& n_roots,
                 const at::Tensor& w_out, const at::Tensor& b_out, const at::Tensor& gamma, const at::Tensor& beta,
                 double drop, int64_t seed, const at::Tensor& step_ctr, const at::Tensor& edge_total, at::Tensor& out,
                 at::Tensor& xsave, at::Tensor& mean, at::Tensor& rstd, const c10::optional<at::Tensor>& peer);
void tgn_out_bwd(const at::Tensor& dout, const at::Tensor& xsave, const at::Tensor& mean, const at::Tensor& rstd,
                 const at::Tensor& gamma, const at::Tensor& n_roots, double drop, int64_t seed,
                 const at::Tensor& step_ctr, const at::Tensor& edge_total, at::Tensor& dpre, at::Tensor& dgamma,
                 at::Tensor& dbeta);
void tgn_attn_proj_bwd(const at::Tensor& memory, const at::Tensor& roots, const at::Tensor& n_roots,
                       const at::Tensor& nbr, const at::Tensor& nbr_eid, const at::Tensor& nbr_dt,
                       const at::Tensor& nbr_cnt, const at::Tensor& efeat, int64_t E, const at::Tensor& te_w,
                       const at::Tensor& te_b, const at::Tensor& wq, const at::Tensor& wk, const at::Tensor& wv,
                       const at::Tensor& dQ, const at::Tensor& dKV, at::Tensor& g_wq, at::Tensor& g_bq,
                       at::Tensor& g_wk, at::Tensor& g_bk, at::Tensor& g_wv, at::Tensor& g_bv, at::Tensor& g_tw,
                       at::Tensor& g_tb, at::Tensor& M_t, at::Tensor& M_1, const c10::optional<at::Tensor>& peer,
                       int64_t part);
void tgn_out_proj_bwd(const at::Tensor& dpre, const at::Tensor& agg, const at::Tensor& memory,
                      const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& w_out, at::Tensor& g_wout,
                      at::Tensor& g_bout, at::Tensor& dagg, const c10::optional<at::Tensor>& peer,
                      int64_t part);
void tgn_link_proj(const at::Tensor& out, const at::Tensor& n_roots, const at::Tensor& w_src, const at::Tensor& b_src,
                   const at::Tensor& w_dst, const at::Tensor& b_dst, at::Tensor& P);
void tgn_link_loss(const at::Tensor& P, const at::Tensor& src_idx, const at::Tensor& dst_idx,
                   const at::Tensor& neg_idx, const at::Tensor& n_ev, const at::Tensor& b_dst,
                   const at::Tensor& w_out, const at::Tensor& b_out, bool need_grad, at::Tensor& scores,
                   at::Tensor& loss, at::Tensor& dP, at::Tensor& g_w_out, at::Tensor& g_b_out, at::Tensor& g_b_dst);
void tgn_metrics(const at::Tensor& scores, const at::Tensor& n_ev, at::Tensor& out);
void tgn_link_proj_bwd(const at::Tensor& dP, const at::Tensor& out, const at::Tensor& n_roots,
                       const at::Tensor& w_src, const at::Tensor& w_dst, at::Tensor& g_wsrc, at::Tensor& g_bsrc,
                       at::Tensor& g_wdst, at::Tensor& g_bdst, at::Tensor& dout, int64_t part);
void adam_flat(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, at::Tensor& step, at::Tensor& done,
               double lr, double b1, double b2, double eps, double wd, double grad_scale);

at::Tensor spmm_csr(const at::Tensor& rowptr, const at::Tensor& col, const at::Tensor& val, const at::Tensor& x,
                    int64_t n_rows, const c10::optional<at::Tensor>& out_opt, bool accumulate,
                    const c10::optional<std::vector<at::Tensor>>& plan);
int64_t spmm_plan_warps_op();
std::vector<at::Tensor> lstm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& h,
                                 const c10::optional<at::Tensor>& c, const at::Tensor& wi, const at::Tensor& bi,
                                 const at::Tensor& wf, const at::Tensor& bf, const at::Tensor& wg,
                                 const at::Tensor& bg, const at::Tensor& wo, const at::Tensor& bo, bool save_gates);
std::vector<at::Tensor> lstm_bwd(const at::Tensor& x, const c10::optional<at::Tensor>& h,
                                 const c10::optional<at::Tensor>& c, const at::Tensor& c_new, const at::Tensor& gates,
                                 const c10::optional<at::Tensor>& dh_opt, const c10::optional<at::Tensor>& dc_opt,
                                 const at::Tensor& wi, const at::Tensor& wf, const at::Tensor& wg,
                                 const at::Tensor& wo, at::Tensor& gwi, at::Tensor& gbi, at::Tensor& gwf,
                                 at::Tensor& gbf, at::Tensor& gwg, at::Tensor& gbg, at::Tensor& gwo,
                                 at::Tensor& gbo);

// peer_ops.cpp
void peer_barrier(const at::Tensor& flag_ptrs, int64_t rank, int64_t world, at::Tensor& epoch, int64_t budget);
void peer_allreduce_adam(const at::Tensor& grad_ptrs, int64_t world, at::Tensor& p, at::Tensor& m, at::Tensor& v,
                         at::Tensor& step, at::Tensor& done, double lr, double b1, double b2, double eps, double wd,
                         double scale);
void tgn_peer_writeback(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& mem_new,
                        const at::Tensor& owner, const at::Tensor& mem_ptrs, const at::Tensor& ts_ptrs,
                        const at::Tensor& ts_max, const c10::optional<std::vector<at::Tensor>>& cache,
                        double thresh, int64_t rank);
void tgn_peer_mail_claim(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& win,
                         const at::Tensor& ev_eid, const at::Tensor& ev_ts, const at::Tensor& owner,
                         const at::Tensor& claim_ptrs);
void tgn_peer_mail_write(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& win,
                         const at::Tensor& src_idx, const at::Tensor& dst_idx, const at::Tensor& ev_eid,
                         const at::Tensor& ev_ts, const at::Tensor& mem_prev, const at::Tensor& efeat, int64_t E,
                         const at::Tensor& owner, const at::Tensor& claim_ptrs, const at::Tensor& mail_ptrs,
                         const at::Tensor& mail_ts_ptrs);

void peer_signal(const at::Tensor& flag_ptrs, int64_t rank, int64_t world, at::Tensor& epoch);
void peer_wait(const at::Tensor& my_flags, int64_t rank, int64_t world, const at::Tensor& epoch, int64_t budget);
void tgn_peer_wait_claim(const at::Tensor& my_flags, int64_t rank, int64_t world, const at::Tensor& epoch,
                         int64_t budget, const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& win,
                         const at::Tensor& ev_eid, const at::Tensor& ev_ts, const at::Tensor& owner,
                         const at::Tensor& claim_ptrs);
void tgn_peer_push(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& mem_new,
                   const at::Tensor& ts_max, const at::Tensor& owner, const at::Tensor& mem_ptrs,
                   const at::Tensor& ts_ptrs, const c10::optional<std::vector<at::Tensor>>& cache, double thresh,
                   int64_t rank, const at::Tensor& win, const at::Tensor& src_idx, const at::Tensor& dst_idx,
                   const at::Tensor& ev_eid, const at::Tensor& ev_ts, const at::Tensor& mem_prev,
                   const at::Tensor& efeat, int64_t E, const at::Tensor& claim_ptrs,
                   const c10::optional<at::Tensor>& mail_ptrs, const c10::optional<at::Tensor>& mail_ts_ptrs);
void peer_rs_adam_ag(const at::Tensor& grad_ptrs, const at::Tensor& param_ptrs, int64_t world, int64_t rank,
                     const at::Tensor& p_local, at::Tensor& m, at::Tensor& v, at::Tensor& step, at::Tensor& done,
                     double lr, double b1, double b2, double eps, double wd, double scale);

at::Tensor spmm_peer_gather(const at::Tensor& rowptr, const at::Tensor& col, const at::Tensor& val,
                            const at::Tensor& peers, const at::Tensor& src_owner, const at::Tensor& src_row,
                            int64_t n_rows, int64_t F);
at::Tensor halo_pull(const at::Tensor& peers, const at::Tensor& src_owner, const at::Tensor& src_row,
                     const at::Tensor& halo_src, int64_t F, int64_t ld);
at::Tensor spmm_two_tables(const at::Tensor& rowptr, const at::Tensor& col, const at::Tensor& val,
                           const at::Tensor& x, const at::Tensor& halo, int64_t n_rows,
                           const c10::optional<std::vector<at::Tensor>>& plan);
std::vector<at::Tensor> rgru_fwd(const at::Tensor& xz, const at::Tensor& xr, const at::Tensor& xc,
                                 const c10::optional<at::Tensor>& h, const at::Tensor& wz, const at::Tensor& bz,
                                 const at::Tensor& wr, const at::Tensor& br, const at::Tensor& wc,
                                 const at::Tensor& bc);
std::vector<at::Tensor> rgru_bwd(const at::Tensor& xz, const at::Tensor& xr, const at::Tensor& xc,
                                 const c10::optional<at::Tensor>& h, const at::Tensor& z, const at::Tensor& r,
                                 const at::Tensor& c, const at::Tensor& rh, const at::Tensor& dhn,
                                 const at::Tensor& wz, const at::Tensor& wr, const at::Tensor& wc, at::Tensor& gwz,
                                 at::Tensor& gbz, at::Tensor& gwr, at::Tensor& gbr, at::Tensor& gwc,
                                 at::Tensor& gbc);
void spmm_peer_push(const at::Tensor& rowptr_t, const at::Tensor& col_t, const at::Tensor& val_t,
                    const at::Tensor& grad_dst, int64_t n_src, const at::Tensor& peers, const at::Tensor& src_owner,
                    const at::Tensor& src_row, int64_t ld, const c10::optional<std::vector<at::Tensor>>& plan);

void tgn_rnn_memory_update(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& mailbox,
                           at::Tensor& memory, at::Tensor& memory_ts, const at::Tensor& ts_max,
                           const at::Tensor& w_ih, const at::Tensor& w_hh, const at::Tensor& b_ih,
                           const at::Tensor& b_hh, at::Tensor& mem_prev, at::Tensor& prev_ts,
                           const c10::optional<at::Tensor>& peer);
void jodie_project(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& memory,
                   const at::Tensor& prev_ts, const at::Tensor& root_ts, double dt_scale, const at::Tensor& w,
                   const at::Tensor& b, at::Tensor& out, at::Tensor& dt, const c10::optional<at::Tensor>& peer);
void jodie_project_bwd(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& memory,
                       const at::Tensor& dt, const at::Tensor& dz, at::Tensor& dw, at::Tensor& db,
                       const c10::optional<at::Tensor>& peer);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "starry_unigraph sm_100a kernels (tcgen05 GEMMs, TGN step, DTDG ops, collectives)";
  m.def("status_read", &status_read, "read (and clear) the device status word", py::arg("clear") = true);
  m.def("launch_count", &su::launch_count, "kernel launches issued by this library so far (host-side count)");
  m.def("set_gemm_precision", &su::set_gemm_precision, "tensor-core operand precision of the GEMMs: tf32 or bf16",
        py::arg("tf32"));
  m.def("gemm_precision_tf32", &su::gemm_precision_tf32);
  m.def("set_tma_store_min_rows", &su::set_tma_store_min_rows,
        "packed GEMMs with plain fp32 outputs of at least this many rows store tiles with TMA (negative: never)");
  m.def("tma_store_min_rows", &su::tma_store_min_rows);
  su::set_workspace_allocator(&su_ws_alloc, &su_ws_free);
  m.def("linear_fwd", &linear_fwd);
  m.def("linear_fwd_into", &linear_fwd_into);
  m.def("linear_dgrad", &linear_dgrad, py::arg("dy"), py::arg("w"), py::arg("mask") = py::none());
  m.def("linear_wgrad", &linear_wgrad, py::arg("dy"), py::arg("x"), py::arg("dw"), py::arg("db"),
        py::arg("mask") = py::none());
  m.def("tgn_prep", &tgn_prep);
  m.def("tgn_sample", &tgn_sample);
  m.def("tgn_memory_update", &tgn_memory_update);
  m.def("tgn_mailbox_write", &tgn_mailbox_write);
  m.def("tgn_rnn_memory_update", &tgn_rnn_memory_update);
  m.def("jodie_project", &jodie_project);
  m.def("jodie_project_bwd", &jodie_project_bwd);
  m.def("tgn_attn_proj", &tgn_attn_proj);
  m.def("tgn_attn_fwd", &tgn_attn_fwd);
  m.def("tgn_attn_bwd", &tgn_attn_bwd);
  m.def("tgn_out_fwd", &tgn_out_fwd);
  m.def("tgn_out_bwd", &tgn_out_bwd);
  m.def("tgn_attn_proj_bwd", &tgn_attn_proj_bwd);
  m.def("tgn_out_proj_bwd", &tgn_out_proj_bwd);
  m.def("tgn_link_proj", &tgn_link_proj);
  m.def("tgn_link_loss", &tgn_link_loss);
  m.def("tgn_metrics", &tgn_metrics);
  m.def("tgn_link_proj_bwd", &tgn_link_proj_bwd);
  m.def("adam_flat", &adam_flat);
  m.def("peer_barrier", &peer_barrier);
  m.def("peer_allreduce_adam", &peer_allreduce_adam);
  m.def("tgn_peer_writeback", &tgn_peer_writeback, py::arg("roots"), py::arg("n_roots"), py::arg("mem_new"),
        py::arg("owner"), py::arg("mem_ptrs"), py::arg("ts_ptrs"), py::arg("ts_max"), py::arg("cache") = py::none(),
        py::arg("thresh") = 0.5, py::arg("rank") = 0);
  m.def("tgn_peer_mail_claim", &tgn_peer_mail_claim);
  m.def("tgn_peer_mail_write", &tgn_peer_mail_write);
  m.def("peer_signal", &peer_signal);
  m.def("peer_wait", &peer_wait);
  m.def("tgn_peer_wait_claim", &tgn_peer_wait_claim);
  m.def("tgn_peer_push", &tgn_peer_push, py::arg("roots"), py::arg("n_roots"), py::arg("mem_new"), py::arg("ts_max"),
        py::arg("owner"), py::arg("mem_ptrs"), py::arg("ts_ptrs"), py::arg("cache"), py::arg("thresh"),
        py::arg("rank"), py::arg("win"), py::arg("src_idx"), py::arg("dst_idx"), py::arg("ev_eid"), py::arg("ev_ts"),
        py::arg("mem_prev"), py::arg("efeat"), py::arg("E"), py::arg("claim_ptrs"), py::arg("mail_ptrs") = py::none(),
        py::arg("mail_ts_ptrs") = py::none());
  m.def("peer_rs_adam_ag", &peer_rs_adam_ag);
  m.def("spmm_csr", &spmm_csr, py::arg("rowptr"), py::arg("col"), py::arg("val"), py::arg("x"), py::arg("n_rows"),
        py::arg("out") = py::none(), py::arg("accumulate") = false, py::arg("plan") = py::none());
  m.def("spmm_plan_warps", &spmm_plan_warps_op, "warps of the item-based SpMM grid on the current device");
  m.def("spmm_peer_gather", &spmm_peer_gather);
  m.def("spmm_peer_push", &spmm_peer_push, py::arg("rowptr_t"), py::arg("col_t"), py::arg("val_t"),
        py::arg("grad_dst"), py::arg("n_src"), py::arg("peers"), py::arg("src_owner"), py::arg("src_row"),
        py::arg("ld") = -1, py::arg("plan") = py::none());
  m.def("halo_pull", &halo_pull, py::arg("peers"), py::arg("src_owner"), py::arg("src_row"), py::arg("halo_src"),
        py::arg("F"), py::arg("ld") = -1);
  m.def("rgru_fwd", &rgru_fwd);
  m.def("rgru_bwd", &rgru_bwd);
  m.def("spmm_two_tables", &spmm_two_tables, py::arg("rowptr"), py::arg("col"), py::arg("val"), py::arg("x"),
        py::arg("halo"), py::arg("n_rows"), py::arg("plan") = py::none());
  m.def("lstm_fwd", &lstm_fwd);
  m.def("lstm_bwd", &lstm_bwd);
}
