// Declarations shared by the CUDA translation units (nvcc) and the torch-side
// wrappers (g++). Nothing here depends on torch headers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "epilogues.cuh"
#include "tc_gemm.cuh"

namespace su {

// ---- device bookkeeping -----------------------------------------------------
int* device_status_ptr(int device);  // per-device status word (bounded waits, bad indices)
// Stream-ordered allocator for GEMM operand images (nullptr: internal workspaces).
using WorkspaceAlloc = void* (*)(size_t bytes, cudaStream_t stream);
using WorkspaceFree = void (*)(void* ptr);
void set_workspace_allocator(WorkspaceAlloc alloc, WorkspaceFree free_fn);
// Host-side count of kernel launches issued by this library (all devices).
void count_launch();
long long launch_count();
int num_sms(int device);
// Operand precision of the tcgen05 GEMMs issued from this thread (a GemmShape
// may also ask for tf32 itself): bf16 (default) or tf32.
void set_gemm_precision(bool tf32);
bool gemm_precision_tf32();
// Packed GEMMs with plain fp32 outputs and at least this many rows store their
// tiles with TMA (negative: never).
void set_tma_store_min_rows(int rows);
int tma_store_min_rows();

// ---- tcgen05 GEMM entry points (one overload per producer/epilogue combo) ---
void gemm(const SegSource& a, const WeightSource& b, const EpiLinear& e, const GemmShape& sh, cudaStream_t st);
void gemm(const SegSource& a, const MNView<WeightSource>& b, const EpiLinear& e, const GemmShape& sh,
          cudaStream_t st);
void gemm(const MNView<SegSource>& a, const MNView<SegSource>& b, const EpiWeightGrad& e, const GemmShape& sh,
          cudaStream_t st);
void gemm(const SegSource& a, const WeightSource& b, const EpiGRU& e, const GemmShape& sh, cudaStream_t st);
void gemm(const SegSource& a, const WeightSource& b, const EpiOutLN& e, const GemmShape& sh, cudaStream_t st);
// Same kernels, reporting into a caller-given device status word instead of the
// lazily allocated per-device one (used by entry points that must not allocate).
void gemm_with_status(const SegSource& a, const MNView<WeightSource>& b, const EpiLinear& e, const GemmShape& sh,
                      cudaStream_t st, int* status);
void gemm_with_status(const MNView<SegSource>& a, const MNView<SegSource>& b, const EpiWeightGrad& e,
                      const GemmShape& sh, cudaStream_t st, int* status);
void launch_time_grad_finish(cudaStream_t st, const float* wk, const float* wv, int ldw, int ct, const float* wq,
                             int ldq, int cq, int Do, int T, const float* Mt, const float* M1, const float* gbq,
                             const float* b, float* dw, float* db);

// ---- TGN step kernels --------------------------------------------------------
struct PrepArgs {
  const int64_t* src;
  const int64_t* dst;
  const float* ts;
  const int* n_ev;
  int bmax;
  int rmax;
  const int64_t* neg_pool;
  int64_t pool_size;
  int* stamp;          // [num_nodes]
  int* node2root;      // [num_nodes]
  int64_t* step_ctr;   // [1]
  uint64_t seed;
  int64_t* roots;      // [rmax]
  int* n_roots;        // [1]
  int* src_idx;        // [bmax]
  int* dst_idx;        // [bmax]
  int64_t* neg;        // [bmax]
  int* neg_idx;        // [bmax]
  float* ts_max;       // [1]
  int64_t* root_ts;    // [1]  (int64-truncated max timestamp, sampler query time)
  unsigned long long* win_key;  // [2 * rmax]
  int* win;            // [2 * rmax]  event index of the last message (src pass, dst pass)
  int* cnt;            // [2 * rmax]
  int* status;
};

void launch_tgn_prep(dim3 grid, dim3 block, cudaStream_t st, PrepArgs a);
void launch_tgn_sample(dim3 grid, dim3 block, cudaStream_t st, const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                  const int64_t* __restrict__ root_ts_scalar, const int64_t* __restrict__ root_ts_vec,
                                  const int64_t* __restrict__ rowptr, const int64_t* __restrict__ nbr,
                                  const int64_t* __restrict__ eid, const int64_t* __restrict__ ets, int k, int policy,
                                  uint64_t seed, const int64_t* __restrict__ step_ctr, int64_t* __restrict__ out_nbr,
                                  int64_t* __restrict__ out_eid, float* __restrict__ out_dt,
                                  int* __restrict__ out_cnt, int* __restrict__ edge_total);
void launch_tgn_mailbox(dim3 grid, dim3 block, cudaStream_t st, const int64_t* __restrict__ roots, const int* __restrict__ n_roots, int rmax,
                                   const int* __restrict__ win, const int* __restrict__ cnt,
                                   const int* __restrict__ src_idx, const int* __restrict__ dst_idx,
                                   const int64_t* __restrict__ ev_eid, const float* __restrict__ ev_ts,
                                   const float* __restrict__ mem_prev, int D, const void* __restrict__ efeat,
                                   int efeat_bf16, int efeat_ld, int e_raw, int E, float* __restrict__ mailbox,
                                   float* __restrict__ mailbox_ts, int64_t* __restrict__ next_pos, int K);
void launch_tgn_attn_fwd(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ Q, const float* __restrict__ KV,
                                    const int* __restrict__ cnt, const int* __restrict__ n_roots, int rmax, int k,
                                    int Do, int H, float att_drop, uint64_t seed, const int64_t* __restrict__ step_ctr,
                                    float* __restrict__ att_p, float* __restrict__ agg);
void launch_tgn_attn_bwd(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ Q, const float* __restrict__ KV,
                                    const float* __restrict__ att_p, const float* __restrict__ dagg,
                                    const int* __restrict__ cnt, const int* __restrict__ n_roots, int rmax, int k,
                                    int Do, int H, float att_drop, uint64_t seed, const int64_t* __restrict__ step_ctr,
                                    float* __restrict__ dKV, float* __restrict__ dQ);
void launch_tgn_out_bwd(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ dout, const float* __restrict__ xsave,
                                   const float* __restrict__ mean, const float* __restrict__ rstd,
                                   const float* __restrict__ gamma, const int* __restrict__ n_roots, int rmax, int Do,
                                   float drop, uint64_t seed, const int64_t* __restrict__ step_ctr,
                                   const int* __restrict__ edge_total, float* __restrict__ dpre,
                                   float* __restrict__ dgamma, float* __restrict__ dbeta);
void launch_tgn_link(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ P, const int* __restrict__ src_idx,
                                const int* __restrict__ dst_idx, const int* __restrict__ neg_idx,
                                const int* __restrict__ n_ev, int bmax, int D, const float* __restrict__ b_dst,
                                const float* __restrict__ w_out, const float* __restrict__ b_out, int need_grad,
                                float* __restrict__ scores, float* __restrict__ loss, float* __restrict__ dP,
                                float* __restrict__ g_w_out, float* __restrict__ g_b_out, float* __restrict__ g_b_dst);
void launch_tgn_metrics(dim3 grid, dim3 block, cudaStream_t st, const float* __restrict__ scores,
                                                           const int* __restrict__ n_ev, int bmax,
                                                           float* __restrict__ out);

// ---- JODIE time projection ---------------------------------------------------
void launch_jodie_prev_ts(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const float* mem_ts,
                          const float* const* ts_peers, const int* owner, float* prev_ts);
void launch_jodie_project(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const float* mem,
                          const float* fresh, int D, const float* prev_ts, const int64_t* root_ts, float dt_scale,
                          const float* w, const float* b, float* out, float* dt_out);
void launch_jodie_project_bwd(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const float* mem,
                              const float* fresh, int D, const float* dt, const float* dz, float* dw, float* db);

// ---- DTDG ---------------------------------------------------------------------
void gemm(const SegSource& a, const WeightSource& b, const EpiLSTM& e, const GemmShape& sh, cudaStream_t st);
// GEMMs whose A image a kernel of the caller wrote (packed path only): false, with
// nothing launched, when that path is disabled or its workspace is unavailable
bool gemm_prepacked(const Prepacked<false>& a, const MNView<WeightSource>& b, const EpiLinear& e, const GemmShape& sh,
                    cudaStream_t st);
bool gemm_prepacked(const Prepacked<true>& a, const MNView<SegSource>& b, const EpiWeightGrad& e, const GemmShape& sh,
                    cudaStream_t st);
bool packed_gemm_enabled();
void gemm(const SegSource& a, const WeightSource& b, const EpiRGruZR& e, const GemmShape& sh, cudaStream_t st);
void gemm(const SegSource& a, const WeightSource& b, const EpiRGruOut& e, const GemmShape& sh, cudaStream_t st);
// reset-gated GRU cell backward, elementwise parts (dtdg_kernels.cu)
void launch_rgru_bwd1(cudaStream_t st, const float* dhn, int dhn_ld, const float* h, int h_ld, const float* z,
                      const float* c, int64_t rows, int H, float* dzr, float* dc_pre, float* dh_acc);
void launch_rgru_bwd2(cudaStream_t st, const float* drh, int drh_ld, const float* h, int h_ld, const float* r,
                      int64_t rows, int H, float* dzr, float* dh_acc);
void launch_add_rows(cudaStream_t st, const float* a, const float* b, int b_ld, int64_t rows, int H, float* out);
// Work plan of the item-based SpMM (F = 64): rows cut into items of at most a
// fixed edge count, runs of items per warp of a fixed grid. Built on the device
// once per CSR (starry_unigraph.data.partition.spmm_plan).
struct SpmmPlan {
  const int* items = nullptr;       // [3][n_items]: row (-row - 1 when split over items), first edge, end edge
  int n_items = 0;
  const int* warp_off = nullptr;    // [warps + 1] item offsets
  int warps = 0;
  const int* split_rows = nullptr;  // rows split over several items (zeroed before their atomic adds)
  int n_split = 0;
};
int spmm_plan_warps(int device);
void launch_spmm_csr(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val, const float* x,
                     int64_t n_rows, int F, float* out, int accumulate, const SpmmPlan* plan = nullptr);
void launch_spmm_peer_gather(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val,
                             const float* const* peers, const int* src_owner, const int* src_row, int64_t n_rows,
                             int F, float* out);
// DTDG halo, pull-once form: unique halo rows copied from the owners' staging
// buffers (P2P loads), then the aggregation over [local rows | halo rows]
void launch_halo_pull(cudaStream_t st, const float* const* peers, const int* owner, const int* lrow,
                      const int* halo_src, int64_t n_halo, int F, int ld, float* out);
void launch_spmm_two_tables(cudaStream_t st, const int64_t* rowptr, const int* col, const float* val, const float* x,
                            int x_ld, const float* halo, int n_split, int64_t n_rows, int F, float* out,
                            const SpmmPlan* plan = nullptr);
void launch_spmm_peer_push(cudaStream_t st, const int64_t* rowptr_t, const int* col_t, const float* val_t,
                           const float* grad_dst, int64_t n_src, int F, int ld, float* const* peers,
                           const int* src_owner, const int* src_row, const SpmmPlan* plan = nullptr);
void launch_lstm_bwd(cudaStream_t st, const float* gates, const float* c_prev, const float* c_new, const float* dh,
                     int dh_ld, const float* dc, int dc_ld, int64_t rows, int H, float* dpre, float* dc_prev);
// gate gradients written as the K-major image of dpre (the input-gradient GEMM's A)
// and the MN-major image of dpre^T (the weight-gradient GEMM's A); H % 32 == 0,
// every pointer 16-byte aligned, dh_ld and dc_ld multiples of 4
void launch_lstm_bwd_pack(cudaStream_t st, const float* gates, const float* c_prev, const float* c_new,
                          const float* dh, int dh_ld, const float* dc, int dc_ld, int64_t rows, int H, uint8_t* img_k,
                          uint8_t* img_mn, float* dc_prev);
// vectorised form with bf16 pre-activation gradients; requires lstm_bwd_bf16_ok()
bool lstm_bwd_bf16_ok(const float* gates, const float* c_prev, const float* c_new, const float* dh, int dh_ld,
                      const float* dc, int dc_ld, int H, const void* dpre, const float* dc_prev);
void launch_lstm_bwd_bf16(cudaStream_t st, const float* gates, const float* c_prev, const float* c_new,
                          const float* dh, int dh_ld, const float* dc, int dc_ld, int64_t rows, int H,
                          __nv_bfloat16* dpre, float* dc_prev);

// ---- peer (NVLink) kernels -----------------------------------------------------
void launch_peer_barrier(cudaStream_t st, uint64_t* const* flag_ptrs, int rank, int W, int64_t* epoch, int* status,
                         long long budget);
void launch_peer_allreduce_adam(cudaStream_t st, int blocks, const float* const* grads, int W, float* p, float* m,
                                float* v, int64_t n, int64_t* step, unsigned int* done, float lr, float b1, float b2,
                                float eps, float wd, float scale);
// historical-cache filter of the write-back (cache == nullptr: push every row)
struct HistCache {
  const int64_t* slot_of = nullptr;  // global node id -> cache row (-1: owned here, no filter)
  float* cache = nullptr;            // [shared nodes, D] last pushed rows
  float* cache_ts = nullptr;         // [shared nodes] ts of the last push (< 0: never pushed)
  float thresh = 0.5f;               // push when 1 - cos(new, cached) > thresh
  int rank = 0;
};
void launch_tgn_peer_writeback(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax,
                               const float* mem_new, int D, const int* owner, float* const* mem_tables,
                               float* const* ts_tables, const float* ts_max, const HistCache& hc);
void launch_tgn_peer_mail_claim(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const int* win,
                                const int64_t* ev_eid, const float* ev_ts, const int* owner,
                                unsigned long long* const* claim_tables);
void launch_tgn_peer_mail_write(cudaStream_t st, const int64_t* roots, const int* n_roots, int rmax, const int* win,
                                const int* src_idx, const int* dst_idx, const int64_t* ev_eid, const float* ev_ts,
                                const float* mem_prev, int D, const void* efeat, int efeat_bf16, int efeat_ld,
                                int e_raw, int E, const int* owner, const unsigned long long* const* claim_tables,
                                float* const* mail_tables, float* const* mail_ts_tables);
// split end-of-step barrier: signal now, wait (fused with the next step's claims) later
void launch_peer_signal(cudaStream_t st, uint64_t* const* flag_ptrs, int rank, int W, int64_t* epoch);
void launch_peer_wait(cudaStream_t st, const uint64_t* my_flags, int rank, int W, const int64_t* epoch, int* status,
                      long long budget);
void launch_tgn_peer_wait_claim(cudaStream_t st, const uint64_t* my_flags, int rank, int W, const int64_t* epoch,
                                int* status, long long budget, const int64_t* roots, const int* n_roots, int rmax,
                                const int* win, const int64_t* ev_eid, const float* ev_ts, const int* owner,
                                unsigned long long* const* claim_tables);
// memory write-back + mailbox write of the claim winners (mail_tables == nullptr: memory only)
void launch_tgn_peer_push(cudaStream_t st, int blocks, const int64_t* roots, const int* n_roots, int rmax,
                          const float* mem_new, const float* ts_max, float* const* mem_tables,
                          float* const* ts_tables, const HistCache& hc, const int* win, const int* src_idx,
                          const int* dst_idx, const int64_t* ev_eid, const float* ev_ts, const float* mem_prev, int D,
                          const void* efeat, int efeat_bf16, int efeat_ld, int e_raw, int E, const int* owner,
                          const unsigned long long* const* claim_tables, float* const* mail_tables,
                          float* const* mail_ts_tables);
// reduce-scatter + Adam on this rank's shard + all-gather of the new parameters
void launch_peer_rs_adam_ag(cudaStream_t st, int blocks, const float* const* grads, float* const* params, int W,
                            int rank, float* m, float* v, int64_t n, int64_t* step, unsigned int* done, float lr,
                            float b1, float b2, float eps, float wd, float scale);

// ---- optimiser ---------------------------------------------------------------
void launch_adam_flat(cudaStream_t st, int blocks, float* p, const float* g, float* m, float* v, int64_t n,
                      int64_t* step, unsigned int* done, float lr, float b1, float b2, float eps, float wd,
                      float grad_scale);

}  // namespace su
