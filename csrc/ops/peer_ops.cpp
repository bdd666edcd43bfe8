// Torch wrappers of the peer (NVLink) kernels. Pointer tables (`*_ptrs`) are
// device int64 tensors holding one device address per rank: the rank's base
// of a symmetric allocation as mapped into this process.
#include "host_common.h"

using namespace su;

template <class T>
static T table(const at::Tensor& t) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kLong && t.is_contiguous(), "pointer table must be cuda int64");
  return reinterpret_cast<T>(t.data_ptr<int64_t>());
}

void peer_barrier(const at::Tensor& flag_ptrs, int64_t rank, int64_t world, at::Tensor& epoch, int64_t budget) {
  TORCH_CHECK(world >= 1 && world <= 32 && flag_ptrs.numel() == world, "peer_barrier: 1 <= world <= 32");
  SU_CHECK_I64(epoch);
  launch_peer_barrier(cur_stream(), table<uint64_t* const*>(flag_ptrs), static_cast<int>(rank),
                      static_cast<int>(world), epoch.data_ptr<int64_t>(), device_status_ptr(epoch.get_device()),
                      static_cast<long long>(budget));
  SU_LAUNCH_CHECK();
}

void peer_allreduce_adam(const at::Tensor& grad_ptrs, int64_t world, at::Tensor& p, at::Tensor& m, at::Tensor& v,
                         at::Tensor& step, at::Tensor& done, double lr, double b1, double b2, double eps, double wd,
                         double scale) {
  SU_CHECK_F32(p); SU_CHECK_F32(m); SU_CHECK_F32(v);
  TORCH_CHECK(p.numel() % 4 == 0, "flat buffers are padded to a multiple of 4");
  const int64_t n = p.numel();
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(num_sms(p.get_device()) * 2,
                                                                               (n / 4 + 255) / 256)));
  launch_peer_allreduce_adam(cur_stream(), blocks, table<const float* const*>(grad_ptrs), static_cast<int>(world),
                             p.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), n,
                             step.data_ptr<int64_t>(), reinterpret_cast<unsigned int*>(done.data_ptr<int>()),
                             static_cast<float>(lr), static_cast<float>(b1), static_cast<float>(b2),
                             static_cast<float>(eps), static_cast<float>(wd), static_cast<float>(scale));
  SU_LAUNCH_CHECK();
}

// cache: optional (slot_of int64 [num_nodes], cache f32 [shared, D], cache_ts f32 [shared]) with
// threshold `thresh` = 1 - alpha and this rank's id: the historical-cache filter of the push
void tgn_peer_writeback(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& mem_new,
                        const at::Tensor& owner, const at::Tensor& mem_ptrs, const at::Tensor& ts_ptrs,
                        const at::Tensor& ts_max, const c10::optional<std::vector<at::Tensor>>& cache,
                        double thresh, int64_t rank) {
  SU_CHECK_I64(roots); SU_CHECK_I32(owner); SU_CHECK_F32(mem_new);
  HistCache hc;
  if (cache.has_value() && !cache->empty()) {
    TORCH_CHECK(cache->size() == 3, "historical cache: (slot_of, cache, cache_ts)");
    const at::Tensor& slot_of = (*cache)[0];
    const at::Tensor& rows = (*cache)[1];
    const at::Tensor& ts = (*cache)[2];
    SU_CHECK_I64(slot_of); SU_CHECK_F32(rows); SU_CHECK_F32(ts); SU_CHECK_CONTIG(rows);
    TORCH_CHECK(rows.size(1) == mem_new.size(1), "historical cache rows must have the memory width");
    hc.slot_of = slot_of.data_ptr<int64_t>();
    hc.cache = rows.data_ptr<float>();
    hc.cache_ts = ts.data_ptr<float>();
    hc.thresh = static_cast<float>(thresh);
    hc.rank = static_cast<int>(rank);
  }
  launch_tgn_peer_writeback(cur_stream(), roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(),
                            static_cast<int>(roots.numel()), mem_new.data_ptr<float>(),
                            static_cast<int>(mem_new.size(1)), owner.data_ptr<int>(), table<float* const*>(mem_ptrs),
                            table<float* const*>(ts_ptrs), ts_max.data_ptr<float>(), hc);
  SU_LAUNCH_CHECK();
}

void tgn_peer_mail_claim(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& win,
                         const at::Tensor& ev_eid, const at::Tensor& ev_ts, const at::Tensor& owner,
                         const at::Tensor& claim_ptrs) {
  launch_tgn_peer_mail_claim(cur_stream(), roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(),
                             static_cast<int>(roots.numel()), win.data_ptr<int>(), ev_eid.data_ptr<int64_t>(),
                             ev_ts.data_ptr<float>(), owner.data_ptr<int>(),
                             table<unsigned long long* const*>(claim_ptrs));
  SU_LAUNCH_CHECK();
}

static int efeat_is_bf16(const at::Tensor& efeat) {
  TORCH_CHECK(efeat.is_cuda() && efeat.dim() == 2 && efeat.stride(1) == 1, "edge features: cuda [E, F], unit stride");
  TORCH_CHECK(efeat.scalar_type() == at::kFloat || efeat.scalar_type() == at::kBFloat16,
              "edge features must be float32 or bfloat16");
  return efeat.scalar_type() == at::kBFloat16 ? 1 : 0;
}

void tgn_peer_mail_write(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& win,
                         const at::Tensor& src_idx, const at::Tensor& dst_idx, const at::Tensor& ev_eid,
                         const at::Tensor& ev_ts, const at::Tensor& mem_prev, const at::Tensor& efeat, int64_t E,
                         const at::Tensor& owner, const at::Tensor& claim_ptrs, const at::Tensor& mail_ptrs,
                         const at::Tensor& mail_ts_ptrs) {
  const int D = static_cast<int>(mem_prev.size(1));
  const int bf = efeat_is_bf16(efeat);
  launch_tgn_peer_mail_write(cur_stream(), roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(),
                             static_cast<int>(roots.numel()), win.data_ptr<int>(), src_idx.data_ptr<int>(),
                             dst_idx.data_ptr<int>(), ev_eid.data_ptr<int64_t>(), ev_ts.data_ptr<float>(),
                             mem_prev.data_ptr<float>(), D, efeat.data_ptr(), bf, static_cast<int>(efeat.stride(0)),
                             static_cast<int>(efeat.size(1)), static_cast<int>(E), owner.data_ptr<int>(),
                             table<const unsigned long long* const*>(claim_ptrs), table<float* const*>(mail_ptrs),
                             table<float* const*>(mail_ts_ptrs));
  SU_LAUNCH_CHECK();
}

void peer_signal(const at::Tensor& flag_ptrs, int64_t rank, int64_t world, at::Tensor& epoch) {
  TORCH_CHECK(world >= 1 && world <= 32 && flag_ptrs.numel() == world, "peer_signal: 1 <= world <= 32");
  SU_CHECK_I64(epoch);
  launch_peer_signal(cur_stream(), table<uint64_t* const*>(flag_ptrs), static_cast<int>(rank),
                     static_cast<int>(world), epoch.data_ptr<int64_t>());
  SU_LAUNCH_CHECK();
}

// Waits (bounded) until every peer signalled this rank's current `epoch` into
// its flag array `my_flags`.
void peer_wait(const at::Tensor& my_flags, int64_t rank, int64_t world, const at::Tensor& epoch, int64_t budget) {
  TORCH_CHECK(world >= 1 && world <= 32 && my_flags.numel() >= world, "peer_wait: 1 <= world <= 32");
  SU_CHECK_I64(my_flags); SU_CHECK_I64(epoch);
  launch_peer_wait(cur_stream(), reinterpret_cast<const uint64_t*>(my_flags.data_ptr<int64_t>()),
                   static_cast<int>(rank), static_cast<int>(world), epoch.data_ptr<int64_t>(),
                   device_status_ptr(epoch.get_device()), static_cast<long long>(budget));
  SU_LAUNCH_CHECK();
}

// Waits until every peer signalled `epoch` into this rank's flag array
// `my_flags` (int64 [>= world]), then posts this step's mailbox claims.
void tgn_peer_wait_claim(const at::Tensor& my_flags, int64_t rank, int64_t world, const at::Tensor& epoch,
                         int64_t budget, const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& win,
                         const at::Tensor& ev_eid, const at::Tensor& ev_ts, const at::Tensor& owner,
                         const at::Tensor& claim_ptrs) {
  TORCH_CHECK(world >= 1 && world <= 32 && my_flags.numel() >= world, "tgn_peer_wait_claim: 1 <= world <= 32");
  SU_CHECK_I64(my_flags); SU_CHECK_I64(epoch); SU_CHECK_I64(roots); SU_CHECK_I32(owner);
  launch_tgn_peer_wait_claim(cur_stream(), reinterpret_cast<const uint64_t*>(my_flags.data_ptr<int64_t>()),
                             static_cast<int>(rank), static_cast<int>(world), epoch.data_ptr<int64_t>(),
                             device_status_ptr(epoch.get_device()), static_cast<long long>(budget),
                             roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(), static_cast<int>(roots.numel()),
                             win.data_ptr<int>(), ev_eid.data_ptr<int64_t>(), ev_ts.data_ptr<float>(),
                             owner.data_ptr<int>(), table<unsigned long long* const*>(claim_ptrs));
  SU_LAUNCH_CHECK();
}

// End-of-step push: memory write-back of every root (historical filter as in
// tgn_peer_writeback) and, when `mail_ptrs` is given, the mailbox slot of the
// roots whose claim won.
void tgn_peer_push(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& mem_new,
                   const at::Tensor& ts_max, const at::Tensor& owner, const at::Tensor& mem_ptrs,
                   const at::Tensor& ts_ptrs, const c10::optional<std::vector<at::Tensor>>& cache, double thresh,
                   int64_t rank, const at::Tensor& win, const at::Tensor& src_idx, const at::Tensor& dst_idx,
                   const at::Tensor& ev_eid, const at::Tensor& ev_ts, const at::Tensor& mem_prev,
                   const at::Tensor& efeat, int64_t E, const at::Tensor& claim_ptrs,
                   const c10::optional<at::Tensor>& mail_ptrs, const c10::optional<at::Tensor>& mail_ts_ptrs) {
  SU_CHECK_I64(roots); SU_CHECK_I32(owner); SU_CHECK_F32(mem_new); SU_CHECK_F32(mem_prev);
  HistCache hc;
  if (cache.has_value() && !cache->empty()) {
    TORCH_CHECK(cache->size() == 3, "historical cache: (slot_of, cache, cache_ts)");
    const at::Tensor& slot_of = (*cache)[0];
    const at::Tensor& rows = (*cache)[1];
    const at::Tensor& ts = (*cache)[2];
    SU_CHECK_I64(slot_of); SU_CHECK_F32(rows); SU_CHECK_F32(ts); SU_CHECK_CONTIG(rows);
    TORCH_CHECK(rows.size(1) == mem_new.size(1), "historical cache rows must have the memory width");
    hc.slot_of = slot_of.data_ptr<int64_t>();
    hc.cache = rows.data_ptr<float>();
    hc.cache_ts = ts.data_ptr<float>();
    hc.thresh = static_cast<float>(thresh);
    hc.rank = static_cast<int>(rank);
  }
  const int D = static_cast<int>(mem_new.size(1));
  const int rmax = static_cast<int>(roots.numel());
  const bool mail = mail_ptrs.has_value() && mail_ts_ptrs.has_value();
  const int bf = efeat_is_bf16(efeat);
  const int blocks = std::max(1, std::min(rmax, num_sms(mem_new.get_device()) * 8));
  launch_tgn_peer_push(cur_stream(), blocks, roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(), rmax,
                       mem_new.data_ptr<float>(), ts_max.data_ptr<float>(), table<float* const*>(mem_ptrs),
                       table<float* const*>(ts_ptrs), hc, win.data_ptr<int>(), src_idx.data_ptr<int>(),
                       dst_idx.data_ptr<int>(), ev_eid.data_ptr<int64_t>(), ev_ts.data_ptr<float>(),
                       mem_prev.data_ptr<float>(), D, efeat.data_ptr(), bf, static_cast<int>(efeat.stride(0)),
                       static_cast<int>(efeat.size(1)), static_cast<int>(E), owner.data_ptr<int>(),
                       table<const unsigned long long* const*>(claim_ptrs),
                       mail ? table<float* const*>(*mail_ptrs) : nullptr,
                       mail ? table<float* const*>(*mail_ts_ptrs) : nullptr);
  SU_LAUNCH_CHECK();
}

// Reduce-scatter + Adam + all-gather: rank `rank` reduces and updates its 1/W
// shard of the flat buffer and stores the new values into every rank's
// parameter buffer (`param_ptrs`). m / v hold valid moments for this rank's
// shard only.
void peer_rs_adam_ag(const at::Tensor& grad_ptrs, const at::Tensor& param_ptrs, int64_t world, int64_t rank,
                     const at::Tensor& p_local, at::Tensor& m, at::Tensor& v, at::Tensor& step, at::Tensor& done,
                     double lr, double b1, double b2, double eps, double wd, double scale) {
  SU_CHECK_F32(p_local); SU_CHECK_F32(m); SU_CHECK_F32(v);
  TORCH_CHECK(p_local.numel() % 4 == 0 && m.numel() == p_local.numel() && v.numel() == p_local.numel(),
              "flat buffers are padded to a multiple of 4 and of equal size");
  TORCH_CHECK(world >= 1 && grad_ptrs.numel() == world && param_ptrs.numel() == world, "pointer tables of W ranks");
  const int64_t n = p_local.numel();
  const int64_t shard4 = (n / 4 + world - 1) / world;
  // 256 threads x 4 float4 per block pass; up to four blocks per SM keep the NVLink loads in flight
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(num_sms(p_local.get_device()) * 4,
                                                                               (shard4 + 1023) / 1024)));
  launch_peer_rs_adam_ag(cur_stream(), blocks, table<const float* const*>(grad_ptrs), table<float* const*>(param_ptrs),
                         static_cast<int>(world), static_cast<int>(rank), m.data_ptr<float>(), v.data_ptr<float>(), n,
                         step.data_ptr<int64_t>(), reinterpret_cast<unsigned int*>(done.data_ptr<int>()),
                         static_cast<float>(lr), static_cast<float>(b1), static_cast<float>(b2),
                         static_cast<float>(eps), static_cast<float>(wd), static_cast<float>(scale));
  SU_LAUNCH_CHECK();
}
