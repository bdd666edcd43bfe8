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

void tgn_peer_mail_write(const at::Tensor& roots, const at::Tensor& n_roots, const at::Tensor& win,
                         const at::Tensor& src_idx, const at::Tensor& dst_idx, const at::Tensor& ev_eid,
                         const at::Tensor& ev_ts, const at::Tensor& mem_prev, const at::Tensor& efeat, int64_t E,
                         const at::Tensor& owner, const at::Tensor& claim_ptrs, const at::Tensor& mail_ptrs,
                         const at::Tensor& mail_ts_ptrs) {
  const int D = static_cast<int>(mem_prev.size(1));
  launch_tgn_peer_mail_write(cur_stream(), roots.data_ptr<int64_t>(), n_roots.data_ptr<int>(),
                             static_cast<int>(roots.numel()), win.data_ptr<int>(), src_idx.data_ptr<int>(),
                             dst_idx.data_ptr<int>(), ev_eid.data_ptr<int64_t>(), ev_ts.data_ptr<float>(),
                             mem_prev.data_ptr<float>(), D, efeat.data_ptr<float>(), static_cast<int>(efeat.stride(0)),
                             static_cast<int>(efeat.size(1)), static_cast<int>(E), owner.data_ptr<int>(),
                             table<const unsigned long long* const*>(claim_ptrs), table<float* const*>(mail_ptrs),
                             table<float* const*>(mail_ts_ptrs));
  SU_LAUNCH_CHECK();
}
