// Torch-side wrapper of the fused flat Adam kernel.
#include "host_common.h"

using namespace su;

void adam_flat(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, at::Tensor& step, at::Tensor& done,
               double lr, double b1, double b2, double eps, double wd, double grad_scale) {
  SU_CHECK_F32(p); SU_CHECK_F32(g); SU_CHECK_CONTIG(p); SU_CHECK_CONTIG(g);
  const int64_t n = p.numel();
  if (n == 0) return;
  const int threads = 256;
  const int64_t want = (n / 4 + threads - 1) / threads;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, num_sms(at::cuda::current_device()) * 4)));
  launch_adam_flat(cur_stream(), blocks, p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                   v.data_ptr<float>(), n, step.data_ptr<int64_t>(),
                   reinterpret_cast<unsigned int*>(done.data_ptr<int>()), static_cast<float>(lr),
                   static_cast<float>(b1), static_cast<float>(b2), static_cast<float>(eps), static_cast<float>(wd),
                   static_cast<float>(grad_scale));
  SU_LAUNCH_CHECK();
}
