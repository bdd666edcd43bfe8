// Fused Adam over a flat fp32 parameter buffer (torch.optim.Adam semantics,
// L2 weight decay folded into the gradient as torch does), plus an optional
// pre-scale of the gradient (e.g. 1/world_size after a SUM all-reduce).
//
// The step counter lives on the device so a captured CUDA graph replays
// with correct bias correction: every block reads t = *step + 1 and the last
// block to finish advances the counter.
#include "kernels.h"

namespace su {

__global__ void adam_flat_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                 float* __restrict__ v, int64_t n, int64_t* __restrict__ step,
                                 unsigned int* __restrict__ done, float lr, float b1, float b2, float eps, float wd,
                                 float grad_scale) {
  const float t = static_cast<float>(*step + 1);
  const float bc1 = 1.f - powf(b1, t);
  const float bc2 = 1.f - powf(b2, t);
  const float step_size = lr / bc1;
  const float bc2_sqrt = sqrtf(bc2);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
  for (int64_t i0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i0 < n; i0 += stride) {
    if (i0 + 4 <= n && (reinterpret_cast<uintptr_t>(p + i0) % 16) == 0) {
      float4 pp = *reinterpret_cast<float4*>(p + i0);
      const float4 gg = *reinterpret_cast<const float4*>(g + i0);
      float4 mm = *reinterpret_cast<float4*>(m + i0);
      float4 vv = *reinterpret_cast<float4*>(v + i0);
      float* pa = &pp.x;
      const float* ga = &gg.x;
      float* ma = &mm.x;
      float* va = &vv.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float gr = ga[j] * grad_scale + wd * pa[j];
        ma[j] = b1 * ma[j] + (1.f - b1) * gr;
        va[j] = b2 * va[j] + (1.f - b2) * gr * gr;
        pa[j] -= step_size * ma[j] / (sqrtf(va[j]) / bc2_sqrt + eps);
      }
      *reinterpret_cast<float4*>(p + i0) = pp;
      *reinterpret_cast<float4*>(m + i0) = mm;
      *reinterpret_cast<float4*>(v + i0) = vv;
    } else {
      for (int64_t i = i0; i < min(n, i0 + 4); ++i) {
        float gr = g[i] * grad_scale + wd * p[i];
        m[i] = b1 * m[i] + (1.f - b1) * gr;
        v[i] = b2 * v[i] + (1.f - b2) * gr * gr;
        p[i] -= step_size * m[i] / (sqrtf(v[i]) / bc2_sqrt + eps);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      *step += 1;
      *done = 0u;
      __threadfence();
    }
  }
}

void launch_adam_flat(cudaStream_t st, int blocks, float* p, const float* g, float* m, float* v, int64_t n,
                      int64_t* step, unsigned int* done, float lr, float b1, float b2, float eps, float wd,
                      float grad_scale) {
  count_launch();
  adam_flat_kernel<<<blocks, 256, 0, st>>>(p, g, m, v, n, step, done, lr, b1, b2, eps, wd, grad_scale);
}

}  // namespace su
