// Instantiations of the tcgen05 GEMM for every (producer, producer, epilogue)
// combination used by the framework, and the per-device bookkeeping
// (status word, SM count). The N tile is chosen from the output width.
#include <algorithm>
#include <cstdio>

#include "kernels.h"

namespace su {

static int* g_status[64] = {nullptr};
static int g_sms[64] = {0};

int* device_status_ptr(int device) {
  if (g_status[device] == nullptr) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    if (cudaMalloc(&g_status[device], sizeof(int) * 4) != cudaSuccess) {
      fprintf(stderr, "starry_unigraph: status word allocation failed\n");
      g_status[device] = nullptr;
    } else {
      cudaMemset(g_status[device], 0, sizeof(int) * 4);
    }
    cudaSetDevice(prev);
  }
  return g_status[device];
}

int num_sms(int device) {
  if (g_sms[device] == 0) {
    cudaDeviceGetAttribute(&g_sms[device], cudaDevAttrMultiProcessorCount, device);
    if (g_sms[device] <= 0) g_sms[device] = 148;
  }
  return g_sms[device];
}

template <int BN, int NSUB, class A, class B, class E>
static void launch_cfg(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st) {
  constexpr int smem = gemm_smem_bytes<BN, NSUB>();
  auto kern = tc_gemm_kernel<BN, NSUB, A, B, E>;
  int device = 0;
  cudaGetDevice(&device);
  static unsigned long long configured = 0ull;
  if (!(configured & (1ull << device))) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured |= (1ull << device);
  }
  const int tiles_m = (sh.M + kBM - 1) / kBM;
  const int tiles_n = (sh.N + BN * NSUB - 1) / (BN * NSUB);
  const int total = tiles_m * tiles_n * std::max(1, sh.ksplit);
  if (total <= 0) return;
  const int per_sm = (smem <= 100 * 1024) ? 2 : 1;
  const int grid = std::min(total, num_sms(device) * per_sm);
  kern<<<grid, kGemmThreads, smem, st>>>(a, b, e, sh, device_status_ptr(device));
}

// launch_cfg with an explicit status word; setup (the shared-memory attribute,
// the SM count) allocates nothing.
template <int BN, int NSUB, class A, class B, class E>
static void launch_cfg_status(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st,
                              int* status) {
  constexpr int smem = gemm_smem_bytes<BN, NSUB>();
  auto kern = tc_gemm_kernel<BN, NSUB, A, B, E>;
  int device = 0;
  cudaGetDevice(&device);
  static unsigned long long configured = 0ull;
  if (!(configured & (1ull << device))) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured |= (1ull << device);
  }
  const int tiles_m = (sh.M + kBM - 1) / kBM;
  const int tiles_n = (sh.N + BN * NSUB - 1) / (BN * NSUB);
  const int total = tiles_m * tiles_n * std::max(1, sh.ksplit);
  if (total <= 0) return;
  const int per_sm = (smem <= 100 * 1024) ? 2 : 1;
  const int grid = std::min(total, num_sms(device) * per_sm);
  kern<<<grid, kGemmThreads, smem, st>>>(a, b, e, sh, status);
}

template <class A, class B, class E>
static void dispatch_status(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st, int* status) {
  if (sh.N <= 128) launch_cfg_status<128, 1>(a, b, e, sh, st, status);
  else if (sh.N <= 256) launch_cfg_status<256, 1>(a, b, e, sh, st, status);
  else launch_cfg_status<256, 2>(a, b, e, sh, st, status);
}

void gemm_with_status(const SegSource& a, const MNView<WeightSource>& b, const EpiLinear& e, const GemmShape& sh,
                      cudaStream_t st, int* status) {
  dispatch_status(a, b, e, sh, st, status);
}
void gemm_with_status(const MNView<SegSource>& a, const MNView<SegSource>& b, const EpiWeightGrad& e,
                      const GemmShape& sh, cudaStream_t st, int* status) {
  dispatch_status(a, b, e, sh, st, status);
}

template <class A, class B, class E>
static void dispatch(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st) {
  if (sh.N <= 128) launch_cfg<128, 1>(a, b, e, sh, st);
  else if (sh.N <= 256) launch_cfg<256, 1>(a, b, e, sh, st);
  else launch_cfg<256, 2>(a, b, e, sh, st);
}

void gemm(const SegSource& a, const WeightSource& b, const EpiLinear& e, const GemmShape& sh, cudaStream_t st) {
  dispatch(a, b, e, sh, st);
}
void gemm(const SegSource& a, const MNView<WeightSource>& b, const EpiLinear& e, const GemmShape& sh,
          cudaStream_t st) {
  dispatch(a, b, e, sh, st);
}
void gemm(const MNView<SegSource>& a, const MNView<SegSource>& b, const EpiWeightGrad& e, const GemmShape& sh,
          cudaStream_t st) {
  dispatch(a, b, e, sh, st);
}
void gemm(const SegSource& a, const WeightSource& b, const EpiGRU& e, const GemmShape& sh, cudaStream_t st) {
  launch_cfg<128, 1>(a, b, e, sh, st);  // one tile = four gates x 32 hidden units (gate-grouped rows)
}
void gemm(const SegSource& a, const WeightSource& b, const EpiOutLN& e, const GemmShape& sh, cudaStream_t st) {
  if (sh.N <= 128) launch_cfg<128, 1>(a, b, e, sh, st);
  else launch_cfg<256, 1>(a, b, e, sh, st);
}

void gemm(const SegSource& a, const WeightSource& b, const EpiLSTM& e, const GemmShape& sh, cudaStream_t st) {
  launch_cfg<128, 1>(a, b, e, sh, st);  // one tile = four gates x 32 hidden units (gate-grouped rows)
}

}  // namespace su
