// Instantiations of the tcgen05 GEMM for every (producer, producer, epilogue)
// combination used by the framework, and the per-device bookkeeping
// (status word, SM count). The N tile is chosen from the output width.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>

#include "kernels.h"
#include "tc_gemm_packed.cuh"

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

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

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
  count_launch();
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
  count_launch();
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

// ---------------------------------------------------------------------------
// packed-operand path: pack A, pack B (full-occupancy grids), then the
// bulk-copy-fed tcgen05 GEMM. The packed images live in a per-device
// workspace that grows outside stream capture only; a call that would need to
// grow it during capture runs the fused-producer kernel instead.
// ---------------------------------------------------------------------------
// One workspace per (device, stream): GEMMs issued concurrently on different
// streams (weight gradients overlapping data gradients) must not share images.
struct Workspace {
  cudaStream_t stream = nullptr;
  uint8_t* ptr = nullptr;
  size_t bytes = 0;
};
constexpr int kMaxStreamsPerDevice = 8;
static Workspace g_ws[64][kMaxStreamsPerDevice];

static uint8_t* workspace(int device, size_t bytes, cudaStream_t st) {
  Workspace* w = nullptr;
  for (int i = 0; i < kMaxStreamsPerDevice; ++i) {
    if (g_ws[device][i].ptr != nullptr && g_ws[device][i].stream == st) {
      w = &g_ws[device][i];
      break;
    }
  }
  if (w == nullptr) {
    for (int i = 0; i < kMaxStreamsPerDevice; ++i) {
      if (g_ws[device][i].ptr == nullptr) {
        w = &g_ws[device][i];
        w->stream = st;
        break;
      }
    }
  }
  if (w == nullptr) return nullptr;  // too many streams: the caller falls back to the fused-producer kernel
  if (bytes <= w->bytes) return w->ptr;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  if (cs != cudaStreamCaptureStatusNone) return nullptr;
  if (w->ptr != nullptr) {
    cudaDeviceSynchronize();  // earlier kernels may still read the old image
    cudaFree(w->ptr);
    w->ptr = nullptr;
    w->bytes = 0;
  }
  const size_t want = bytes + bytes / 2;
  void* p = nullptr;
  if (cudaMalloc(&p, want) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  w->ptr = static_cast<uint8_t*>(p);
  w->bytes = want;
  w->stream = st;
  return w->ptr;
}

// Optional stream-ordered allocator for the packed images (set by the torch
// extension to the caching allocator, which also serves stream capture from the
// graph's private pool). Without it the per-stream workspaces above are used.
static WorkspaceAlloc g_ws_alloc = nullptr;
static WorkspaceFree g_ws_free = nullptr;
void set_workspace_allocator(WorkspaceAlloc a, WorkspaceFree f) {
  g_ws_alloc = a;
  g_ws_free = f;
}

static bool packed_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("SU_GEMM_FUSED_PRODUCERS");
    v = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

template <int ROWS, class Src>
static void launch_pack(const Src& src, uint8_t* out, int mn, const int* mn_dev, int k, int device, cudaStream_t st) {
  const int tiles = (mn + ROWS - 1) / ROWS;
  const int nchunks = (k + kBK - 1) / kBK;
  const int64_t total = static_cast<int64_t>(tiles) * nchunks * ROWS * 8;
  if (total <= 0) return;
  const int64_t want = (total + 255) / 256;
  const int blocks = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(num_sms(device)) * 16));
  count_launch();
  pack_kernel<ROWS, Src><<<blocks, 256, 0, st>>>(src, out, tiles, nchunks, mn, mn_dev, mn);
}

// ---------------------------------------------------------------------------
// TMA-store epilogue selection (EpiLinear with plain fp32 stores, large M)
// ---------------------------------------------------------------------------
static int tma_rows_from_env() {
  const char* e = getenv("SU_TMA_STORE_MIN_ROWS");
  return e != nullptr ? atoi(e) : 2048;
}
static std::atomic<int> g_tma_store_min_rows{tma_rows_from_env()};
void set_tma_store_min_rows(int rows) { g_tma_store_min_rows.store(rows); }
int tma_store_min_rows() { return g_tma_store_min_rows.load(); }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      p = nullptr;
    }
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Tensor map of an fp32 [rows, cols] matrix with row stride `ld` elements for
// boxes of `box_cols` x 32 rows: 32 columns with the 128-byte swizzle, 16 with
// the 64-byte one. False when it cannot be encoded.
static bool encode_store_map(CUtensorMap* map, const float* base, int rows, int cols, int ld, int box_cols = 32) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr || rows <= 0 || cols <= 0 || (box_cols != 32 && box_cols != 16)) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld & 3) != 0) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * sizeof(float)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), 32};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, box_cols == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int NSUB, bool TF32, class A, class B, class E>
static bool launch_packed_impl(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st);

template <int BN, int NSUB, bool TF32, class A, class B, class E>
static bool launch_packed(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st) {
  if constexpr (std::is_same<E, EpiLinear>::value && NSUB == 1) {
    const int min_rows = g_tma_store_min_rows.load(std::memory_order_relaxed);
    if (min_rows >= 0 && sh.M >= min_rows && sh.m_dev == nullptr && sh.ksplit <= 1 && e.out != nullptr &&
        e.out_bf16 == nullptr && e.accumulate == 0 && e.scatter == nullptr && e.ncols > 0 &&
        (e.bias == nullptr || (reinterpret_cast<uintptr_t>(e.bias) & 15) == 0) &&
        (e.bias2 == nullptr || ((reinterpret_cast<uintptr_t>(e.bias2) & 15) == 0 && (e.bias_split & 3) == 0))) {
      EpiLinearTma t;
      if (encode_store_map(&t.tmap, e.out, sh.M, e.ncols, e.ldo)) {
        t.ncols = e.ncols;
        t.bias = e.bias;
        t.bias2 = e.bias2;
        t.bias_split = e.bias_split;
        t.act = e.act;
        t.scale = e.scale;
        return launch_packed_impl<BN, NSUB, TF32>(a, b, t, sh, st);
      }
    }
  }
  if constexpr (std::is_same<E, EpiLSTM>::value && NSUB == 1) {
    const int min_rows = g_tma_store_min_rows.load(std::memory_order_relaxed);
    if (min_rows >= 0 && sh.M >= min_rows && sh.m_dev == nullptr && e.vec && e.DP == kLstmGroup &&
        e.H % kLstmGroup == 0 && e.h_out != nullptr && e.c_out != nullptr) {
      EpiLSTM t = e;
      t.tma = 1;
      const int gcols = 64 * (e.H / kLstmGroup);
      if ((e.gates == nullptr || encode_store_map(&t.map_g, e.gates, sh.M, gcols, gcols, 32)) &&
          encode_store_map(&t.map_c, e.c_out, sh.M, e.H, e.H, 16) &&
          encode_store_map(&t.map_h, e.h_out, sh.M, e.H, e.H, 16))
        return launch_packed_impl<BN, NSUB, TF32>(a, b, t, sh, st);
    }
  }
  return launch_packed_impl<BN, NSUB, TF32>(a, b, e, sh, st);
}

template <int BN, int NSUB, bool TF32, class A, class B, class E>
static bool launch_packed_impl(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st) {
  constexpr int B_ROWS = BN * NSUB;
  constexpr int smem = packed_smem_bytes<BN, NSUB, E>();
  constexpr bool kPrepackedA = is_prepacked<A>::value;
  static_assert(!(TF32 && kPrepackedA), "pre-packed operand images are bf16");
  int device = 0;
  cudaGetDevice(&device);
  const size_t abytes = kPrepackedA ? 0 : packed_bytes(sh.M, sh.K, kBM, TF32);
  const size_t bbytes = packed_bytes(sh.N, sh.K, B_ROWS, TF32);
  if (packed_bytes(sh.M, sh.K, kBM, TF32) == 0 || bbytes == 0) return true;
  uint8_t* ws = g_ws_alloc ? static_cast<uint8_t*>(g_ws_alloc(abytes + bbytes, st)) : workspace(device, abytes + bbytes, st);
  if (ws == nullptr) return false;
  // tf32: both operands K-major (transposed sources are transposed by the pack kernel)
  auto kern = tc_gemm_packed_kernel<BN, NSUB, TF32 ? false : A::kMN, TF32 ? false : B::kMN, E, TF32>;
  static unsigned long long configured = 0ull;
  if (!(configured & (1ull << device))) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured |= (1ull << device);
  }
  // one launch packs both operands; the GEMM is launched with programmatic
  // stream serialisation so its prologue (barriers, TMEM) overlaps the packing
  const int nchunks = (sh.K + chunk_k(TF32) - 1) / chunk_k(TF32);
  const int tiles_a = (sh.M + kBM - 1) / kBM;
  const int tiles_b = (sh.N + B_ROWS - 1) / B_ROWS;
  const int64_t va = pack_items<kBM, TF32, A::kMN>(tiles_a, nchunks);
  const int64_t vb = pack_items<B_ROWS, TF32, B::kMN>(tiles_b, nchunks);
  const int cap = num_sms(device) * 16;
  const uint8_t* pa = ws;
  const uint8_t* pb = ws + abytes;
  if constexpr (kPrepackedA) {
    (void)va;
    const int blocks_b = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((vb + 255) / 256, cap)));
    count_launch();
    pack_kernel<B_ROWS, B, TF32><<<blocks_b, 256, 0, st>>>(b, ws, tiles_b, nchunks, sh.N, nullptr, sh.N);
    pa = a.image;
    pb = ws;
  } else {
    const int blocks_a = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((va + 255) / 256, cap)));
    const int blocks_b = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((vb + 255) / 256, cap / 2)));
    count_launch();
    pack2_kernel<kBM, A, B_ROWS, B, TF32><<<blocks_a + blocks_b, 256, 0, st>>>(
        a, b, ws, ws + abytes, tiles_a, tiles_b, nchunks, sh.M, sh.m_dev, sh.N, blocks_a);
  }
  const int total = tiles_a * tiles_b * std::max(1, sh.ksplit);
  const int grid = std::min(total, num_sms(device));
  int* status = device_status_ptr(device);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPackedThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  cudaLaunchKernelEx(&cfg, kern, pa, pb, e, sh, status);
  if (g_ws_alloc) g_ws_free(ws);  // stream-ordered: reused only by work queued after these kernels
  return true;
}

// Precision of the GEMMs whose shape does not say (GemmShape::tf32 = 0), for
// the whole process (autograd runs backward kernels from its own threads): set
// by set_gemm_precision (the TGN / JODIE engines and the DTDG trainer select
// runtime.precision before they issue a step).
static std::atomic<int> g_tf32{0};

// Host-detected failure reported through the device status word (read by the
// host after the step): the low byte of a zero word set to `code` (< 256).
static void record_host_error(int code) {
  int device = 0;
  cudaGetDevice(&device);
  int* st = device_status_ptr(device);
  if (st != nullptr) cudaMemsetAsync(st, code, 1, nullptr);
}
void set_gemm_precision(bool tf32) { g_tf32.store(tf32 ? 1 : 0); }
bool gemm_precision_tf32() { return g_tf32.load() != 0; }

template <int BN, int NSUB, class A, class B, class E>
static void launch_any(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st) {
  if (sh.tf32 || g_tf32.load(std::memory_order_relaxed)) {
    GemmShape s2 = sh;
    s2.tf32 = 1;
    // tf32 operands exist in the packed form only (the fused-producer kernel stages bf16 tiles)
    if (!launch_packed<BN, NSUB, true>(a, b, e, s2, st)) {
      fprintf(stderr, "starry_unigraph: tf32 GEMM needs an operand workspace (allocation failed)\n");
      record_host_error(kTooLarge);
    }
    return;
  }
  if (!packed_disabled() && launch_packed<BN, NSUB, false>(a, b, e, sh, st)) return;
  launch_cfg<BN, NSUB>(a, b, e, sh, st);
}

template <class A, class B, class E>
static void dispatch(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st) {
  if (sh.N <= 128) launch_any<128, 1>(a, b, e, sh, st);
  else if (sh.N <= 256) launch_any<256, 1>(a, b, e, sh, st);
  else launch_any<256, 2>(a, b, e, sh, st);
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
// Pre-packed A (no fused-producer fallback exists for it): false when the packed
// path is disabled or its workspace cannot be allocated, nothing launched then.
template <class A, class B, class E>
static bool dispatch_prepacked(const A& a, const B& b, const E& e, const GemmShape& sh, cudaStream_t st) {
  if (packed_disabled()) return false;  // bf16 images only (written by the caller's kernels)
  if (sh.N <= 128) return launch_packed<128, 1, false>(a, b, e, sh, st);
  if (sh.N <= 256) return launch_packed<256, 1, false>(a, b, e, sh, st);
  return launch_packed<256, 2, false>(a, b, e, sh, st);
}
bool gemm_prepacked(const Prepacked<false>& a, const MNView<WeightSource>& b, const EpiLinear& e, const GemmShape& sh,
                    cudaStream_t st) {
  return dispatch_prepacked(a, b, e, sh, st);
}
bool gemm_prepacked(const Prepacked<true>& a, const MNView<SegSource>& b, const EpiWeightGrad& e, const GemmShape& sh,
                    cudaStream_t st) {
  return dispatch_prepacked(a, b, e, sh, st);
}
bool packed_gemm_enabled() { return !packed_disabled(); }

void gemm(const SegSource& a, const WeightSource& b, const EpiGRU& e, const GemmShape& sh, cudaStream_t st) {
  launch_any<128, 1>(a, b, e, sh, st);  // one tile = four gates x 32 hidden units (gate-grouped rows)
}
void gemm(const SegSource& a, const WeightSource& b, const EpiOutLN& e, const GemmShape& sh, cudaStream_t st) {
  if (sh.N <= 128) launch_any<128, 1>(a, b, e, sh, st);
  else launch_any<256, 1>(a, b, e, sh, st);
}

void gemm(const SegSource& a, const WeightSource& b, const EpiRGruZR& e, const GemmShape& sh, cudaStream_t st) {
  launch_any<128, 1>(a, b, e, sh, st);  // one tile = [z | r] x 16 units, four times
}
void gemm(const SegSource& a, const WeightSource& b, const EpiRGruOut& e, const GemmShape& sh, cudaStream_t st) {
  if (sh.N <= 128) launch_any<128, 1>(a, b, e, sh, st);
  else launch_any<256, 1>(a, b, e, sh, st);
}
void gemm(const SegSource& a, const WeightSource& b, const EpiLSTM& e, const GemmShape& sh, cudaStream_t st) {
  launch_any<128, 1>(a, b, e, sh, st);  // one tile = four gates x 32 hidden units (gate-grouped rows)
}

}  // namespace su
