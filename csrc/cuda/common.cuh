// Shared device helpers for the sm_100a kernels of starry_unigraph.
//
// * PTX wrappers for mbarriers, tcgen05 (TMEM allocation, UMMA issue, commit,
//   TMEM loads) and proxy fences.
// * Bounded waits: every spin on an mbarrier or a peer flag gives up after a
//   clock64() budget, records an error code in a device status word and lets
//   the kernel unwind (free TMEM, return) instead of hanging the GPU.
// * A counter-based Philox-4x32-10 generator (Salmon et al., SC'11) used for
//   negative sampling, uniform neighbour sampling and dropout masks, so that
//   forward and backward regenerate identical masks without storing them.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace su {

// ---------------------------------------------------------------------------
// Error status (host reads it after the step; never trap on device)
// ---------------------------------------------------------------------------
enum StatusCode : int {
  kOk = 0,
  kTimeoutFull = 1,     // MMA warp waited too long for operand stage
  kTimeoutEmpty = 2,    // producer waited too long for a free stage
  kTimeoutAccum = 3,    // epilogue waited too long for the accumulator
  kTimeoutTmemFree = 4, // MMA waited too long for the epilogue to drain TMEM
  kBadIndex = 5,        // an index was out of range (access skipped)
  kPeerTimeout = 6,     // a peer flag never arrived
  kTooLarge = 7,        // a size exceeded a compiled-in bound
};

// ~2 s at the B200 boost clock; far beyond any legitimate intra-kernel wait.
constexpr long long kWaitBudgetCycles = 4000000000LL;

// Instruction descriptor for kind::f16 with BF16 A/B, FP32 accumulate, both
// operands K-major, shape M x N.
#ifdef __CUDACC__
__host__ __device__
#endif
constexpr uint32_t umma_idesc_bf16_f32(int M, int N) {
  return (1u << 4)            // D format: F32
         | (1u << 7)          // A format: BF16
         | (1u << 10)         // B format: BF16
         | (0u << 15)         // A K-major
         | (0u << 16)         // B K-major
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor for kind::tf32 (fp32 operands read as TF32, FP32
// accumulate), both operands K-major, shape M x N.
#ifdef __CUDACC__
__host__ __device__
#endif
constexpr uint32_t umma_idesc_tf32_f32(int M, int N) {
  return (1u << 4)            // D format: F32
         | (2u << 7)          // A format: TF32
         | (2u << 10)         // B format: TF32
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

#ifdef __CUDACC__

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Arrive on `bar` and add `bytes` to the transaction count it waits for.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Bulk (untiled, no multicast) global -> shared copy completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Tiled TMA store of one 2D box from shared memory to global memory (bulk
// async-group completion, no multicast). `tmap` is the generic address of a
// CUtensorMap in parameter / constant / global memory; (x, y) the box origin
// in elements (x: innermost; x * element size a multiple of 16 bytes, both >= 0).
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's bulk groups are still reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N of this thread's bulk groups are still in flight (writes done).
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Returns false when the budget ran out (caller records a status and unwinds).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles) return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Proxy / tcgen05 fences
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMEM allocation (one full warp executes these)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors (layouts as defined by the tcgen05 shared-memory matrix
// descriptor: start address, leading/stride byte offsets in 16-byte units,
// version 1, layout type in bits 61..63).
// ---------------------------------------------------------------------------
// K-major, no swizzle ("interleaved" core matrices of 8 rows x 16 bytes):
//   LBO = byte distance between K-adjacent core matrices
//   SBO = byte distance between 8-row groups
__device__ __forceinline__ uint64_t umma_desc_kmajor_noswizzle(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  // base offset 0, lbo mode 0, layout type 0 (SWIZZLE_NONE)
  return d;
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05 ops of this thread finish.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Each thread of the warp reads 16 consecutive fp32 columns of its own TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Split form: issue several loads, overlap them with global loads, then one
// tmem_wait_ld() before the registers are read.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8_issue(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <int N>
__device__ __forceinline__ void tmem_wait_ld4n(uint32_t (&a)[N], uint32_t (&b)[N], uint32_t (&c)[N],
                                               uint32_t (&d)[N]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(a[i]), "+r"(b[i]), "+r"(c[i]), "+r"(d[i]));
}
// The asm outputs of the issued loads are passed through as read-write operands
// so the compiler cannot move a read of them above the wait.
__device__ __forceinline__ void tmem_wait_ld4(uint32_t (&a)[16], uint32_t (&b)[16], uint32_t (&c)[16],
                                              uint32_t (&d)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) asm volatile("" : "+r"(a[i]), "+r"(b[i]), "+r"(c[i]), "+r"(d[i]));
}

// One wait for every load issued into `r` (any length).
template <int N>
__device__ __forceinline__ void tmem_wait_ld_all(uint32_t (&r)[N]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// read-only 16-byte global load through the non-coherent path (data that no
// thread of the running kernel writes)
__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// ---------------------------------------------------------------------------
// Philox-4x32-10 counter-based RNG
// ---------------------------------------------------------------------------
struct Philox {
  __device__ static __forceinline__ uint4 round(uint4 c, uint2 k) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
    uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    return make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
  }
  // Returns four 32-bit random words for (seed, counter, subsequence).
  __device__ static __forceinline__ uint4 gen(uint64_t seed, uint64_t counter, uint32_t sub) {
    uint4 c = make_uint4((uint32_t)counter, (uint32_t)(counter >> 32), sub, 0x9E3779B9u);
    uint2 k = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
#pragma unroll
    for (int i = 0; i < 10; ++i) {
      c = round(c, k);
      k.x += 0x9E3779B9u;
      k.y += 0xBB67AE85u;
    }
    return c;
  }
  __device__ static __forceinline__ float uniform(uint32_t x) {  // [0, 1)
    return (x >> 8) * (1.0f / 16777216.0f);
  }
};

// Dropout keep decision for element `idx` of stream `stream` (same in fwd/bwd).
__device__ __forceinline__ bool dropout_keep(uint64_t seed, uint64_t idx, uint32_t stream, float p) {
  if (p <= 0.f) return true;
  uint4 r = Philox::gen(seed, idx >> 2, stream);
  uint32_t w = (idx & 3) == 0 ? r.x : (idx & 3) == 1 ? r.y : (idx & 3) == 2 ? r.z : r.w;
  return Philox::uniform(w) >= p;
}

// Keep decisions of elements idx4 .. idx4+3 (idx4 a multiple of 4): one Philox
// call, the same decisions dropout_keep gives element by element.
__device__ __forceinline__ void dropout_keep4(uint64_t seed, uint64_t idx4, uint32_t stream, float p, bool (&k)[4]) {
  if (p <= 0.f) {
    k[0] = k[1] = k[2] = k[3] = true;
    return;
  }
  const uint4 r = Philox::gen(seed, idx4 >> 2, stream);
  k[0] = Philox::uniform(r.x) >= p;
  k[1] = Philox::uniform(r.y) >= p;
  k[2] = Philox::uniform(r.z) >= p;
  k[3] = Philox::uniform(r.w) >= p;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
// Gate activations of the fused RNN-cell epilogues: the hardware exp2 and
// reciprocal units (__expf, __frcp_rn) and tanh.approx.f32 (max relative error
// about 2^-11, finer than the bf16 rounding of the GEMM operands feeding them).
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// sigmoid(x) = (1 + tanh(x / 2)) / 2: one tanh.approx (a single special-function
// instruction) and two FMAs, with tanh_fast's absolute error halved.
__device__ __forceinline__ float sigmoid_fast(float x) { return fmaf(0.5f, tanh_fast(0.5f * x), 0.5f); }

// Round 4 floats to TF32 (round to nearest, ties away from zero: cvt.rna) and
// return them as one 16-byte vector of 32-bit containers.
__device__ __forceinline__ uint4 pack_tf32x4(const float* f) {
  uint4 u;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u.x) : "f"(f[0]));
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u.y) : "f"(f[1]));
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u.z) : "f"(f[2]));
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u.w) : "f"(f[3]));
  return u;
}

// Pack 8 floats to 8 bf16 (one 16-byte vector).
__device__ __forceinline__ uint4 pack_bf16x8(const float* f) {
  uint4 u;
  __nv_bfloat162 t;
  t = __floats2bfloat162_rn(f[0], f[1]);
  u.x = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2bfloat162_rn(f[2], f[3]);
  u.y = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2bfloat162_rn(f[4], f[5]);
  u.z = *reinterpret_cast<uint32_t*>(&t);
  t = __floats2bfloat162_rn(f[6], f[7]);
  u.w = *reinterpret_cast<uint32_t*>(&t);
  return u;
}

#endif  // __CUDACC__

}  // namespace su
