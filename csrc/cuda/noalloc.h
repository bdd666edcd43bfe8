// Allocation-free C entry point of the fused LSTM-cell backward.
//
// This entry point has no counterpart in the reference framework; it exists
// for callers that must not allocate device memory while they run: a host
// runtime with its own fixed memory budget, a custom allocator that may not be
// re-entered, or code linked without PyTorch. It runs the same kernels as the
// `lstm_bwd` op of the Python extension (elementwise gate gradients, then the
// input and weight gradients on the tcgen05 GEMM), but every buffer is the
// caller's except one temporary, which lives in a fixed-size static device
// array of this library (SU_NOALLOC_SCRATCH_BYTES per device).
//
// Nothing here calls cudaMalloc, cudaFree or any library routine that
// allocates (PyTorch included).
//
// Rules for callers:
//  * The first call on each device looks the scratch array up
//    (cudaGetSymbolAddress) and sets the GEMM kernels' shared-memory attribute.
//    Make that first call outside any stream capture.
//  * There is ONE scratch array per device. Two calls whose work overlaps on the
//    same device (different streams, or different host threads) race on it and
//    give wrong results. Issue the calls of one device on one stream, or order
//    them with events.
//  * Must start at zero (or hold the gradient to add to): gw_*, gb_* (the weight
//    and bias gradients are accumulated, +=). Fully overwritten: dxh, dc_prev.
//    The scratch array needs no initialisation.
//  * Sizes above the scratch capacity are rejected with SU_NOALLOC_ERR_SCRATCH
//    before anything is launched; su_noalloc_scratch_required() gives the need.
#pragma once

#include <cstddef>

#define SU_NOALLOC_SCRATCH_BYTES (32u << 20)

#define SU_NOALLOC_OK 0
#define SU_NOALLOC_ERR_ARGUMENT (-1)
#define SU_NOALLOC_ERR_SCRATCH (-2)
#define SU_NOALLOC_ERR_CUDA (-3)

#ifdef __cplusplus
extern "C" {
#endif

// Backward of (h', c') = LSTMCell(x, (h, c)) for `rows` rows.
//   x        [rows, in_dim]            forward input
//   h_prev   [rows, hidden] or NULL    previous hidden state (NULL: zeros)
//   c_prev   [rows, hidden] or NULL    previous cell state (NULL: zeros)
//   c_new    [rows, hidden]            forward cell output
//   gates    [rows, 64*ceil(hidden/16)] post-activation gates (i, f, g, o) as saved by the
//                                      forward: per row, per group of 16 units, i f g o x 16
//   dh, dc   [rows, hidden] or NULL    upstream gradients of h' and c'
//   w_*      [hidden, in_dim + hidden] gate weights, row-major ([W_x | W_h])
//   gw_*     [hidden, in_dim + hidden] weight gradients (accumulated)
//   gb_*     [hidden]                  bias gradients (accumulated)
//   dxh      [rows, in_dim + hidden]   out: d x in columns [0, in_dim), d h_prev in [in_dim, in_dim + hidden)
//   dc_prev  [rows, hidden]            out: d c_prev
// All pointers are fp32 device pointers, contiguous and 16-byte aligned.
// `stream` is a cudaStream_t (NULL: the legacy default stream).
// Returns SU_NOALLOC_OK or a negative SU_NOALLOC_ERR_* code.
int su_lstm_cell_backward_noalloc(const float* x, const float* h_prev, const float* c_prev, const float* c_new,
                                  const float* gates, const float* dh, const float* dc, const float* w_i,
                                  const float* w_f, const float* w_g, const float* w_o, float* gw_i, float* gb_i,
                                  float* gw_f, float* gb_f, float* gw_g, float* gb_g, float* gw_o, float* gb_o,
                                  float* dxh, float* dc_prev, int rows, int in_dim, int hidden, void* stream);

// Scratch bytes that a call of this shape needs (compare with SU_NOALLOC_SCRATCH_BYTES).
size_t su_noalloc_scratch_required(int rows, int in_dim, int hidden);

// Capacity of the static scratch array, in bytes.
size_t su_noalloc_scratch_capacity(void);

// Copies the status words of the calls made through this entry point (4 ints;
// word 0 is 0 while every bounded wait of the GEMM kernels finished, else the
// first failure's code: 1-4 a wait that gave up, 7 a size above a kernel bound)
// to `out4`. It first waits for every stream of the current device
// (cudaDeviceSynchronize), so calls issued on non-blocking streams are included.
// The status is sticky: it keeps the first failure of any call since the library
// was loaded or since the last su_noalloc_status_reset(). Returns SU_NOALLOC_OK
// or SU_NOALLOC_ERR_CUDA.
int su_noalloc_status(int* out4);

// Clears the status words of the current device (waits for the device first).
int su_noalloc_status_reset(void);

// Human-readable text of a return code.
const char* su_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
