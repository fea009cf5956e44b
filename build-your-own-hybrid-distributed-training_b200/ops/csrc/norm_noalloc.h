// Declaration of the allocation-free norm-backward entry point (defined in norm_noalloc.cu).
//
// This entry point has no counterpart in the reference implementation.  It is for callers that
// cannot allocate device memory, for example a runtime that pre-plans every buffer in a fixed pool
// or a host process that forbids cudaMalloc once start-up is over.  Its scratch (the per-block
// partial sums of the weight and bias gradients) lives in one file-scope device array of
// 2 x 128 x 8192 floats (8 MiB) that every GPU loading the library holds until the process exits.
//
// Contract:
//   * dy: [rows, d] gradient of the normalised output (bf16 when dy_is_bf16, else fp32; may be null);
//   * dr: [rows, d] fp32 gradient arriving on the residual stream (may be null);
//   * r: [rows, d] fp32 residual-stream values that the forward normalised;
//   * w: [d] norm weight (bf16 when w_is_bf16, else fp32);
//   * mean, rstd: [rows] fp32 statistics saved by the forward.  `mean` is read for LayerNorm
//     (rms = 0) only; for RMSNorm (rms = 1) it is ignored and may be null;
//   * outputs: dres [rows, d] fp32; ddelta [rows, d] in bf16 or fp32 (may be null); dw [d] fp32;
//     db [d] fp32 (LayerNorm only; ignored and may be null for RMSNorm);
//   * work is queued on `stream` on the current device;
//   * d may be 1..8192 (any value, not only multiples of 8); larger d returns 2;
//   * the first call on each device looks up the scratch array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make that first call before
//     any stream capture begins;
//   * every call shares the scratch array and leaves its contents behind; calls that overlap on
//     the GPU (other streams, other host threads) race on it, so the caller serialises them;
//   * no cudaMalloc, cudaFree or allocating library routine is called.
//
// Return codes: 0 success; 1 bad sizes or a missing required pointer; 2 hidden size above 8192;
// 1000 + cudaError_t for a failure in the one-time set-up or in a launch.
#pragma once

#include <cuda_runtime.h>

#define HT_NORM_NOALLOC_MAX_COLS 8192

#ifdef __cplusplus
extern "C" {
#endif

int ht_norm_backward_noalloc(const void* dy, int dy_is_bf16, const float* dr, const float* r, const void* w, int w_is_bf16,
                             const float* mean, const float* rstd, float* dres, void* ddelta, int ddelta_is_bf16, float* dw,
                             float* db, int rows, int d, int rms, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
