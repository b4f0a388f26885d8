// Public C interface of the allocation-free fused RMSNorm / adaLN backward (implemented in noalloc.cu).
//
// This interface has no counterpart in the reference.  It is for callers of this library that cannot allocate
// device memory while they run an op: a plugin executed inside a host framework that owns every device allocation
// and forbids cudaMalloc during its enqueue call, or latency-critical code that cannot take the implicit device
// synchronisation cudaMalloc / cudaFree may cause.  The partial-sum scratch of the backward lives in a fixed
// file-scope __device__ array of the library (16 MiB per GPU that loads the library, held until the process exits)
// instead of a per-call allocation; the caller passes every input and output.
//
// Rules (the implementation file repeats them beside the code):
//   * capacity tgo_noalloc_scratch_floats() floats; a problem needs B * ceil(T / rows) * 4 * D floats for the row
//     chunk `rows` (a multiple of 32) that tgo_noalloc_adanorm_rows() reports; B = M / T must not exceed 65535
//     (one grid row per sample);
//   * every call shares the one array, so calls that overlap on the GPU (unordered streams, concurrent host
//     threads) race and give wrong results; the array keeps the last call's contents, and every element a call
//     reads was written earlier in the same call, so nothing needs clearing;
//   * the first call on a device looks up the array's device address (cudaGetSymbolAddress, with that device
//     current) and caches it: make that first call before any stream capture begins;
//   * no cudaMalloc, cudaFree or allocating library routine is called;
//   * bf16 pointers must be 16-byte aligned and fp32 pointers 4-byte aligned; the batch strides of scale and gate
//     (in elements) must be non-negative multiples of 8.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

enum TgoNoAllocStatus {
  TGO_NOALLOC_OK = 0,
  TGO_NOALLOC_BAD_ARGS = 1,   // null pointer, misaligned pointer or stride, D % 8 != 0, D > 4096, M % T != 0
  TGO_NOALLOC_TOO_LARGE = 2,  // B * 4 * D floats exceed the scratch array, or B > 65535
  TGO_NOALLOC_CUDA_ERROR = 3, // a CUDA call failed (symbol lookup or kernel launch)
};

// Capacity of the scratch array in floats.
long long tgo_noalloc_scratch_floats(void);

// Human-readable text for a status code.
const char* tgo_noalloc_error_string(int code);

// Row chunk (rows of one sample per CTA) the entry point uses for M rows of D channels in samples of T rows, or
// -1 when the problem is rejected as too large.
int tgo_noalloc_adanorm_rows(int M, int D, int T);

// Backward of  x_new = x + gate * y ;  h = rmsnorm(x_new) * w * (1 + scale) + shift   over M = B * T rows of D.
// Inputs (device pointers, bf16 unless noted): dh [M, D]; dxe [M, D] or null (extra gradient into x_new);
// xn [M, D] (x_new of the forward); rstd [M] fp32; w [D] fp32; scale [B, D] or null (batch stride mod_bs);
// y [M, D] or null; gate [B, D] or null (batch stride gate_bs).
// Outputs: dx [M, D]; dy [M, D] (only with y and gate); dshift, dscale [B, D] fp32 (only with scale);
// dgate [B, D] fp32 (only with y and gate); dw [D] fp32 is accumulated (+=), so clear it first for a plain
// gradient.  Runs on `stream` and returns a TgoNoAllocStatus.
int tgo_adanorm_bwd_noalloc(const void* dh, const void* dxe, const void* xn, const float* rstd, const float* w,
                            const void* scale, long long mod_bs, const void* y, const void* gate, long long gate_bs,
                            void* dx, void* dy, float* dshift, float* dscale, float* dgate, float* dw, int M, int D,
                            int T, cudaStream_t stream);

#ifdef __cplusplus
}  // extern "C"
#endif
