// Allocation-free entry point for the fused RMSNorm / adaLN backward (C interface declared in noalloc.h).
//
// This entry point has no counterpart in the reference; it exists for callers of this library that cannot
// allocate device memory at the moment they run the op: for example a plugin executed inside a host framework
// that owns every device allocation and forbids cudaMalloc during its enqueue call, or latency-critical code that
// cannot afford the implicit device synchronisation cudaMalloc / cudaFree may cause.  The regular entry point
// (`adanorm_bwd` in ops.cpp) asks torch's allocator for a per-call partial-sum buffer; this one uses a fixed
// scratch array that lives in the library image instead.
//
// Scratch: `g_noalloc_scratch`, a file-scope __device__ array of kNoAllocScratchFloats floats (16 MiB).  Every
// GPU on which the library is loaded holds it until the process exits.  The caller still passes all inputs and
// outputs.  Limits and rules:
//   * the partial sums need B * ceil(T / rows) * 4 * D floats; the entry point picks the smallest row chunk
//     (a multiple of 32) that fits and returns TGO_NOALLOC_TOO_LARGE when even one chunk per sample
//     (B * 4 * D floats) does not fit, or when B exceeds 65535 (the kernels put one grid row per sample);
//   * every call shares the one array and the row pass overwrites every element it later reads, so nothing needs
//     clearing between calls; two calls that overlap on the GPU (different streams without ordering, or two
//     host threads) race on the array and give wrong results;
//   * the first call on each device looks up the array's device address with cudaGetSymbolAddress (with that
//     device current) and caches it; make that first call before any stream capture begins;
//   * pointers and strides are checked on the host before anything is launched: the kernels move bf16 rows and
//     the scale / gate vectors in 16-byte loads and stores, so bf16 pointers must be 16-byte aligned and the batch
//     strides multiples of 8 elements; fp32 pointers must be 4-byte aligned;
//   * no cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "kernels.h"
#include "noalloc.h"

namespace {

constexpr long long kNoAllocScratchFloats = 4ll * 1024 * 1024;  // 16 MiB of fp32
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

// Device address of the scratch array on the current device (looked up once per device).  In host code the name
// g_noalloc_scratch is only a host-side stand-in, so it is never passed to a kernel directly.
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

// Capacity of the scratch array in floats.
long long tgo_noalloc_scratch_floats() { return kNoAllocScratchFloats; }

const char* tgo_noalloc_error_string(int code) {
  switch (code) {
    case TGO_NOALLOC_OK: return "ok";
    case TGO_NOALLOC_BAD_ARGS:
      return "invalid arguments (null pointer, bf16 pointer not 16-byte aligned, fp32 pointer not 4-byte aligned, "
             "scale / gate batch stride negative or not a multiple of 8, D % 8 != 0, D > 4096, or M % T != 0)";
    case TGO_NOALLOC_TOO_LARGE:
      return "problem too large for the fixed scratch array (needs B * 4 * D floats at least; capacity "
             "4194304 floats) or more than 65535 samples (B = M / T)";
    case TGO_NOALLOC_CUDA_ERROR: return "CUDA error (see cudaGetLastError)";
    default: return "unknown";
  }
}

// Smallest row chunk (a multiple of 32) whose partial sums fit the scratch array, or -1 if none does.
static int noalloc_rows(long long M, long long D, long long T) {
  if (M <= 0 || D <= 0 || T <= 0 || M % T != 0) return -1;
  const long long B = M / T;
  if (B > 65535 || B * 4ll * D > kNoAllocScratchFloats) return -1;
  long long rows = 32;
  while (B * ((T + rows - 1) / rows) * 4ll * D > kNoAllocScratchFloats) rows += 32;
  return static_cast<int>(rows);
}

int tgo_noalloc_adanorm_rows(int M, int D, int T) { return noalloc_rows(M, D, T); }

static bool misaligned(const void* p, unsigned bytes) {
  return p != nullptr && (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) != 0;
}

// Backward of  x_new = x + gate * y ;  h = rmsnorm(x_new) * w * (1 + scale) + shift   over M = B * T rows of D.
// Inputs (device pointers, bf16 unless noted): dh [M, D]; dxe [M, D] or null (extra gradient into x_new);
// xn [M, D] (x_new of the forward); rstd [M] fp32; w [D] fp32; scale [B, D] or null (batch stride mod_bs);
// y [M, D] or null; gate [B, D] or null (batch stride gate_bs).
// Outputs: dx [M, D]; dy [M, D] (only with y and gate); dshift, dscale [B, D] fp32 (only with scale);
// dgate [B, D] fp32 (only with y and gate); dw [D] fp32 is accumulated (+=), so clear it first for a plain
// gradient.
// Same results as the allocating entry point, on the given stream.
int tgo_adanorm_bwd_noalloc(const void* dh, const void* dxe, const void* xn, const float* rstd, const float* w,
                            const void* scale, long long mod_bs, const void* y, const void* gate, long long gate_bs,
                            void* dx, void* dy, float* dshift, float* dscale, float* dgate, float* dw, int M, int D,
                            int T, cudaStream_t stream) {
  if (dh == nullptr || xn == nullptr || rstd == nullptr || w == nullptr || dx == nullptr || dw == nullptr ||
      M <= 0 || D <= 0 || T <= 0 || D % 8 != 0 || D > 4096 || M % T != 0)
    return TGO_NOALLOC_BAD_ARGS;
  if (scale != nullptr && (dshift == nullptr || dscale == nullptr)) return TGO_NOALLOC_BAD_ARGS;
  if (gate != nullptr && y != nullptr && (dy == nullptr || dgate == nullptr)) return TGO_NOALLOC_BAD_ARGS;
  // 16-byte vector loads / stores of bf16 rows and of the scale / gate vectors; scalar fp32 accesses.
  for (const void* p : {dh, dxe, xn, scale, y, gate, static_cast<const void*>(dx), static_cast<const void*>(dy)})
    if (misaligned(p, 16)) return TGO_NOALLOC_BAD_ARGS;
  for (const void* p : {static_cast<const void*>(rstd), static_cast<const void*>(w), static_cast<const void*>(dshift),
                        static_cast<const void*>(dscale), static_cast<const void*>(dgate),
                        static_cast<const void*>(dw)})
    if (misaligned(p, 4)) return TGO_NOALLOC_BAD_ARGS;
  if (scale != nullptr && (mod_bs < 0 || mod_bs % 8 != 0)) return TGO_NOALLOC_BAD_ARGS;
  if (gate != nullptr && (gate_bs < 0 || gate_bs % 8 != 0)) return TGO_NOALLOC_BAD_ARGS;
  const int rows = noalloc_rows(M, D, T);
  if (rows < 0) return TGO_NOALLOC_TOO_LARGE;
  float* scratch = nullptr;
  if (scratch_for_current_device(&scratch) != cudaSuccess) return TGO_NOALLOC_CUDA_ERROR;

  tgo::AdaNormBwdParams p{};
  p.dh = static_cast<const __nv_bfloat16*>(dh);
  p.dxe = static_cast<const __nv_bfloat16*>(dxe);
  p.xn = static_cast<const __nv_bfloat16*>(xn);
  p.rstd = rstd;
  p.w = w;
  p.scale = static_cast<const __nv_bfloat16*>(scale);
  p.mod_bs = mod_bs;
  p.y = static_cast<const __nv_bfloat16*>(y);
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.gate_bs = gate_bs;
  p.dx = static_cast<__nv_bfloat16*>(dx);
  p.dy = (gate != nullptr && y != nullptr) ? static_cast<__nv_bfloat16*>(dy) : nullptr;
  p.partial = scratch;
  p.M = M;
  p.D = D;
  p.T = T;
  p.rows_per_cta = rows;
  p.chunks = (T + rows - 1) / rows;
  const cudaError_t e = tgo::adanorm_bwd_launch(p, scale != nullptr ? dshift : nullptr,
                                                scale != nullptr ? dscale : nullptr, p.dy != nullptr ? dgate : nullptr,
                                                dw, stream);
  return e == cudaSuccess ? TGO_NOALLOC_OK : TGO_NOALLOC_CUDA_ERROR;
}

}  // extern "C"
