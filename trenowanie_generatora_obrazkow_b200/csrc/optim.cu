// Optimizer tail after the backward pass, in two launches instead of the library's per-op multi-tensor kernels:
//
// grad_norm  every CTA sums the squares of its chunk of every gradient segment, adds them to one accumulator, and
//            the last CTA to finish (atomic counter) turns the total into the global norm and the clip coefficient
//            min(1, clip / (norm + 1e-6)) on the device, then resets the accumulator and the counter. Nothing is
//            read back to the host, and the gradients are not rescaled: the optimizers take the coefficient.
// adamw      decoupled-weight-decay Adam (torch.optim.AdamW semantics, amsgrad off) over a segment table of
//            (param, grad, exp_avg, exp_avg_sq, bf16 shadow, EMA) pointers: g = coef * grad;
//            m = b1 m + (1 - b1) g; v = b2 v + (1 - b2) g^2; p = p (1 - lr wd) - (lr / bc1) m / (sqrt(v) / sqrt(bc2)
//            + eps); then the bf16 shadow copy of p (read by the next forward's GEMMs) and the EMA
//            e += rate (p - e), both where the segment has them.
// Reference behaviour being replaced: clip_grad_norm_ + torch.optim.AdamW(fused=True) + torch._foreach_lerp_ of the
// EMA (reference train.py:338, 942, 966).
#include "common.cuh"
#include "kernels.h"

namespace tgo {

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
  if (w == 0)
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;  // valid in thread 0
}

__global__ void __launch_bounds__(256) grad_norm_kernel(GradNormParams p) {
  __shared__ float red[8];
  __shared__ bool last;
  const int c = blockIdx.x, C = gridDim.x;
  float sq = 0.f;
  for (int s = 0; s < p.nsegs; ++s) {
    const float* g = reinterpret_cast<const float*>(p.segs[2 * s]);
    const long long n = p.segs[2 * s + 1];
    const long long chunk = ((n + C - 1) / C + 3) / 4 * 4;
    const long long a = (long long)c * chunk, b = min(n, a + chunk);
    const bool vec = reinterpret_cast<uintptr_t>(g) % 16 == 0;
    long long i = a + threadIdx.x * 4;
    if (vec) {
      for (; i + 4 <= b; i += (long long)blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4*>(g + i);
        sq += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
    }
    long long j = vec ? i : a + threadIdx.x;
    const long long jstep = vec ? 1 : blockDim.x;
    for (; j < b; j += jstep) sq += g[j] * g[j];
  }
  sq = block_reduce_sum(sq, red);
  if (threadIdx.x == 0) {
    if (sq != 0.f) atomicAdd(p.acc, sq);
    __threadfence();
    last = atomicAdd(p.counter, 1u) == (unsigned)(C - 1);
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    float total = atomicExch(p.acc, 0.f);
    if (p.extra_sumsq != nullptr) total += *p.extra_sumsq;
    const float norm = sqrtf(total);
    *p.gnorm = norm;
    *p.coef = p.clip > 0.f ? fminf(1.f, p.clip / (norm + 1e-6f)) : 1.f;
    *p.counter = 0u;
  }
}

__device__ __forceinline__ void adamw_elem(float& w, float& m, float& v, float g, const float* h) {
  m = h[4] * m + (1.f - h[4]) * g;
  v = h[5] * v + (1.f - h[5]) * g * g;
  w = w * h[0] - h[1] * m / (sqrtf(v) * h[2] + h[3]);
}

__global__ void __launch_bounds__(256) adamw_kernel(AdamWParams p) {
  const int c = blockIdx.x, C = gridDim.x;
  const float coef = p.coef != nullptr ? *p.coef : 1.f;
  const float r = p.ema_rate;
  for (int s = 0; s < p.nsegs; ++s) {
    const long long* t = p.segs + 8 * s;
    float* w = reinterpret_cast<float*>(t[0]);
    const float* g = reinterpret_cast<const float*>(t[1]);
    float* m = reinterpret_cast<float*>(t[2]);
    float* v = reinterpret_cast<float*>(t[3]);
    __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(t[4]);
    float* ema = reinterpret_cast<float*>(t[5]);
    const long long n = t[6];
    const float* h = p.hyper + 6 * t[7];
    const long long chunk = ((n + C - 1) / C + 3) / 4 * 4;
    const long long a = (long long)c * chunk, b = min(n, a + chunk);
    const bool vec = ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(g) |
                       reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v) |
                       reinterpret_cast<uintptr_t>(ema)) % 16 == 0) &&
                     reinterpret_cast<uintptr_t>(sh) % 8 == 0;
    long long i = a + threadIdx.x * 4;
    if (vec) {
      for (; i + 4 <= b; i += (long long)blockDim.x * 4) {
        float4 W = *reinterpret_cast<float4*>(w + i);
        const float4 G = *reinterpret_cast<const float4*>(g + i);
        float4 M = *reinterpret_cast<float4*>(m + i);
        float4 V = *reinterpret_cast<float4*>(v + i);
        adamw_elem(W.x, M.x, V.x, G.x * coef, h);
        adamw_elem(W.y, M.y, V.y, G.y * coef, h);
        adamw_elem(W.z, M.z, V.z, G.z * coef, h);
        adamw_elem(W.w, M.w, V.w, G.w * coef, h);
        *reinterpret_cast<float4*>(w + i) = W;
        *reinterpret_cast<float4*>(m + i) = M;
        *reinterpret_cast<float4*>(v + i) = V;
        if (sh != nullptr) *reinterpret_cast<uint2*>(sh + i) = make_uint2(pack_bf16x2(W.x, W.y), pack_bf16x2(W.z, W.w));
        if (ema != nullptr) {
          float4 E = *reinterpret_cast<float4*>(ema + i);
          E.x += r * (W.x - E.x);
          E.y += r * (W.y - E.y);
          E.z += r * (W.z - E.z);
          E.w += r * (W.w - E.w);
          *reinterpret_cast<float4*>(ema + i) = E;
        }
      }
    }
    long long j = vec ? i : a + threadIdx.x;
    const long long jstep = vec ? 1 : blockDim.x;
    for (; j < b; j += jstep) {
      float W = w[j], M = m[j], V = v[j];
      adamw_elem(W, M, V, g[j] * coef, h);
      w[j] = W;
      m[j] = M;
      v[j] = V;
      if (sh != nullptr) sh[j] = __float2bfloat16_rn(W);
      if (ema != nullptr) ema[j] += r * (W - ema[j]);
    }
  }
}

cudaError_t grad_norm_launch(const GradNormParams& p, int blocks, cudaStream_t s) {
  grad_norm_kernel<<<blocks, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t adamw_launch(const AdamWParams& p, int blocks, cudaStream_t s) {
  if (p.nsegs == 0) return cudaSuccess;
  adamw_kernel<<<blocks, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace tgo
