// Elementwise kernels of the sampler and of the flow-matching step.
//
// euler_cfg: one Euler step with classifier-free guidance (reference aurora/fid.py:35-37,
//   aurora/hf_pipeline.py:753-759), reading the denoiser's token-major output directly:
//     v   = v_u + w (v_c - v_u)           v_u = out[b], v_c = out[B + b]   (out: [2B, T, C] token-major)
//     z  += dt * v                        z: [B, C, T] fp32 (latent layout)
//   so the [2B, T, C] -> [2B, C, H, W] transpose and the separate guidance / update passes never materialise.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tgo {

// grid: (T / 32, C / 32, B); block 32 x 8; a 32 x 32 (token, channel) tile transposed through shared memory
__global__ void euler_cfg_kernel(const __nv_bfloat16* __restrict__ out, float* __restrict__ z, int B, int T, int C,
                                 float dt, float w) {
  __shared__ float tile[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32, b = blockIdx.z;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int i = ty; i < 32; i += 8) {
    const int t = t0 + i, c = c0 + tx;
    float v = 0.f;
    if (t < T && c < C) {
      const float vu = __bfloat162float(out[((long long)b * T + t) * C + c]);
      const float vc = __bfloat162float(out[((long long)(B + b) * T + t) * C + c]);
      v = vu + w * (vc - vu);
    }
    tile[i][tx] = v;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int c = c0 + i, t = t0 + tx;
    if (t < T && c < C) z[((long long)b * C + c) * T + t] += dt * tile[tx][i];
  }
}

cudaError_t euler_cfg_launch(const __nv_bfloat16* out, float* z, int B, int T, int C, float dt, float w,
                             cudaStream_t s) {
  dim3 grid((T + 31) / 32, (C + 31) / 32, B), block(32, 8);
  euler_cfg_kernel<<<grid, block, 0, s>>>(out, z, B, T, C, dt, w);
  return cudaGetLastError();
}

// fm_inputs: the flow-matching input and target of a training micro-batch (reference aurora/model.py FlowModel,
// train.py:662-668), in the layouts their consumers read:
//     z_t    = (1 - t) x0 + t eps   -> bf16 token-major [B, T, C] (the patch-in GEMM's A operand)
//     target = eps - x0             -> fp32 token-major [B, T, C] (compared with the token-major velocity)
// from x0 / eps fp32 [B, C, T] (latent layout), one pass through a shared 32 x 32 transpose tile.
__global__ void fm_inputs_kernel(const float* __restrict__ x0, const float* __restrict__ eps,
                                 const float* __restrict__ t, __nv_bfloat16* __restrict__ z_tok,
                                 float* __restrict__ target, int T, int C) {
  __shared__ float tz[32][33], tg[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32, b = blockIdx.z;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const float tb = t[b];
  for (int i = ty; i < 32; i += 8) {  // read along tokens (contiguous in the latent layout)
    const int c = c0 + i, tt = t0 + tx;
    float z = 0.f, g = 0.f;
    if (tt < T && c < C) {
      const long long off = ((long long)b * C + c) * T + tt;
      const float x = x0[off], e = eps[off];
      z = (1.f - tb) * x + tb * e;
      g = e - x;
    }
    tz[i][tx] = z;
    tg[i][tx] = g;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {  // write along channels (contiguous in the token-major layout)
    const int tt = t0 + i, c = c0 + tx;
    if (tt < T && c < C) {
      const long long off = ((long long)b * T + tt) * C + c;
      z_tok[off] = __float2bfloat16(tz[tx][i]);
      target[off] = tg[tx][i];
    }
  }
}

cudaError_t fm_inputs_launch(const float* x0, const float* eps, const float* t, __nv_bfloat16* z_tok, float* target,
                             int B, int T, int C, cudaStream_t s) {
  dim3 grid((T + 31) / 32, (C + 31) / 32, B), block(32, 8);
  fm_inputs_kernel<<<grid, block, 0, s>>>(x0, eps, t, z_tok, target, T, C);
  return cudaGetLastError();
}

// Per-row symmetric int8 quantisation of activations (the W8A8 GEMM's A operand): scale = max |x| / 127 (at least
// 1e-12), q = round-to-nearest-even(x / scale) clamped to [-127, 127]. One warp per row; the row is read twice, the
// second time from L1 / L2. K must be a multiple of 8 (16-byte bf16 loads, 8-byte int8 stores).
__global__ void __launch_bounds__(256) quantize_rows_i8_kernel(const __nv_bfloat16* __restrict__ x, int8_t* __restrict__ q,
                                                               float* __restrict__ scale, int M, int K) {
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const __nv_bfloat16* src = x + row * K;
  float amax = 0.f;
  for (int c = lane * 8; c < K; c += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = fmaxf(amax, 1e-12f) / 127.f;
  const float inv = 1.f / s;
  if (lane == 0) scale[row] = s;
  int8_t* dst = q + row * K;
  for (int c = lane * 8; c < K; c += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      const int a = max(-127, min(127, __float2int_rn(f.x * inv)));
      const int b = max(-127, min(127, __float2int_rn(f.y * inv)));
      w[i >> 1] |= ((uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8)) << ((i & 1) * 16);
    }
    *reinterpret_cast<uint2*>(dst + c) = make_uint2(w[0], w[1]);
  }
}

cudaError_t quantize_rows_i8_launch(const __nv_bfloat16* x, int8_t* q, float* scale, int M, int K, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  if (K <= 0 || K % 8 != 0) return cudaErrorInvalidValue;
  quantize_rows_i8_kernel<<<(M + 7) / 8, 256, 0, s>>>(x, q, scale, M, K);
  return cudaGetLastError();
}

}  // namespace tgo
