// Fused normalisation kernels (memory-bound; one pass over the activations each way).
//
// adanorm: residual update + RMSNorm + adaLN modulation of a DiT block
//     x_new = x + gate * y            (gate per (batch, channel); optional; y optional)
//     h     = rmsnorm(x_new) * w * (1 + scale) + shift                (scale / shift optional)
//   reference aurora/model.py:27-34 (RMSNorm) and :204-210 (DenoiserBlock modulation and gated residuals).
//   The backward produces dx, dy and the per-(batch, channel) sums dshift / dscale / dgate and the per-channel dw
//   through per-CTA partial sums in a scratch buffer and a second reduction pass.
//
// qknorm_rope: per-head RMSNorm of q and k (optional) followed by interleaved-pair RoPE (reference
//   aurora/model.py:37-40, :98-99, :164), reading the fused qkv GEMM output in place.
//
// swiglu: g = silu(a) * b on the fused in_proj output [a | b] (reference aurora/model.py:102-110).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tgo {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void load8(const bf16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void store8(bf16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16(v)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum; `red` holds 2 x 32 floats, `slot` alternates between consecutive calls so one barrier suffices.
__device__ __forceinline__ float block_sum(float v, float* red, int slot) {
  v = warp_sum(v);
  const int nw = (blockDim.x + 31) >> 5;
  if (lane_id() == 0) red[slot * 32 + warp_id()] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[slot * 32 + i];
  return s;
}

// ------------------------------------------------------------------------------------------------------------------
// adanorm forward
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float2 block_sum2(float a, float b, float* red, int slot);
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]);

// Two rows per iteration: every load of both rows is issued first and their sums of squares share one block
// reduction (half the barriers, twice the loads in flight).
__global__ void __launch_bounds__(1024) adanorm_fwd_kernel(AdaNormFwdParams p) {
  __shared__ float red[128];
  const int c0 = threadIdx.x * 8;
  const bool active = c0 < p.D;
  float w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = active ? p.w[c0 + i] : 0.f;
  const int row0 = blockIdx.x * p.rows_per_cta;
  const int row1 = min(p.M, row0 + p.rows_per_cta);
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  int slot = 0;
  for (int row = row0; row < row1; row += 2, slot ^= 1) {
    const bool two = row + 1 < row1;
    uint4 ux[2], uy[2], ug[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const bool ok = active && (k == 0 || two);
      const long long off = (long long)(row + k) * p.D + c0;
      const int b = (row + k) / p.T;
      ux[k] = ok ? *reinterpret_cast<const uint4*>(p.x + off) : zero;
      uy[k] = (ok && p.y != nullptr) ? *reinterpret_cast<const uint4*>(p.y + off) : zero;
      ug[k] = (ok && p.y != nullptr && p.gate != nullptr)
                  ? *reinterpret_cast<const uint4*>(p.gate + (long long)b * p.gate_bs + c0) : zero;
    }
    float x[2][8], ss[2] = {0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      unpack8(ux[k], x[k]);
      if (p.y != nullptr) {
        float y[8];
        unpack8(uy[k], y);
        if (p.gate != nullptr) {
          float g[8];
          unpack8(ug[k], g);
#pragma unroll
          for (int i = 0; i < 8; ++i) x[k][i] = bf16_round(x[k][i] + bf16_round(g[i] * y[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) x[k][i] = bf16_round(x[k][i] + y[i]);
        }
        if (active && (k == 0 || two)) store8(p.x_out + (long long)(row + k) * p.D + c0, x[k]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss[k] += x[k][i] * x[k][i];
    }
    const float2 tot = block_sum2(ss[0], ss[1], red, slot);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (k == 1 && !two) break;
      const float r = rsqrtf((k == 0 ? tot.x : tot.y) / p.D + p.eps);
      if (threadIdx.x == 0) p.rstd[row + k] = r;
      if (!active) continue;
      const int b = (row + k) / p.T;
      const float rb = bf16_round(r);
      float h[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = bf16_round(x[k][i] * rb) * w[i];
      if (p.scale != nullptr) {
        float sc[8], sh[8];
        load8(p.scale + (long long)b * p.mod_bs + c0, sc);
        load8(p.shift + (long long)b * p.mod_bs + c0, sh);
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = h[i] * (1.f + sc[i]) + sh[i];
      }
      store8(p.h + (long long)(row + k) * p.D + c0, h);
    }
  }
}

// Warp-per-row variant for D = 256 NC: lane l owns columns k * 256 + 8 l (k < NC), 16-byte accesses. All NC x / y
// (and gate) loads of a row are issued before any use, the row sum of squares is a shuffle reduction (no block
// barrier), and x_new stays packed bf16 between the two passes, so 2 blocks of 8 warps fit per SM with every
// warp's loads in flight. The bf16-rounded steps run as packed bf16x2 arithmetic on the FMA pipe: x + bf16(g y)
// (two roundings, as the autocast ops) and bf16(x_new rstd_bf16) (the product of two bf16 values is exact in fp32,
// so one bf16x2 multiply rounds it identically); fp32 <-> bf16 conversions per element otherwise saturate the
// conversion unit (XU) before HBM.
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  return u;
}
__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 b) { return *reinterpret_cast<uint32_t*>(&b); }

template <int NC>
__global__ void __launch_bounds__(256, 2) adanorm_fwd_warp_kernel(AdaNormFwdParams p) {
  const int row = blockIdx.x * 8 + warp_id();
  if (row >= p.M) return;
  const int c_lane = lane_id() * 8;
  const int b = row / p.T;
  const long long off = (long long)row * p.D + c_lane;
  const bool res = p.y != nullptr, gated = res && p.gate != nullptr;
  uint4 ux[NC], uy[NC], ug[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k) ux[k] = *reinterpret_cast<const uint4*>(p.x + off + k * 256);
  if (res) {
#pragma unroll
    for (int k = 0; k < NC; ++k) uy[k] = *reinterpret_cast<const uint4*>(p.y + off + k * 256);
  }
  if (gated) {
#pragma unroll
    for (int k = 0; k < NC; ++k)
      ug[k] = *reinterpret_cast<const uint4*>(p.gate + (long long)b * p.gate_bs + k * 256 + c_lane);
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    uint32_t* xw = reinterpret_cast<uint32_t*>(&ux[k]);
    if (res) {
      const uint32_t* yw = reinterpret_cast<const uint32_t*>(&uy[k]);
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(&ug[k]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        xw[i] = bf2_bits(gated ? __hadd2(as_bf2(xw[i]), __hmul2(as_bf2(gw[i]), as_bf2(yw[i])))
                               : __hadd2(as_bf2(xw[i]), as_bf2(yw[i])));
      *reinterpret_cast<uint4*>(p.x_out + off + k * 256) = ux[k];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(as_bf2(xw[i]));
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / p.D + p.eps);
  if (lane_id() == 0) p.rstd[row] = r;
  const __nv_bfloat162 rb2 = __float2bfloat162_rn(r);
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int c = k * 256 + c_lane;
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&ux[k]);
    const float4 w0 = *reinterpret_cast<const float4*>(p.w + c), w1 = *reinterpret_cast<const float4*>(p.w + c + 4);
    const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float h[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 n = __bfloat1622float2(__hmul2(as_bf2(xw[i]), rb2));
      h[2 * i] = n.x * w[2 * i];
      h[2 * i + 1] = n.y * w[2 * i + 1];
    }
    if (p.scale != nullptr) {
      float sc[8], sh[8];
      load8(p.scale + (long long)b * p.mod_bs + c, sc);
      load8(p.shift + (long long)b * p.mod_bs + c, sh);
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = fmaf(h[i], 1.f + sc[i], sh[i]);
    }
    *reinterpret_cast<uint4*>(p.h + off + k * 256) = pack8(h);
  }
}

// ------------------------------------------------------------------------------------------------------------------
// adanorm backward: row pass (dx, dy, per-CTA partial column sums)
// partial layout: [B][chunks][4][D] = dshift, dscale, dgate, dw
// ------------------------------------------------------------------------------------------------------------------
// Two rows per iteration: both rows' inputs are loaded up front (raw bf16, 16 bytes per tensor and thread) so
// twice the loads are in flight, and the two row dot products share one block reduction (half the barriers).
__device__ __forceinline__ float2 block_sum2(float a, float b, float* red, int slot) {
  a = warp_sum(a);
  b = warp_sum(b);
  const int nw = (blockDim.x + 31) >> 5;
  if (lane_id() == 0) {
    red[slot * 64 + warp_id()] = a;
    red[slot * 64 + 32 + warp_id()] = b;
  }
  __syncthreads();
  float sa = 0.f, sb = 0.f;
  for (int i = 0; i < nw; ++i) {
    sa += red[slot * 64 + i];
    sb += red[slot * 64 + 32 + i];
  }
  return make_float2(sa, sb);
}

__device__ __forceinline__ float block_sum1(float a, float* red, int slot) {
  a = warp_sum(a);
  const int nw = (blockDim.x + 31) >> 5;
  if (lane_id() == 0) red[slot * 64 + warp_id()] = a;
  __syncthreads();
  float sa = 0.f;
  for (int i = 0; i < nw; ++i) sa += red[slot * 64 + i];
  return sa;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <int R>
__global__ void __launch_bounds__(512) adanorm_bwd_kernel(AdaNormBwdParams p) {
  __shared__ float red[128];
  const int c0 = threadIdx.x * 8;
  const bool active = c0 < p.D;
  const int b = blockIdx.y, j = blockIdx.x;
  const int row0 = b * p.T + j * p.rows_per_cta;
  const int row1 = min((b + 1) * p.T, row0 + p.rows_per_cta);
  const bool has_dxe = p.dxe != nullptr, has_y = p.y != nullptr && p.gate != nullptr;
  // per channel: cw = (1 + scale) w, the gate g; the sums are dshift = sum dh, S = sum dh n (dscale = w S and
  // dw = (1 + scale) S, formed at the end) and dgate = sum dx y
  float cw[8], g[8];
  float a_shift[8], a_s[8], a_gate[8];
  auto channel_consts = [&](float (&w)[8], float (&sc1)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w[i] = active ? p.w[c0 + i] : 0.f;
      sc1[i] = 1.f;
    }
    if (active && p.scale != nullptr) {
      load8(p.scale + (long long)b * p.mod_bs + c0, sc1);
#pragma unroll
      for (int i = 0; i < 8; ++i) sc1[i] += 1.f;
    }
  };
  {
    float w[8], sc1[8];
    channel_consts(w, sc1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      cw[i] = sc1[i] * w[i];
      g[i] = 1.f;
      a_shift[i] = a_s[i] = a_gate[i] = 0.f;
    }
  }
  if (active && p.gate != nullptr) load8(p.gate + (long long)b * p.gate_bs + c0, g);
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  // R rows per block reduction; the next R rows' dh / x_new loads are issued before this group's reduction and
  // stores, so loads stay in flight across the block barrier (without it every group waited for its loads with
  // nothing else outstanding)
  struct Pair {
    uint4 dh[R], xn[R];
    float r[R];
  };
  auto fetch = [&](int row, Pair& f) {
    const bool two = row + 1 < row1;
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const bool ok = active && (k == 0 || two);
      const long long off = (long long)(row + k) * p.D + c0;
      f.dh[k] = ok ? *reinterpret_cast<const uint4*>(p.dh + off) : zero;
      f.xn[k] = ok ? *reinterpret_cast<const uint4*>(p.xn + off) : zero;
      f.r[k] = (k == 0 || two) ? p.rstd[row + k] : 0.f;
    }
  };
  Pair cur;
  if (row0 < row1) fetch(row0, cur);
  int slot = 0;
  for (int row = row0; row < row1; row += R, slot ^= 1) {
    const bool two = R == 2 && row + 1 < row1;
    const bool more = row + R < row1;
    Pair nxt;
    if (more) fetch(row + R, nxt);
    uint4 u_e[R], u_y[R];  // needed only after the reduction: issued now, they arrive during it
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const bool ok = active && (k == 0 || two);
      const long long off = (long long)(row + k) * p.D + c0;
      u_e[k] = (ok && has_dxe) ? *reinterpret_cast<const uint4*>(p.dxe + off) : zero;
      u_y[k] = (ok && has_y) ? *reinterpret_cast<const uint4*>(p.y + off) : zero;
    }
    float dot[2] = {0.f, 0.f};
#pragma unroll
    for (int k = 0; k < R; ++k) {
      float dh[8], xn[8];
      unpack8(cur.dh[k], dh);
      unpack8(cur.xn[k], xn);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float n = xn[i] * cur.r[k];
        const float dn = dh[i] * n;
        a_shift[i] += dh[i];
        a_s[i] += dn;
        dot[k] += dn * cw[i];
      }
    }
    const float2 tot = R == 2 ? block_sum2(dot[0], dot[1], red, slot) : make_float2(block_sum1(dot[0], red, slot), 0.f);
    const float mdot[2] = {tot.x / p.D, tot.y / p.D};
#pragma unroll
    for (int k = 0; k < R; ++k) {
      if (!active || (k == 1 && !two)) continue;
      const long long off = (long long)(row + k) * p.D + c0;
      float dh[8], xn[8], dx[8];
      unpack8(cur.dh[k], dh);
      unpack8(cur.xn[k], xn);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float n = xn[i] * cur.r[k];
        dx[i] = cur.r[k] * (dh[i] * cw[i] - n * mdot[k]);
      }
      if (has_dxe) {
        float e[8];
        unpack8(u_e[k], e);
#pragma unroll
        for (int i = 0; i < 8; ++i) dx[i] += e[i];
      }
      store8(p.dx + off, dx);
      if (has_y) {
        float y[8], dy[8];
        unpack8(u_y[k], y);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          a_gate[i] += dx[i] * y[i];
          dy[i] = dx[i] * g[i];
        }
        store8(p.dy + off, dy);
      }
    }
    if (more) cur = nxt;
  }
  if (active) {
    float w[8], sc1[8];
    channel_consts(w, sc1);
    float* dst = p.partial + ((long long)(b * p.chunks + j) * 4) * p.D + c0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      dst[i] = a_shift[i];
      dst[p.D + i] = w[i] * a_s[i];
      dst[2 * p.D + i] = a_gate[i];
      dst[3 * p.D + i] = sc1[i] * a_s[i];
    }
  }
}

// Reduce the partials: one thread per (sample, channel) sums its chunks; dw[c] += (atomically) over samples.
__global__ void adanorm_bwd_reduce_kernel(const float* __restrict__ partial, float* __restrict__ dshift,
                                          float* __restrict__ dscale, float* __restrict__ dgate,
                                          float* __restrict__ dw, int B, int chunks, int D) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (c >= D) return;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  for (int j = 0; j < chunks; ++j) {
    const float* src = partial + ((long long)(b * chunks + j) * 4) * D + c;
    s0 += src[0];
    s1 += src[D];
    s2 += src[2 * D];
    s3 += src[3 * D];
  }
  if (dshift) dshift[(long long)b * D + c] = s0;
  if (dscale) dscale[(long long)b * D + c] = s1;
  if (dgate) dgate[(long long)b * D + c] = s2;
  atomicAdd(&dw[c], s3);
}

cudaError_t adanorm_fwd_launch(const AdaNormFwdParams& p, cudaStream_t s) {
  if (p.D % 256 == 0 && p.D <= 2048) {  // warp per row (wider rows would spill the held row)
    const unsigned grid = (unsigned)((p.M + 7) / 8);
    switch (p.D / 256) {
      case 4: adanorm_fwd_warp_kernel<4><<<grid, 256, 0, s>>>(p); return cudaGetLastError();
      case 8: adanorm_fwd_warp_kernel<8><<<grid, 256, 0, s>>>(p); return cudaGetLastError();
      default: break;
    }
  }
  const int threads = ((p.D / 8 + 31) / 32) * 32;
  const int grid = (p.M + p.rows_per_cta - 1) / p.rows_per_cta;
  adanorm_fwd_kernel<<<grid, threads, 0, s>>>(p);
  return cudaGetLastError();
}

static int g_qknorm_bwd_unroll = 4;  // heads per lane group with loads in flight (2 or 4)
cudaError_t qknorm_set_bwd_unroll(int u) {
  if (u != 2 && u != 4) return cudaErrorInvalidValue;
  g_qknorm_bwd_unroll = u;
  return cudaSuccess;
}

// rows per block reduction: 2 (default; 128 registers with a few spilled to L1) measured 0.199 ms at 32 x 1024 x 2048
// against 0.236 ms for 1 (116 registers, no spills) and 0.216-0.239 ms before the next pair's loads were issued early
static int g_adanorm_bwd_rows = 2;
cudaError_t adanorm_set_bwd_rows(int rows) {
  if (rows != 1 && rows != 2) return cudaErrorInvalidValue;
  g_adanorm_bwd_rows = rows;
  return cudaSuccess;
}

cudaError_t adanorm_bwd_launch(const AdaNormBwdParams& p, float* dshift, float* dscale, float* dgate, float* dw,
                               cudaStream_t s) {
  const int threads = ((p.D / 8 + 31) / 32) * 32;
  dim3 grid(p.chunks, p.M / p.T);
  if (g_adanorm_bwd_rows == 1) adanorm_bwd_kernel<1><<<grid, threads, 0, s>>>(p);
  else adanorm_bwd_kernel<2><<<grid, threads, 0, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  adanorm_bwd_reduce_kernel<<<dim3((p.D + 127) / 128, p.M / p.T), 128, 0, s>>>(p.partial, dshift, dscale, dgate,
                                                                               dw, p.M / p.T, p.chunks, p.D);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------------------------
// q/k RMSNorm + RoPE. HD / 8 lanes per (row, head) item, 8 contiguous elements (16 bytes) per lane, so a warp
// covers 32 / (HD / 8) items; RoPE pairs (even, odd) never straddle lanes.
// ------------------------------------------------------------------------------------------------------------------
template <int LPH>
__device__ __forceinline__ float group_sum(float v) {  // sum over aligned groups of LPH lanes
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ void load8f(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
}

// One warp per token row walks that row's q and k heads, HD / 8 lanes per head (8 elements per lane), several heads
// per load batch: the row's RoPE table entries and the norm weights are read once per warp and reused for every head
// (per-head table reads made the table traffic twice the activation traffic), and each lane keeps UNROLL 16-byte
// loads in flight.
template <int HD>
__global__ void __launch_bounds__(256) qknorm_rope_fwd_kernel(QKNormRopeParams p) {
  constexpr int LPH = HD / 8, HPI = 32 / LPH, UNROLL = 4;  // lanes per head, heads per pass, passes per batch
  const int heads = p.hq + p.hkv;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + warp_id();
  if (row >= p.M) return;  // whole warps leave together: the shuffles below stay warp-uniform
  const int sub = lane_id() / LPH;
  const int e0 = (lane_id() % LPH) * 8;
  float cs[8], sn[8], wq[8], wk[8];
  if (p.cos != nullptr) {
    const long long b = row / p.T, t = row % p.T;
    load8f(p.cos + b * p.rope_bs + t * HD + e0, cs);
    load8f(p.sin + b * p.rope_bs + t * HD + e0, sn);
  }
  if (p.q_w != nullptr) load8f(p.q_w + e0, wq);
  if (p.k_w != nullptr) load8f(p.k_w + e0, wk);
  const bf16* src = p.qkv + row * p.ld_qkv;
  for (int h0 = 0; h0 < heads; h0 += UNROLL * HPI) {
    uint4 ux[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int hh = h0 + u * HPI + sub;
      ux[u] = hh < heads ? *reinterpret_cast<const uint4*>(src + (long long)hh * HD + e0) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int hh = h0 + u * HPI + sub;
      const bool valid = hh < heads, is_q = hh < p.hq;
      const float* nw = is_q ? p.q_w : p.k_w;
      const uint32_t* xw = reinterpret_cast<const uint32_t*>(&ux[u]);
      float x[8];
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(as_bf2(xw[i]));
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
      ss = group_sum<LPH>(ss);  // every lane takes part (q_w / k_w presence is uniform per head group only)
      if (nw != nullptr) {
        const float r = rsqrtf(ss / HD + p.eps);
        const __nv_bfloat162 rb2 = __float2bfloat162_rn(r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // bf16(x rstd_bf16): one packed multiply, then the fp32 weight
          const float2 n = __bfloat1622float2(__hmul2(as_bf2(xw[i]), rb2));
          x[2 * i] = n.x * (is_q ? wq[2 * i] : wk[2 * i]);
          x[2 * i + 1] = n.y * (is_q ? wq[2 * i + 1] : wk[2 * i + 1]);
        }
        if (valid && e0 == 0)
          (is_q ? p.rstd_q : p.rstd_k)[row * (is_q ? p.hq : p.hkv) + (is_q ? hh : hh - p.hq)] = r;
      }
      if (p.cos != nullptr) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float a = x[i], c = x[i + 1];
          x[i] = a * cs[i] - c * sn[i];
          x[i + 1] = c * cs[i + 1] + a * sn[i + 1];
        }
      }
      if (valid) {
        bf16* dst = is_q ? p.q_out + row * p.ld_q + (long long)hh * HD + e0
                         : p.k_out + row * p.ld_k + (long long)(hh - p.hq) * HD + e0;
        *reinterpret_cast<uint4*>(dst) = pack8(x);
      }
    }
  }
}

// Backward: dq / dk (post-RoPE) -> d(pre-norm q / k) written into dqkv; dw_q, dw_k accumulated (+=).
// Mirror of the forward's layout: one warp per token row walks all of the row's q and k heads, HD / 8 lanes per head,
// so the row's RoPE table entries and the norm weights are loaded once per row, and each lane keeps UNROLL heads'
// loads (incoming gradient, pre-norm input) in flight. dq may be the attention backward's fp32 accumulator (then no
// separate fp32 -> bf16 conversion pass runs before this one). Persistent grid: a warp walks rows with a grid stride,
// keeps its dw partials in registers (a lane's channel slice e0 is the same for every head), then one shared-memory
// reduction and one global atomic per element and CTA.
template <int HD>
__device__ __forceinline__ void load8_any(const void* base, long long off, bool f32, float (&g)[8]) {
  if (f32) {
    load8f(reinterpret_cast<const float*>(base) + off, g);
  } else {
    load8(reinterpret_cast<const bf16*>(base) + off, g);
  }
}

template <int HD, int UNROLL>
__global__ void __launch_bounds__(256, 2) qknorm_rope_bwd_kernel(QKNormRopeParams p, const void* __restrict__ dq,
                                                              long long ld_dq, int dq_f32,
                                                              const bf16* __restrict__ dk, long long ld_dk,
                                                              bf16* __restrict__ dqkv, long long ld_dqkv,
                                                              float* __restrict__ dwq, float* __restrict__ dwk) {
  constexpr int LPH = HD / 8, HPI = 32 / LPH;
  __shared__ float s_dw[2][HD];
  for (int i = threadIdx.x; i < 2 * HD; i += blockDim.x) (&s_dw[0][0])[i] = 0.f;
  __syncthreads();
  const int heads = p.hq + p.hkv;
  const int sub = lane_id() / LPH;
  const int e0 = (lane_id() % LPH) * 8;
  const bool norm = p.q_w != nullptr;  // q_w and k_w are both given or both absent
  float wq[8], wk[8], acc_q[8], acc_k[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc_q[i] = acc_k[i] = wq[i] = wk[i] = 0.f;
  if (norm) {
    load8f(p.q_w + e0, wq);
    load8f(p.k_w + e0, wk);
  }
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + warp_id(); row < p.M; row += warps) {
    float cs[8], sn[8];
    if (p.cos != nullptr) {
      const long long b = row / p.T, t = row % p.T;
      load8f(p.cos + b * p.rope_bs + t * HD + e0, cs);
      load8f(p.sin + b * p.rope_bs + t * HD + e0, sn);
    }
    for (int h0 = 0; h0 < heads; h0 += UNROLL * HPI) {
      float g[UNROLL][8];
      uint4 ux[UNROLL];
      float r[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {  // every load of the batch first
        const int hh = h0 + u * HPI + sub;
        const bool valid = hh < heads, is_q = hh < p.hq;
        if (valid) {
          if (is_q) load8_any<HD>(dq, row * ld_dq + (long long)hh * HD + e0, dq_f32 != 0, g[u]);
          else load8(dk + row * ld_dk + (long long)(hh - p.hq) * HD + e0, g[u]);
          ux[u] = norm ? *reinterpret_cast<const uint4*>(p.qkv + row * p.ld_qkv + (long long)hh * HD + e0)
                       : make_uint4(0u, 0u, 0u, 0u);
          r[u] = norm ? (is_q ? p.rstd_q[row * p.hq + hh] : p.rstd_k[row * p.hkv + (hh - p.hq)]) : 0.f;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) g[u][i] = 0.f;
          ux[u] = make_uint4(0u, 0u, 0u, 0u);
          r[u] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int hh = h0 + u * HPI + sub;
        const bool valid = hh < heads, is_q = hh < p.hq;
        if (p.cos != nullptr) {  // transpose of the rotation
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            const float a = g[u][i], c = g[u][i + 1];
            g[u][i] = a * cs[i] + c * sn[i + 1];
            g[u][i + 1] = c * cs[i + 1] - a * sn[i];
          }
        }
        if (norm) {
          const uint32_t* xw = reinterpret_cast<const uint32_t*>(&ux[u]);
          float n[8];
          float dot = 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(as_bf2(xw[i]));
            n[2 * i] = f.x * r[u];
            n[2 * i + 1] = f.y * r[u];
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (is_q) acc_q[i] += g[u][i] * n[i];
            else acc_k[i] += g[u][i] * n[i];
            g[u][i] *= is_q ? wq[i] : wk[i];  // d(normalised x)
            dot += g[u][i] * n[i];
          }
          dot = group_sum<LPH>(dot) / HD;
#pragma unroll
          for (int i = 0; i < 8; ++i) g[u][i] = r[u] * (g[u][i] - n[i] * dot);
        }
        if (valid) store8(dqkv + row * ld_dqkv + (long long)hh * HD + e0, g[u]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    atomicAdd(&s_dw[0][e0 + i], acc_q[i]);
    atomicAdd(&s_dw[1][e0 + i], acc_k[i]);
  }
  __syncthreads();
  if (norm && dwq != nullptr)
    for (int i = threadIdx.x; i < HD; i += blockDim.x) atomicAdd(&dwq[i], s_dw[0][i]);
  if (norm && dwk != nullptr)
    for (int i = threadIdx.x; i < HD; i += blockDim.x) atomicAdd(&dwk[i], s_dw[1][i]);
}

cudaError_t qknorm_rope_fwd_launch(const QKNormRopeParams& p, cudaStream_t s) {
  const unsigned grid = (unsigned)(((long long)p.M + 7) / 8);  // one warp per token row, 8 warps per block
  if (p.hd == 128) qknorm_rope_fwd_kernel<128><<<grid, 256, 0, s>>>(p);
  else if (p.hd == 64) qknorm_rope_fwd_kernel<64><<<grid, 256, 0, s>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t qknorm_rope_bwd_launch(const QKNormRopeParams& p, const void* dq, long long ld_dq, bool dq_f32,
                                   const bf16* dk, long long ld_dk, bf16* dqkv, long long ld_dqkv, float* dwq,
                                   float* dwk, cudaStream_t s) {
  const long long rows = p.M;  // one warp per row, 8 warps per block, at most 4 blocks per SM (grid stride)
  const unsigned grid = (unsigned)std::min<long long>((rows + 7) / 8, (long long)num_sms() * 4);
  const int f32 = dq_f32 ? 1 : 0;
#define TGO_QKB(HD, U) qknorm_rope_bwd_kernel<HD, U><<<grid, 256, 0, s>>>(p, dq, ld_dq, f32, dk, ld_dk, dqkv, \
                                                                          ld_dqkv, dwq, dwk)
  if (p.hd == 128) {
    if (g_qknorm_bwd_unroll == 4) TGO_QKB(128, 4); else TGO_QKB(128, 2);
  } else if (p.hd == 64) {
    if (g_qknorm_bwd_unroll == 4) TGO_QKB(64, 4); else TGO_QKB(64, 2);
  } else {
    return cudaErrorInvalidValue;
  }
#undef TGO_QKB
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------------------------
// SwiGLU on [a | b] rows: g = silu(a) * b (silu rounded to bf16 first, as an autocast bf16 silu would be)
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float silu_f(float a) { return a / (1.f + __expf(-a)); }

// Flat index over 8-element groups (n8 < 2^31, checked by the launchers): 32-bit index arithmetic (a 64-bit division
// per group dominated the instruction count), two groups per thread per step with all their loads issued first.
__global__ void swiglu_fwd_kernel(const bf16* __restrict__ ab, bf16* __restrict__ g, int n8, int H) {
  const unsigned H8 = (unsigned)(H / 8);
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < (unsigned)n8; i += 2 * stride) {
    const bool two = i + stride < (unsigned)n8;
    float a[2][8], b[2][8];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const unsigned ii = k == 0 ? i : (two ? i + stride : i);
      const unsigned row = ii / H8, c = (ii - row * H8) * 8;
      load8(ab + (long long)row * 2 * H + c, a[k]);
      load8(ab + (long long)row * 2 * H + H + c, b[k]);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (k == 1 && !two) break;
      const unsigned ii = i + k * stride;
      const unsigned row = ii / H8, c = (ii - row * H8) * 8;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = bf16_round(silu_f(a[k][e])) * b[k][e];
      store8(g + (long long)row * H + c, o);
    }
  }
}

__global__ void swiglu_bwd_kernel(const bf16* __restrict__ ab, const bf16* __restrict__ dg, bf16* __restrict__ dab,
                                  int n8, int H) {
  const unsigned H8 = (unsigned)(H / 8);
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < (unsigned)n8; i += 2 * stride) {
    const bool two = i + stride < (unsigned)n8;
    float a[2][8], b[2][8], d[2][8];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const unsigned ii = k == 0 ? i : (two ? i + stride : i);
      const unsigned row = ii / H8, c = (ii - row * H8) * 8;
      load8(ab + (long long)row * 2 * H + c, a[k]);
      load8(ab + (long long)row * 2 * H + H + c, b[k]);
      load8(dg + (long long)row * H + c, d[k]);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (k == 1 && !two) break;
      const unsigned ii = i + k * stride;
      const unsigned row = ii / H8, c = (ii - row * H8) * 8;
      float da[8], db[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float sg = 1.f / (1.f + __expf(-a[k][e]));
        const float sv = a[k][e] * sg;
        db[e] = d[k][e] * sv;
        da[e] = d[k][e] * b[k][e] * sg * (1.f + a[k][e] * (1.f - sg));
      }
      store8(dab + (long long)row * 2 * H + c, da);
      store8(dab + (long long)row * 2 * H + H + c, db);
    }
  }
}

cudaError_t swiglu_fwd_launch(const bf16* ab, bf16* g, long long M, int H, cudaStream_t s) {
  const long long n8 = M * (H / 8);
  if (n8 >= (1ll << 31) || H % 8 != 0) return cudaErrorInvalidValue;
  const int grid = (int)std::min<long long>((n8 + 511) / 512, (long long)num_sms() * 8);
  swiglu_fwd_kernel<<<grid, 256, 0, s>>>(ab, g, (int)n8, H);
  return cudaGetLastError();
}

cudaError_t swiglu_bwd_launch(const bf16* ab, const bf16* dg, bf16* dab, long long M, int H, cudaStream_t s) {
  const long long n8 = M * (H / 8);
  if (n8 >= (1ll << 31) || H % 8 != 0) return cudaErrorInvalidValue;
  const int grid = (int)std::min<long long>((n8 + 511) / 512, (long long)num_sms() * 8);
  swiglu_bwd_kernel<<<grid, 256, 0, s>>>(ab, dg, dab, (int)n8, H);
  return cudaGetLastError();
}

}  // namespace tgo
