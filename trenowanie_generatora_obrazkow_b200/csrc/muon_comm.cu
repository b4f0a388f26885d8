// Sharded Muon over NVLink peer memory: the gradient reduce-scatter to the owner of each matrix, the owner's
// momentum / Nesterov / Newton-Schulz input preparation, and the all-gather of the orthogonalised updates fused
// with the parameter update. Reference semantics: aurora/muon.py:89-194 (every rank all-reduces all gradients,
// keeps the full momentum, orthogonalises its contiguous slice of each shape bucket and all-gathers the bf16
// updates through NCCL). Here a matrix's gradient only travels to its owner, the momentum exists only on the
// owner, and the update all-gather writes straight into every peer's update buffer, where the same kernel applies
// it to the fp32 master weights and refreshes their bf16 shadow copies (read by the next forward's GEMMs).
//
// muon_rs        (one launch per gradient bucket, from the backward pass, on the gradient-reduction stream)
//   phase 0  wait until every peer finished reading this rank's staging in the previous launch (done flags),
//            cast this CTA's chunk of the fp32 bucket into the bf16 staging, ready[rank][cta] := epoch at every peer
//   phase 1  wait for every peer's ready flags, then for this CTA's share of the rank's owned segments sum the
//            peers' bf16 staging over NVLink loads in fp32, scale by 1 / world, store fp32 into the owned-gradient
//            buffer and accumulate its sum of squares (for the global gradient-norm clip)
//   phase 2  done[rank][cta] := epoch at every peer
// muon_momentum  (local) coef-scaled gradient -> momentum (fp32, or bf16 with stochastic rounding) -> Nesterov
//            direction as the bf16 Newton-Schulz input
// muon_ag_apply  (one launch per optimizer step, after Newton-Schulz)
//   phase 0  push this CTA's chunk of the rank's owned updates into every peer's update buffer (16-byte NVLink
//            stores), ag[rank][cta] := epoch at every peer
//   phase 1  wait for every peer's ag flags; for this CTA's chunk of every matrix: p = p (1 - lr wd) - lr s U, and
//            the bf16 shadow := bf16(p)
// Flag waits are bounded by a globaltimer deadline: a peer that never arrives turns into ERR_PEER_TIMEOUT in the
// error word and the kernel returns. No cluster or TMA multicast is used.
#include "comm.cuh"
#include "kernels.h"

namespace tgo {

// Wait until all world x C flags of `flags` equal v (threads of the block share the polling). Bounded.
__device__ bool wait_all_flags(const uint32_t* flags, int count, uint32_t v, uint64_t deadline, int* err,
                               int* ok_sh) {
  for (int i = threadIdx.x; i < count; i += blockDim.x)
    if (!flag_wait(flags + i, v, deadline, err)) *ok_sh = 0;
  __syncthreads();
  return *ok_sh != 0;
}

__device__ __forceinline__ void signal_all_peers(uint32_t* const* flags, int world, long long slot, uint32_t v) {
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) flag_store_release(flags[threadIdx.x] + slot, v);
}

__device__ __forceinline__ float block_sum(float v) {
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
  if (w == 0)
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------------------------------------------------------
// reduce-scatter to owners
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) muon_rs_kernel(MuonRSParams p) {
  const int c = blockIdx.x, C = gridDim.x;
  __shared__ int ok_sh;
  if (threadIdx.x == 0) ok_sh = 1;
  __syncthreads();
  const uint64_t deadline = global_ns() + p.timeout_ns;
  const int WC = p.world * C;
  uint32_t* ready = p.flags[p.rank];
  uint32_t* done = p.flags[p.rank] + WC;
  // ---- phase 0: staging free again? then cast my chunk ----
  if (p.prev_epoch != 0 && !wait_all_flags(done, WC, p.prev_epoch, deadline, p.err, &ok_sh)) return;
  const long long chunk = ((p.n + C - 1) / C + 7) / 8 * 8;
  const long long c0 = (long long)c * chunk, c1 = min(p.n, c0 + chunk);
  __nv_bfloat16* stage = p.staging[p.rank];
  for (long long i = c0 + threadIdx.x * 8; i < c1; i += (long long)blockDim.x * 8) {
    if (i + 8 <= c1) {
      const float4 a = *reinterpret_cast<const float4*>(p.grads + i);
      const float4 b = *reinterpret_cast<const float4*>(p.grads + i + 4);
      uint4 u;
      u.x = pack_bf16x2(a.x, a.y);
      u.y = pack_bf16x2(a.z, a.w);
      u.z = pack_bf16x2(b.x, b.y);
      u.w = pack_bf16x2(b.z, b.w);
      *reinterpret_cast<uint4*>(stage + i) = u;
    } else {
      for (long long k = i; k < c1; ++k) stage[k] = __float2bfloat16_rn(p.grads[k]);
    }
  }
  signal_all_peers(p.flags, p.world, (long long)p.rank * C + c, p.epoch);
  // ---- phase 1: reduce my owned segments (this CTA's share) ----
  if (!wait_all_flags(ready, WC, p.epoch, deadline, p.err, &ok_sh)) return;
  const long long ochunk = ((p.owned + C - 1) / C + 7) / 8 * 8;
  const long long o0 = (long long)c * ochunk, o1 = min(p.owned, o0 + ochunk);
  float sq = 0.f;
  long long seg_base = 0;  // owned index of the current segment's first element
  for (int s = 0; s < p.nsegs && seg_base < o1; ++s) {
    const long long src = p.segs[3 * s], dst = p.segs[3 * s + 1], n = p.segs[3 * s + 2];
    const long long lo = max(o0, seg_base), hi = min(o1, seg_base + n);
    if (lo < hi) {
      const long long a = lo - seg_base, b = hi - seg_base;  // element range inside this segment
      const bool vec = ((src + a) % 8 == 0) && ((dst + a) % 4 == 0);
      if (vec) {
        for (long long i = a + threadIdx.x * 8; i < b; i += (long long)blockDim.x * 8) {
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (i + 8 <= b) {
            for (int q = 0; q < p.world; ++q) {
              const int peer = (p.rank + q) % p.world;
              const uint4 u = ld_v4_volatile(p.staging[peer] + src + i);
              const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float2 f = __bfloat1622float2(h[k]);
                acc[2 * k] += f.x;
                acc[2 * k + 1] += f.y;
              }
            }
            float4* o = reinterpret_cast<float4*>(p.g_owned + dst + i);
            float r[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              r[k] = acc[k] * p.scale;
              sq += r[k] * r[k];
            }
            o[0] = make_float4(r[0], r[1], r[2], r[3]);
            o[1] = make_float4(r[4], r[5], r[6], r[7]);
          } else {
            for (long long j = i; j < b; ++j) {
              float acc1 = 0.f;
              for (int q = 0; q < p.world; ++q) {
                acc1 += __bfloat162float(ld_bf16_volatile(p.staging[(p.rank + q) % p.world] + src + j));
              }
              const float r = acc1 * p.scale;
              sq += r * r;
              p.g_owned[dst + j] = r;
            }
          }
        }
      } else {
        for (long long j = a + threadIdx.x; j < b; j += blockDim.x) {
          float acc1 = 0.f;
          for (int q = 0; q < p.world; ++q) {
            acc1 += __bfloat162float(ld_bf16_volatile(p.staging[(p.rank + q) % p.world] + src + j));
          }
          const float r = acc1 * p.scale;
          sq += r * r;
          p.g_owned[dst + j] = r;
        }
      }
    }
    seg_base += n;
  }
  sq = block_sum(sq);
  if (threadIdx.x == 0 && p.sumsq != nullptr && sq != 0.f) atomicAdd(p.sumsq, sq);
  // ---- phase 2: my reads of every peer's staging are finished ----
  signal_all_peers(p.flags, p.world, WC + (long long)p.rank * C + c, p.epoch);
}

// ------------------------------------------------------------------------------------------------------------------
// owner-side momentum + Nesterov direction -> bf16 Newton-Schulz input
// ------------------------------------------------------------------------------------------------------------------
// Stochastic rounding noise: splitmix64 (Steele, Lea, Flood 2014; public-domain finaliser by S. Vigna) of
// (seed, element index), 16 uniform bits added below the bf16 mantissa before truncation.
__device__ __forceinline__ uint32_t sr_bits(unsigned long long seed, long long i) {
  unsigned long long z = seed + 0x9E3779B97F4A7C15ull * (unsigned long long)(i + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (uint32_t)(z & 0xFFFFu);
}
__device__ __forceinline__ __nv_bfloat16 round_stochastic(float x, unsigned long long seed, long long i) {
  uint32_t b = __float_as_uint(x);
  if ((b & 0x7F800000u) != 0x7F800000u) b = (b + sr_bits(seed, i)) & 0xFFFF0000u;  // finite values only
  else b &= 0xFFFF0000u;
  return __ushort_as_bfloat16((unsigned short)(b >> 16));
}

__global__ void muon_momentum_kernel(MuonMomentumParams p) {
  const float coef = *p.coef;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < p.n; i += (long long)gridDim.x * blockDim.x) {
    const float g = p.g[i] * coef;
    float m = p.buf_f32 != nullptr ? p.buf_f32[i] : __bfloat162float(p.buf_bf16[i]);
    m = m + (1.f - p.mu) * (g - m);  // lerp(m, g, 1 - mu)
    if (p.buf_f32 != nullptr) p.buf_f32[i] = m;
    else p.buf_bf16[i] = round_stochastic(m, p.seed, i);
    const float mq = p.buf_f32 != nullptr ? m : __bfloat162float(p.buf_bf16[i]);
    const float d = p.nesterov ? g + p.mu * (mq - g) : mq;  // lerp(g, m, mu)
    p.x_out[i] = __float2bfloat16_rn(d);
  }
}

// ------------------------------------------------------------------------------------------------------------------
// all-gather of the updates fused with the parameter update
// ------------------------------------------------------------------------------------------------------------------
// Chunk c (of C) of every matrix segment: p = p * decay + alpha * U, the bf16 shadow := bf16(p), and the EMA
// e += ema_rate (p - e) where the segment has one.
__device__ void apply_segments(const __nv_bfloat16* U, const long long* segs, const float* coefs, int nsegs, int c,
                               int C, float ema_rate) {
  for (int s = 0; s < nsegs; ++s) {
    float* w = reinterpret_cast<float*>(segs[5 * s]);
    __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(segs[5 * s + 1]);
    const long long off = segs[5 * s + 2], n = segs[5 * s + 3];
    float* ema = reinterpret_cast<float*>(segs[5 * s + 4]);
    const float alpha = coefs[2 * s], decay = coefs[2 * s + 1];
    const long long chunk = ((n + C - 1) / C + 7) / 8 * 8;
    const long long a = (long long)c * chunk, b = min(n, a + chunk);
    const bool vec = (off % 8 == 0) && (reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
                     (sh == nullptr || reinterpret_cast<uintptr_t>(sh) % 16 == 0) &&
                     (ema == nullptr || reinterpret_cast<uintptr_t>(ema) % 16 == 0);
    long long i = a + threadIdx.x * 8;
    if (vec) {
      for (; i + 8 <= b; i += (long long)blockDim.x * 8) {
        const uint4 uu = ld_v4_volatile(U + off + i);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&uu);
        float4* wp = reinterpret_cast<float4*>(w + i);
        float4 w0 = wp[0], w1 = wp[1];
        float2 u0 = __bfloat1622float2(h[0]), u1 = __bfloat1622float2(h[1]);
        float2 u2 = __bfloat1622float2(h[2]), u3 = __bfloat1622float2(h[3]);
        w0.x = w0.x * decay + alpha * u0.x;
        w0.y = w0.y * decay + alpha * u0.y;
        w0.z = w0.z * decay + alpha * u1.x;
        w0.w = w0.w * decay + alpha * u1.y;
        w1.x = w1.x * decay + alpha * u2.x;
        w1.y = w1.y * decay + alpha * u2.y;
        w1.z = w1.z * decay + alpha * u3.x;
        w1.w = w1.w * decay + alpha * u3.y;
        wp[0] = w0;
        wp[1] = w1;
        if (sh != nullptr) {
          uint4 o;
          o.x = pack_bf16x2(w0.x, w0.y);
          o.y = pack_bf16x2(w0.z, w0.w);
          o.z = pack_bf16x2(w1.x, w1.y);
          o.w = pack_bf16x2(w1.z, w1.w);
          *reinterpret_cast<uint4*>(sh + i) = o;
        }
        if (ema != nullptr) {
          float4* ep = reinterpret_cast<float4*>(ema + i);
          float4 e0 = ep[0], e1 = ep[1];
          e0.x += ema_rate * (w0.x - e0.x);
          e0.y += ema_rate * (w0.y - e0.y);
          e0.z += ema_rate * (w0.z - e0.z);
          e0.w += ema_rate * (w0.w - e0.w);
          e1.x += ema_rate * (w1.x - e1.x);
          e1.y += ema_rate * (w1.y - e1.y);
          e1.z += ema_rate * (w1.z - e1.z);
          e1.w += ema_rate * (w1.w - e1.w);
          ep[0] = e0;
          ep[1] = e1;
        }
      }
    }
    // scalar path: misaligned segments, and the < 8-element tail of an aligned one (one thread holds it)
    long long j = vec ? i : a + threadIdx.x;
    const long long jstep = vec ? 1 : blockDim.x;
    for (; j < b; j += jstep) {
      const float u = __bfloat162float(ld_bf16_volatile(U + off + j));
      const float v = w[j] * decay + alpha * u;
      w[j] = v;
      if (sh != nullptr) sh[j] = __float2bfloat16_rn(v);
      if (ema != nullptr) ema[j] += ema_rate * (v - ema[j]);
    }
  }
}

__global__ void __launch_bounds__(512) muon_ag_apply_kernel(MuonAGParams p) {
  const int c = blockIdx.x, C = gridDim.x;
  __shared__ int ok_sh;
  if (threadIdx.x == 0) ok_sh = 1;
  __syncthreads();
  const uint64_t deadline = global_ns() + p.timeout_ns;
  // ---- phase 0: push my owned ranges (chunk c of their concatenation) to every peer ----
  const long long ochunk = ((p.owned + C - 1) / C + 7) / 8 * 8;
  const long long o0 = (long long)c * ochunk, o1 = min(p.owned, o0 + ochunk);
  long long base = 0;
  const __nv_bfloat16* mine = p.upd[p.rank];
  for (int r = 0; r < p.nown && base < o1; ++r) {
    const long long off = p.own[2 * r], n = p.own[2 * r + 1];
    const long long lo = max(o0, base), hi = min(o1, base + n);
    if (lo < hi) {
      const long long a = off + lo - base, b = off + hi - base;  // muon-space element range
      if (a % 8 == 0 && b % 8 == 0) {
        for (long long i = a + threadIdx.x * 8; i < b; i += (long long)blockDim.x * 8) {
          const uint4 u = *reinterpret_cast<const uint4*>(mine + i);
          for (int q = 1; q < p.world; ++q)
            *reinterpret_cast<uint4*>(p.upd[(p.rank + q) % p.world] + i) = u;
        }
      } else {
        for (long long i = a + threadIdx.x; i < b; i += blockDim.x)
          for (int q = 1; q < p.world; ++q) p.upd[(p.rank + q) % p.world][i] = mine[i];
      }
    }
    base += n;
  }
  signal_all_peers(p.flags, p.world, (long long)p.rank * C + c, p.epoch);
  // ---- phase 1: every update has landed; apply chunk c of every matrix ----
  if (!wait_all_flags(p.flags[p.rank], p.world * C, p.epoch, deadline, p.err, &ok_sh)) return;
  apply_segments(p.upd[p.rank], p.segs, p.coefs, p.nsegs, c, C, p.ema_rate);
}

// ------------------------------------------------------------------------------------------------------------------
// single-owner step: momentum read straight from the gradients (segment table), and the local apply
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float momentum_elem(const MuonSegMomentumParams& p, float g, long long i, float* mq) {
  float m = p.buf_f32 != nullptr ? p.buf_f32[i] : __bfloat162float(p.buf_bf16[i]);
  m = m + (1.f - p.mu) * (g - m);
  if (p.buf_f32 != nullptr) {
    p.buf_f32[i] = m;
    *mq = m;
  } else {
    const __nv_bfloat16 r = round_stochastic(m, p.seed, i);
    p.buf_bf16[i] = r;
    *mq = __bfloat162float(r);
  }
  return p.nesterov ? g + p.mu * (*mq - g) : *mq;
}

__global__ void __launch_bounds__(256) muon_seg_momentum_kernel(MuonSegMomentumParams p) {
  const int c = blockIdx.x, C = gridDim.x;
  const float coef = *p.coef;
  for (int s = 0; s < p.nsegs; ++s) {
    const float* g = reinterpret_cast<const float*>(p.segs[3 * s]);
    const long long off = p.segs[3 * s + 1], n = p.segs[3 * s + 2];
    const long long chunk = ((n + C - 1) / C + 7) / 8 * 8;
    const long long a = (long long)c * chunk, b = min(n, a + chunk);
    const bool vec = (off % 8 == 0) && (reinterpret_cast<uintptr_t>(g) % 16 == 0);
    long long i = a + threadIdx.x * 8;
    if (vec) {
      for (; i + 8 <= b; i += (long long)blockDim.x * 8) {
        const long long f = off + i;  // flat index of the first of 8 elements
        const float4 g0 = *reinterpret_cast<const float4*>(g + i);
        const float4 g1 = *reinterpret_cast<const float4*>(g + i + 4);
        const float gv[8] = {g0.x * coef, g0.y * coef, g0.z * coef, g0.w * coef,
                             g1.x * coef, g1.y * coef, g1.z * coef, g1.w * coef};
        float m[8], d[8];
        if (p.buf_f32 != nullptr) {
          float4* mp = reinterpret_cast<float4*>(p.buf_f32 + f);
          const float4 m0 = mp[0], m1 = mp[1];
          m[0] = m0.x; m[1] = m0.y; m[2] = m0.z; m[3] = m0.w;
          m[4] = m1.x; m[5] = m1.y; m[6] = m1.z; m[7] = m1.w;
#pragma unroll
          for (int k = 0; k < 8; ++k) m[k] = m[k] + (1.f - p.mu) * (gv[k] - m[k]);
          mp[0] = make_float4(m[0], m[1], m[2], m[3]);
          mp[1] = make_float4(m[4], m[5], m[6], m[7]);
        } else {
          uint4* mp = reinterpret_cast<uint4*>(p.buf_bf16 + f);
          uint4 mu4 = *mp;
          __nv_bfloat16* mb = reinterpret_cast<__nv_bfloat16*>(&mu4);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float mk = __bfloat162float(mb[k]);
            mb[k] = round_stochastic(mk + (1.f - p.mu) * (gv[k] - mk), p.seed, f + k);
            m[k] = __bfloat162float(mb[k]);
          }
          *mp = mu4;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) d[k] = p.nesterov ? gv[k] + p.mu * (m[k] - gv[k]) : m[k];
        uint4 u;
        u.x = pack_bf16x2(d[0], d[1]);
        u.y = pack_bf16x2(d[2], d[3]);
        u.z = pack_bf16x2(d[4], d[5]);
        u.w = pack_bf16x2(d[6], d[7]);
        *reinterpret_cast<uint4*>(p.x_out + f) = u;
      }
    }
    long long j = vec ? i : a + threadIdx.x;
    const long long jstep = vec ? 1 : blockDim.x;
    for (; j < b; j += jstep) {
      float mq;
      p.x_out[off + j] = __float2bfloat16_rn(momentum_elem(p, g[j] * coef, off + j, &mq));
    }
  }
}

__global__ void __launch_bounds__(512) muon_apply_kernel(MuonApplyParams p) {
  apply_segments(p.upd, p.segs, p.coefs, p.nsegs, blockIdx.x, gridDim.x, p.ema_rate);
}

cudaError_t muon_rs_launch(const MuonRSParams& p, int blocks, cudaStream_t s) {
  if (p.world < 1 || p.world > kMaxPeers || blocks * p.world > kMuonMaxFlags) return cudaErrorInvalidValue;
  muon_rs_kernel<<<blocks, 512, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t muon_momentum_launch(const MuonMomentumParams& p, cudaStream_t s) {
  if (p.n == 0) return cudaSuccess;
  const long long want = (p.n + 255) / 256;
  const int blocks = (int)(want < 148 * 8 ? want : 148 * 8);
  muon_momentum_kernel<<<blocks, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t muon_ag_apply_launch(const MuonAGParams& p, int blocks, cudaStream_t s) {
  if (p.world < 1 || p.world > kMaxPeers || blocks * p.world > kMuonMaxFlags) return cudaErrorInvalidValue;
  muon_ag_apply_kernel<<<blocks, 512, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t muon_seg_momentum_launch(const MuonSegMomentumParams& p, int blocks, cudaStream_t s) {
  if (p.nsegs == 0) return cudaSuccess;
  muon_seg_momentum_kernel<<<blocks, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t muon_apply_launch(const MuonApplyParams& p, int blocks, cudaStream_t s) {
  if (p.nsegs == 0) return cudaSuccess;
  muon_apply_kernel<<<blocks, 512, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace tgo
