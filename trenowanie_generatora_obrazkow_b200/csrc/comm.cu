// Peer-memory collectives over NVLink / NVSwitch: one kernel per GPU, talking to its peers through buffers that
// every rank mapped from every other rank (CUDA IPC), with epoch-numbered flags instead of a host round trip.
//
// allreduce_bf16: the data-parallel gradient average with bf16 transport (what the reference's DDP bf16 compress
// hook does through NCCL, train.py:774-779), fused into one launch:
//   phase 0  cast   : this rank's fp32 gradient chunk -> bf16 staging (local HBM), then flag0[rank][cta] = epoch
//   phase 1  reduce : for its own slice, load the bf16 chunk of every peer's staging over NVLink, sum in fp32,
//                     scale 1 / world, and store the bf16 result into every peer's result buffer (P2P stores),
//                     then flag1[rank][cta] = epoch at every peer
//   phase 2  gather : wait for every peer's flag1, convert the now complete bf16 result chunk back to fp32 grads
// CTA c of every rank owns chunk c of every slice in every phase, so the only synchronisation is per-(peer, CTA)
// flags: no grid-wide barrier and no host involvement. NVLink traffic per rank is 2 (world-1)/world x n x 2 bytes
// (bf16), the minimum for an all-reduce.
// Every flag wait is bounded (globaltimer): on time-out the kernel records ERR_PEER_TIMEOUT in the error word
// and returns, so a missing peer ends the call instead of holding the GPU.
#include "comm.cuh"
#include "kernels.h"

namespace tgo {

__global__ void __launch_bounds__(512) allreduce_bf16_kernel(PeerAllReduceParams p) {
  const int c = blockIdx.x, C = gridDim.x;
  const long long slice = p.slice;                    // elements per rank slice (multiple of 8)
  const long long chunk = ((slice + C - 1) / C + 7) / 8 * 8;
  const long long c0 = (long long)c * chunk;
  const long long c1 = min(slice, c0 + chunk);
  __shared__ int ok_sh;
  if (threadIdx.x == 0) ok_sh = 1;
  const uint64_t deadline = global_ns() + p.timeout_ns;

  // ---- phase 0: cast my fp32 gradients of chunk c of every slice into my bf16 staging ----
  __nv_bfloat16* stage = p.staging[p.rank];
  for (int s = 0; s < p.world; ++s) {
    const long long base = s * slice;
    for (long long i = c0 + threadIdx.x * 8; i < c1; i += (long long)blockDim.x * 8) {
      const long long g = base + i;
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = (g + k < p.n) ? p.grads[g + k] : 0.f;
      uint4 u;
      u.x = pack_bf16x2(v[0], v[1]);
      u.y = pack_bf16x2(v[2], v[3]);
      u.z = pack_bf16x2(v[4], v[5]);
      u.w = pack_bf16x2(v[6], v[7]);
      *reinterpret_cast<uint4*>(stage + g) = u;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    flag_store_release(p.flags[p.rank] + c, p.epoch);  // my staging chunk c is ready (read by every peer)
  }
  // ---- phase 1: reduce my slice, chunk c, from every peer; push the result to every peer ----
  if (threadIdx.x < p.world) {
    if (!flag_wait(p.flags[threadIdx.x] + c, p.epoch, deadline, p.err)) ok_sh = 0;
  }
  __syncthreads();
  if (!ok_sh) return;
  const long long mine = (long long)p.rank * slice;
  for (long long i = c0 + threadIdx.x * 8; i < c1; i += (long long)blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < p.world; ++q) {
      const int peer = (p.rank + q) % p.world;  // start at a different peer on every rank
      const uint4 u = ld_v4_volatile(p.staging[peer] + mine + i);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0] * p.scale, acc[1] * p.scale);
    o.y = pack_bf16x2(acc[2] * p.scale, acc[3] * p.scale);
    o.z = pack_bf16x2(acc[4] * p.scale, acc[5] * p.scale);
    o.w = pack_bf16x2(acc[6] * p.scale, acc[7] * p.scale);
    for (int q = 0; q < p.world; ++q) {
      const int peer = (p.rank + q) % p.world;
      *reinterpret_cast<uint4*>(p.result[peer] + mine + i) = o;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
  __syncthreads();
  if (threadIdx.x < p.world) flag_store_release(p.flags[threadIdx.x] + C + (long long)p.rank * C + c, p.epoch);
  // ---- phase 2: wait for every slice's chunk c, convert to fp32 gradients ----
  if (threadIdx.x < p.world) {
    if (!flag_wait(p.flags[p.rank] + C + (long long)threadIdx.x * C + c, p.epoch, deadline, p.err)) ok_sh = 0;
  }
  __syncthreads();
  if (!ok_sh) return;
  const __nv_bfloat16* res = p.result[p.rank];
  for (int s = 0; s < p.world; ++s) {
    const long long base = s * slice;
    for (long long i = c0 + threadIdx.x * 8; i < c1; i += (long long)blockDim.x * 8) {
      const long long g = base + i;
      const uint4 u = ld_v4_volatile(res + g);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        if (g + 2 * k < p.n) p.grads[g + 2 * k] = f.x;
        if (g + 2 * k + 1 < p.n) p.grads[g + 2 * k + 1] = f.y;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------------------------
// peer_copy: stream a local buffer into another GPU's buffer with NVLink stores (the OPD weight snapshot
// broadcast), then publish `version` in the destination's version word. Completion across CTAs: every CTA adds 1 to
// a local arrival counter after a system fence; the CTA that brings it to version * gridDim.x (the counter is never
// reset, so successive versions need no clearing) writes the version word with a release store.
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) peer_copy_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                                        long long n16, uint32_t* dst_version,
                                                        unsigned long long* counter, uint32_t version) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n16; i += (long long)gridDim.x * blockDim.x)
    dst[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned long long target = (unsigned long long)version * gridDim.x;
    if (atomicAdd(counter, 1ull) + 1 == target) flag_store_release(dst_version, version);
  }
}

cudaError_t peer_copy_launch(void* dst, const void* src, long long nbytes, uint32_t* dst_version,
                             unsigned long long* counter, uint32_t version, int blocks, cudaStream_t s) {
  if (nbytes % 16 != 0 || (reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(src) & 15))
    return cudaErrorInvalidValue;
  peer_copy_kernel<<<blocks, 512, 0, s>>>(reinterpret_cast<uint4*>(dst), reinterpret_cast<const uint4*>(src),
                                          nbytes / 16, dst_version, counter, version);
  return cudaGetLastError();
}

cudaError_t allreduce_bf16_launch(const PeerAllReduceParams& p, int blocks, cudaStream_t s) {
  allreduce_bf16_kernel<<<blocks, 512, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace tgo
