// Expert-parallel MoE exchange over NVLink peer memory: the dispatch side of the all-to-all fused with the token
// gather, the combine side fused with the routing-weighted sum. The expert GEMMs in between (gemm.cu, peer modes)
// wait for the dispatched rows tile by tile and store their outputs straight into the sources' combine buffers.
//
//   dispatch (source rank):  for every slot (expert e, position i < C) of this rank: row = x[src_tok] (* scale), or
//                            zeros for an empty slot, stored into owner r = e / local at
//                            recv_r[((e % local) * world + rank) * C + i]; the CTA that finishes the owner's rows
//                            sets arrive_r[rank] = epoch (release, system scope)
//   combine (source rank):   out[t] = sum_k w[t, k] * ybuf[slot[t, k]] once every owner's done flag shows epoch
//   release (owner rank):    free_s[rank] = epoch on every source s: the receive rows may be overwritten
//
// Before writing into an owner's receive buffer the dispatch waits until that owner released the previous
// epoch's rows (its backward pass still reads them for the expert weight gradient). All waits are bounded: a
// time-out records ERR_PEER_TIMEOUT and the kernel returns.
#include <algorithm>

#include "comm.cuh"
#include "kernels.h"

namespace tgo {

namespace {

__device__ __forceinline__ uint4 scale_row8(uint4 u, float s) {
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float2 f = __bfloat1622float2(h[e]);
    h[e] = __floats2bfloat162_rn(f.x * s, f.y * s);
  }
  return u;
}

}  // namespace

// grid (blocks_per_owner, world): blockIdx.y = owner rank; warps copy rows of D bf16 with 16-byte stores
__global__ void __launch_bounds__(256) moe_dispatch_kernel(MoEDispatchParams p) {
  const int owner = blockIdx.y;
  __shared__ int ok_sh;
  if (threadIdx.x == 0) {  // back-pressure (forward dispatch only): the owner released the previous epoch's rows
    const uint64_t deadline = global_ns() + p.timeout_ns;
    ok_sh = (p.free_flags == nullptr || flag_wait(p.free_flags + owner, p.epoch - 1, deadline, p.err)) ? 1 : 0;
  }
  __syncthreads();
  if (!ok_sh) return;
  const int rows = p.local * p.C;  // this rank's rows for the owner's experts
  const int vec = p.D / 8;         // 16-byte chunks per row
  const int warps = blockDim.x / 32, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __nv_bfloat16* dst_base = p.recv[owner];
  for (int i = blockIdx.x * warps + warp; i < rows; i += gridDim.x * warps) {
    const int j = i / p.C, pos = i - j * p.C;
    const int slot = (owner * p.local + j) * p.C + pos;
    const int t = p.src_tok[slot];
    const float sc = (p.scale != nullptr && t >= 0) ? p.scale[slot] : 1.f;
    const uint4* src = reinterpret_cast<const uint4*>(p.x + (long long)(t < 0 ? 0 : t) * p.D);
    uint4* dst = reinterpret_cast<uint4*>(dst_base + ((long long)(j * p.world + p.rank) * p.C + pos) * p.D);
    for (int c = lane; c < vec; c += 32) {
      uint4 u = make_uint4(0u, 0u, 0u, 0u);
      if (t >= 0) {
        u = src[c];
        if (p.scale != nullptr) u = scale_row8(u, sc);
      }
      dst[c] = u;  // NVLink store into the owner's memory (or a local store for the own experts)
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // every thread's row stores (ordered by the barrier) before the count
    if (atomicAdd(p.counter + owner, 1u) + 1u == gridDim.x) flag_store_release(p.arrive[owner] + p.rank, p.epoch);
  }
}

// one warp per token; the block's first thread waits for every owner's done flag
__global__ void __launch_bounds__(256) moe_combine_kernel(MoECombineParams p) {
  __shared__ int ok_sh;
  if (threadIdx.x == 0) {
    const uint64_t deadline = global_ns() + p.timeout_ns;
    int ok = 1;
    for (int r = 0; r < p.world && ok; ++r) ok = flag_wait(p.done + r, p.epoch, deadline, p.err) ? 1 : 0;
    ok_sh = ok;
  }
  __syncthreads();
  if (!ok_sh) return;
  const int vec = p.D / 8;
  const int warps = blockDim.x / 32, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int t = blockIdx.x * warps + warp; t < p.N; t += gridDim.x * warps) {
    int sl[4];
    float wk[4];
    for (int k = 0; k < p.k && k < 4; ++k) {
      sl[k] = p.slot[(long long)t * p.k + k];
      wk[k] = (p.w != nullptr) ? p.w[(long long)t * p.k + k] : 1.f;
    }
    uint4* out = reinterpret_cast<uint4*>(p.out + (long long)t * p.D);
    for (int c = lane; c < vec; c += 32) {
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      for (int k = 0; k < p.k && k < 4; ++k) {
        if (sl[k] < 0) continue;
        // written by other GPUs: read through L2 (the peers' stores land there), not a possibly stale L1 line
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p.ybuf + (long long)sl[k] * p.D) + c);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[2 * e] += wk[k] * f.x;
          acc[2 * e + 1] += wk[k] * f.y;
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      out[c] = o;
    }
  }
}

struct FreePeers {
  uint32_t* f[kMaxPeers];
};

__global__ void moe_release_kernel(FreePeers fp, int rank, int world, uint32_t epoch) {
  if (threadIdx.x < world) flag_store_release(fp.f[threadIdx.x] + rank, epoch);
}

cudaError_t moe_dispatch_launch(const MoEDispatchParams& p, int blocks_per_owner, cudaStream_t s) {
  if (p.world < 1 || p.world > kMaxPeers || p.D % 8 != 0 || p.C <= 0 || p.E != p.local * p.world)
    return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(p.counter, 0, sizeof(unsigned) * p.world, s);
  if (e != cudaSuccess) return e;
  moe_dispatch_kernel<<<dim3(blocks_per_owner, p.world), 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t moe_combine_launch(const MoECombineParams& p, cudaStream_t s) {
  if (p.k < 1 || p.k > 4 || p.D % 8 != 0 || p.world < 1 || p.world > kMaxPeers) return cudaErrorInvalidValue;
  const int blocks = std::max(1, std::min((p.N + 7) / 8, num_sms() * 8));
  moe_combine_kernel<<<blocks, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t moe_release_launch(uint32_t* const* free_peer, int rank, int world, uint32_t epoch, cudaStream_t s) {
  if (world < 1 || world > kMaxPeers) return cudaErrorInvalidValue;
  FreePeers fp{};
  for (int r = 0; r < world; ++r) fp.f[r] = free_peer[r];
  moe_release_kernel<<<1, 32, 0, s>>>(fp, rank, world, epoch);
  return cudaGetLastError();
}

}  // namespace tgo
