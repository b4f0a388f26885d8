// Persistent warp-specialised bf16 GEMM for sm_100a: TMA -> SMEM ring -> tcgen05.mma (one elected thread) ->
// double-buffered TMEM accumulators -> fused epilogue.
//
//   C[b, m, n] = alpha * sum_k A[b, m, k] * B[b, n, k]  (+ beta * D[b, m, n])      (bf16 or fp32 output)
//
// A and B may each be stored K-major (contraction dim contiguous) or MN-major (output dim contiguous); the
// instruction descriptor's transpose bits select the shared-memory layout, so the same kernel serves
//   forward  y  = x  @ W^T   (A K-major,  B K-major)
//   dgrad    dx = dy @ W     (A K-major,  B MN-major)
//   wgrad    dW = dy^T @ x   (A MN-major, B MN-major)
// and the Newton-Schulz products of the Muon optimizer (X X^T, A A, B X).
//
// Roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer, warps 2-5 = epilogue
// (warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31, i.e. rows of the 128-row tile).
// Replaces the cuBLAS Linear GEMMs (reference aurora/model.py:102-188 under autocast) and the cuBLAS baddbmm of
// the Newton-Schulz step (reference aurora/ns_triton.py:78).
#include <algorithm>

#include "comm.cuh"
#include "kernels.h"

namespace tgo {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;

// EPI_I8: int8 A and B (kind::i8 MMAs, int32 accumulators), bf16 C = acc * alpha * row_scale[m] * col_scale[n]
enum GemmEpi { EPI_BF16 = 0, EPI_F32 = 1, EPI_F32_ACC = 2, EPI_SWIGLU = 3, EPI_I8 = 4 };
enum GemmPeerMode { PEER_NONE = 0, PEER_WAIT_A = 1, PEER_SCATTER_C = 2, GROUPED = 3 };


template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * GEMM_BK * 2;       // 16 or 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int C_STAGE = 4096;  // TMA epilogue: one 32 x 32 staging tile per epilogue warp
  static constexpr int SMEM = STAGES * STAGE_BYTES + 4 * C_STAGE + 1024;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators (256 or 512 columns)
};

// SwiGLU epilogue: the B rows are interleaved in blocks of 128 (gate block k, then up block k), so a 256-column tile
// holds 128 gate and the 128 matching up columns; out[row, n0 / 2 + j] = silu(gate_j) * up_j (bf16), rounded as the
// separate GEMM + SwiGLU kernels round it (bf16 products, bf16 silu).
__device__ __forceinline__ void gemm_store_swiglu(const GemmParams& p, int b, int row, int col0,
                                                  const uint32_t (&gt)[32], const uint32_t (&ut)[32]) {
  if (row >= p.M || col0 >= p.N / 2) return;
  __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)b * p.bsc + (long long)row * p.ldc + col0;
  const bool full = col0 + 32 <= p.N / 2;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (full || col0 + j * 8 < p.N / 2) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float a = __bfloat162float(__float2bfloat16(__uint_as_float(gt[j * 8 + e])));
        const float u = __bfloat162float(__float2bfloat16(__uint_as_float(ut[j * 8 + e])));
        o[e] = __bfloat162float(__float2bfloat16(a / (1.f + __expf(-a)))) * u;
      }
      uint4 w;
      w.x = pack_bf16x2(o[0], o[1]);
      w.y = pack_bf16x2(o[2], o[3]);
      w.z = pack_bf16x2(o[4], o[5]);
      w.w = pack_bf16x2(o[6], o[7]);
      *reinterpret_cast<uint4*>(c + j * 8) = w;
    }
  }
}

// MoE scatter: the bf16 row goes to its source rank's combine buffer (a peer address)
__device__ __forceinline__ void gemm_store_chunk_peer(const GemmParams& p, int b, int row, int col0,
                                                      const uint32_t (&r)[32]) {
  if (row >= p.M || col0 >= p.N) return;
  const int s = row / p.peer.src_rows;
  __nv_bfloat16* c = p.peer.out[s] + ((long long)(p.peer.b_base + b) * p.peer.src_rows + (row - s * p.peer.src_rows)) *
                                         p.ldc + col0;
  const bool full = col0 + 32 <= p.N;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (full || col0 + j * 8 < p.N) {
      uint4 u;
      u.x = pack_bf16x2(__uint_as_float(r[j * 8 + 0]) * p.alpha, __uint_as_float(r[j * 8 + 1]) * p.alpha);
      u.y = pack_bf16x2(__uint_as_float(r[j * 8 + 2]) * p.alpha, __uint_as_float(r[j * 8 + 3]) * p.alpha);
      u.z = pack_bf16x2(__uint_as_float(r[j * 8 + 4]) * p.alpha, __uint_as_float(r[j * 8 + 5]) * p.alpha);
      u.w = pack_bf16x2(__uint_as_float(r[j * 8 + 6]) * p.alpha, __uint_as_float(r[j * 8 + 7]) * p.alpha);
      *reinterpret_cast<uint4*>(c + j * 8) = u;
    }
  }
}

template <int EPI>
__device__ __forceinline__ void gemm_store_chunk(const GemmParams& p, int b, int row, int col0, const uint32_t (&r)[32]) {
  if (row >= p.M || col0 >= p.N) return;
  float v[32];
  const float a = p.row_scale != nullptr ? p.alpha * p.row_scale[row] : p.alpha;
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * a;
  const bool full = col0 + 32 <= p.N;
  if constexpr (EPI == EPI_BF16) {
    if (p.D != nullptr) {
      const __nv_bfloat16* d = p.D + (long long)b * p.bsd + (long long)row * p.ldd + col0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (full || col0 + j * 8 < p.N) {
          uint4 u = *reinterpret_cast<const uint4*>(d + j * 8);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 f = __bfloat1622float2(h[e]);
            v[j * 8 + 2 * e] += p.beta * f.x;
            v[j * 8 + 2 * e + 1] += p.beta * f.y;
          }
        }
      }
    }
    __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)b * p.bsc + (long long)row * p.ldc + col0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (full || col0 + j * 8 < p.N) {
        uint4 u;
        u.x = pack_bf16x2(v[j * 8 + 0], v[j * 8 + 1]);
        u.y = pack_bf16x2(v[j * 8 + 2], v[j * 8 + 3]);
        u.z = pack_bf16x2(v[j * 8 + 4], v[j * 8 + 5]);
        u.w = pack_bf16x2(v[j * 8 + 6], v[j * 8 + 7]);
        *reinterpret_cast<uint4*>(c + j * 8) = u;
      }
    }
  } else {
    float* c = reinterpret_cast<float*>(p.C) + (long long)b * p.bsc + (long long)row * p.ldc + col0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (full || col0 + j * 4 < p.N) {
        float4 o = make_float4(v[j * 4], v[j * 4 + 1], v[j * 4 + 2], v[j * 4 + 3]);
        if constexpr (EPI == EPI_F32_ACC) {
          float4 old = *reinterpret_cast<const float4*>(c + j * 4);
          o.x += old.x;
          o.y += old.y;
          o.z += old.z;
          o.w += old.w;
        }
        *reinterpret_cast<float4*>(c + j * 4) = o;
      }
    }
  }
}

// TMA epilogue of the GEMM kernels: a warp stages its 32 rows x 32 columns in shared memory in the tensor map's
// swizzled layout (bf16: 64-byte rows, 64-byte swizzle; fp32: 128-byte rows, 128-byte swizzle; both conflict-free for
// one 16-byte store per lane and phase), then one lane issues the TMA store (or, for the fp32 accumulate epilogue,
// the TMA reduce-add, so the fp32 gradient bucket is never read by the SM). Per-row global stores from the epilogue
// cost 32 L1 wavefronts per warp instruction on the same data path as the tensor core's shared-memory operand reads.
template <int EPI>
__device__ __forceinline__ void gemm_stage_chunk(const GemmParams& p, int row, uint8_t* buf, int lane,
                                                 const uint32_t (&r)[32]) {
  const float a = (p.row_scale != nullptr && row < p.M) ? p.alpha * p.row_scale[row] : p.alpha;
  if constexpr (EPI == EPI_BF16) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 u;
      u.x = pack_bf16x2(__uint_as_float(r[j * 8 + 0]) * a, __uint_as_float(r[j * 8 + 1]) * a);
      u.y = pack_bf16x2(__uint_as_float(r[j * 8 + 2]) * a, __uint_as_float(r[j * 8 + 3]) * a);
      u.z = pack_bf16x2(__uint_as_float(r[j * 8 + 4]) * a, __uint_as_float(r[j * 8 + 5]) * a);
      u.w = pack_bf16x2(__uint_as_float(r[j * 8 + 6]) * a, __uint_as_float(r[j * 8 + 7]) * a);
      *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = u;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 f;
      f.x = __uint_as_float(r[j * 4 + 0]) * a;
      f.y = __uint_as_float(r[j * 4 + 1]) * a;
      f.z = __uint_as_float(r[j * 4 + 2]) * a;
      f.w = __uint_as_float(r[j * 4 + 3]) * a;
      *reinterpret_cast<float4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) = f;
    }
  }
}
// int8 GEMM: 32 int32 accumulators of one row -> scaled bf16, staged like EPI_BF16 (64-byte swizzled rows)
__device__ __forceinline__ void gemm_stage_chunk_i8(const GemmParams& p, int row, int col0, uint8_t* buf, int lane,
                                                    const uint32_t (&r)[32]) {
  const float a = (p.row_scale != nullptr && row < p.M) ? p.alpha * p.row_scale[row] : p.alpha;
  float f[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float cs = (p.col_scale != nullptr && col0 + j < p.N) ? p.col_scale[col0 + j] : 1.f;
    f[j] = __int2float_rn((int)r[j]) * a * cs;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    u.x = pack_bf16x2(f[j * 8 + 0], f[j * 8 + 1]);
    u.y = pack_bf16x2(f[j * 8 + 2], f[j * 8 + 3]);
    u.z = pack_bf16x2(f[j * 8 + 4], f[j * 8 + 5]);
    u.w = pack_bf16x2(f[j * 8 + 6], f[j * 8 + 7]);
    *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = u;
  }
}
__device__ __forceinline__ void gemm_stage_swiglu(uint8_t* buf, int lane, const uint32_t (&gt)[32],
                                                  const uint32_t (&ut)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float a = __bfloat162float(__float2bfloat16(__uint_as_float(gt[j * 8 + e])));
      const float u = __bfloat162float(__float2bfloat16(__uint_as_float(ut[j * 8 + e])));
      o[e] = __bfloat162float(__float2bfloat16(a / (1.f + __expf(-a)))) * u;
    }
    uint4 w;
    w.x = pack_bf16x2(o[0], o[1]);
    w.y = pack_bf16x2(o[2], o[3]);
    w.z = pack_bf16x2(o[4], o[5]);
    w.w = pack_bf16x2(o[6], o[7]);
    *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = w;
  }
}

// Symmetric-product epilogue helpers (2-CTA kernel, bf16 C): the tile's fp32 values with the beta D term, staged
// as itself or transposed in the 64-byte-swizzled 32 x 32 layout of C's tensor map.
__device__ __forceinline__ void syrk_values(const GemmParams& p, int b, int row, int col0, const uint32_t (&r)[32],
                                            float (&f)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(r[i]) * p.alpha;
  if (p.D != nullptr && row < p.M) {
    const __nv_bfloat16* d = p.D + (long long)b * p.bsd + (long long)row * p.ldd + col0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (col0 + j * 8 < p.N) {
        uint4 u = *reinterpret_cast<const uint4*>(d + j * 8);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 v = __bfloat1622float2(h[e]);
          f[j * 8 + 2 * e] += p.beta * v.x;
          f[j * 8 + 2 * e + 1] += p.beta * v.y;
        }
      }
    }
  }
}
__device__ __forceinline__ void syrk_stage(uint8_t* buf, int lane, const float (&f)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    u.x = pack_bf16x2(f[j * 8 + 0], f[j * 8 + 1]);
    u.y = pack_bf16x2(f[j * 8 + 2], f[j * 8 + 3]);
    u.z = pack_bf16x2(f[j * 8 + 4], f[j * 8 + 5]);
    u.w = pack_bf16x2(f[j * 8 + 6], f[j * 8 + 7]);
    *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = u;
  }
}
// transposed: staged row k = column k of the chunk. Lane pairs exchange one value per two rows, so every lane
// stores 32-bit words: even lanes (T[k][l], T[k][l+1]), odd lanes (T[k+1][l-1], T[k+1][l]); the two rows a store
// instruction covers fill all 32 banks.
__device__ __forceinline__ void syrk_stage_t(uint8_t* buf, int lane, const float (&f)[32]) {
  const bool odd = lane & 1;
  const int col = lane & ~1;
#pragma unroll
  for (int k = 0; k < 32; k += 2) {
    const float recv = __shfl_xor_sync(0xffffffffu, odd ? f[k] : f[k + 1], 1);
    const uint32_t word = odd ? pack_bf16x2(recv, f[k + 1]) : pack_bf16x2(f[k], recv);
    const int trow = odd ? k + 1 : k;
    *reinterpret_cast<uint32_t*>(buf + trow * 64 + (((col >> 3) ^ ((trow >> 1) & 3)) << 4) + ((col * 2) & 15)) = word;
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI, int PEER = PEER_NONE>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = warp_id(), lane = lane_id();
  const int num_m = (p.M + GEMM_BM - 1) / GEMM_BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int tiles_per_batch = num_m * num_n;
  int num_tiles = tiles_per_batch * p.batch;
  const int num_kb = (p.K + GEMM_BK - 1) / GEMM_BK;
  // GROUPED: row-block prefix over the groups (device-side schedule: no host read of the group sizes)
  __shared__ int grp_off[PEER == GROUPED ? kMaxGroups + 1 : 1];
  __shared__ int grp_mb[PEER == GROUPED ? kMaxGroups + 1 : 1];

  if (threadIdx.x == 0) {
    if constexpr (PEER == GROUPED) {
      int acc = 0;
      for (int g = 0; g <= p.batch; ++g) {
        grp_off[g] = p.group_offsets[g];
        grp_mb[g] = acc;
        if (g < p.batch) acc += (p.group_offsets[g + 1] - p.group_offsets[g] + GEMM_BM - 1) / GEMM_BM;
      }
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);  // one arrival per epilogue warp
    }
    abort_sh = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  if constexpr (PEER == GROUPED) num_tiles = grp_mb[p.batch] * num_n;
  // tile -> (batch / group b, first row m0 within it, first column n0, A / C row base, valid rows)
  auto decode = [&](int tile, int& b, int& m0, int& n0, int& row_base, int& rows) {
    if constexpr (PEER == GROUPED) {
      const int mb = tile / num_n;
      n0 = (tile % num_n) * BN;
      int lo = 0, hi = p.batch - 1;  // last group whose first row block is <= mb
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (grp_mb[mid] <= mb) lo = mid; else hi = mid - 1;
      }
      b = lo;
      m0 = (mb - grp_mb[lo]) * GEMM_BM;
      row_base = grp_off[lo];
      rows = grp_off[lo + 1] - grp_off[lo];
    } else {
      b = tile / tiles_per_batch;
      const int r = tile % tiles_per_batch;
      m0 = (r / num_n) * GEMM_BM;
      n0 = (r % num_n) * BN;
      row_base = 0;
      rows = p.M;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t arrived = 0;  // PEER_WAIT_A: bit s = the rows of source s are in place
      for (int tile = blockIdx.x; tile < num_tiles && !abort_sh; tile += gridDim.x) {
        int b, m0, n0, row_base, rows;
        decode(tile, b, m0, n0, row_base, rows);
        (void)rows;
        if constexpr (PEER == PEER_WAIT_A) {
          const int src = m0 / p.peer.src_rows;
          if (!((arrived >> src) & 1u)) {
            if (!flag_wait(p.peer.arrive + src, p.peer.epoch, global_ns() + p.peer.timeout_ns, p.err)) {
              abort_sh = 1;
              break;
            }
            arrived |= 1u << src;
            // the rows were written by another GPU's generic-proxy stores: order them before the TMA reads
            asm volatile("fence.proxy.async.global;" ::: "memory");
          }
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_mode(&empty_bar[stage], phase ^ 1, p.err, ERR_MBAR_TIMEOUT_PRODUCER, (p.poll & 4) != 0)) {
            abort_sh = 1;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          const int k0 = kb * GEMM_BK;
          if constexpr (PEER == GROUPED) {
            tma_load_3d(sa, &tmA, &full_bar[stage], k0, row_base + m0, 0);  // rows past the group: not stored
          } else if constexpr (!A_MN) {
            tma_load_3d(sa, &tmA, &full_bar[stage], k0, m0, b);
          } else {
            tma_load_3d(sa, &tmA, &full_bar[stage], m0, k0, b);
            tma_load_3d(sa + 8192, &tmA, &full_bar[stage], m0 + 64, k0, b);
          }
          if constexpr (!B_MN) {
            tma_load_3d(sb, &tmB, &full_bar[stage], k0, n0, b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_3d(sb + j * 8192, &tmB, &full_bar[stage], n0 + j * 64, k0, b);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // On abort, wait (bounded) until the copies already issued have landed before the CTA can exit.
      if (abort_sh) {
        for (int s = 0; s < STAGES; ++s) mbar_wait(&full_bar[s], 0, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_bf16_f32(GEMM_BM, BN, A_MN, B_MN);
      // descriptors of stage 0; a 16-element k step is 32 B (K-major) or 2 KB (MN-major), in 16-byte units
      const uint64_t a_desc0 = A_MN ? sdesc_sw128(smem_u32(smem), 8192, 1024) : sdesc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t b_desc0 = B_MN ? sdesc_sw128(smem_u32(smem) + Cfg::A_BYTES, 8192, 1024)
                                    : sdesc_sw128(smem_u32(smem) + Cfg::A_BYTES, 16, 1024);
      constexpr uint64_t A_KSTEP = A_MN ? 128 : 2, B_KSTEP = B_MN ? 128 : 2;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !abort_sh; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_mode(&tempty_bar[acc], acc_phase ^ 1, p.err, ERR_MBAR_TIMEOUT_MMA, (p.poll & 1) != 0)) {
          abort_sh = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_mode(&full_bar[stage], phase, p.err, ERR_MBAR_TIMEOUT_MMA, (p.poll & 1) != 0)) {
            abort_sh = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sdesc_add(a_desc0, stage * Cfg::STAGE_BYTES);
          const uint64_t bd = sdesc_add(b_desc0, stage * Cfg::STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k)
            umma_f16(d_tmem, ad + k * A_KSTEP, bd + k * B_KSTEP, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty_bar[stage]);  // frees the stage once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);  // accumulator ready for the epilogue
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int ok = 1;
      if (lane == 0)
        ok = mbar_wait_mode(&tfull_bar[acc], acc_phase, p.err, ERR_MBAR_TIMEOUT_EPILOGUE, (p.poll & 2) != 0) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        abort_sh = 1;
        break;
      }
      __syncwarp();
      tc_fence_after();
      int b, m0, n0, row_base, rows;
      decode(tile, b, m0, n0, row_base, rows);
      const int row = m0 + q * 32 + lane;
      const uint32_t tbase = tmem_base + acc * BN + ((uint32_t)(q * 32) << 16);
      if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t gv[32], uv[32];
          tmem_ld_32x32b_x32(tbase + c * 32, gv);
          tmem_ld_32x32b_x32(tbase + BN / 2 + c * 32, uv);
          tmem_ld_wait();
          gemm_store_swiglu(p, b, row, n0 / 2 + c * 32, gv, uv);
        }
      } else
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + c * 32, v);
        tmem_ld_wait();
        if constexpr (PEER == PEER_SCATTER_C) {
          gemm_store_chunk_peer(p, b, row, n0 + c * 32, v);
        } else if constexpr (PEER == GROUPED) {
          if (row < rows) gemm_store_chunk<EPI>(p, 0, row_base + row, n0 + c * 32, v);
        } else {
          if (p.c_tma != 0) {  // TMA epilogue (see gemm_stage_chunk), one staging tile per warp
            uint8_t* buf = smem + STAGES * Cfg::STAGE_BYTES + q * Cfg::C_STAGE;
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
            gemm_stage_chunk<EPI>(p, row, buf, lane, v);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if constexpr (EPI == EPI_F32_ACC) tma_reduce_add_3d(&tmC, buf, n0 + c * 32, m0 + q * 32, b);
              else tma_store_3d(&tmC, buf, n0 + c * 32, m0 + q * 32, b);
              bulk_commit_group();
            }
          } else {
            gemm_store_chunk<EPI>(p, b, row, n0 + c * 32, v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if constexpr (PEER == PEER_SCATTER_C) {
        // this warp's 32 rows of the tile are stored: count it; the warp completing its source raises the flag
        if (lane == 0) {
          const int src = m0 / p.peer.src_rows;
          __threadfence_system();
          if (atomicAdd(p.peer.done_count + src, 1u) + 1u == p.peer.tile_warps_per_src)
            flag_store_release(p.peer.done_flag[src], p.peer.epoch);
        }
      }
    }
    if (PEER == PEER_NONE && p.c_tma != 0 && lane == 0) bulk_wait_group_all();  // C written before the CTA retires
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}


// ----------------------------------------------------------------------------------------------------------------
// 2-CTA variant: a cluster of two CTAs (one TPC) computes a 256 x 256 tile with tcgen05.mma.cta_group::2.
// CTA r of the pair loads rows [m0 + 128 r, +128) of A and rows [n0 + 128 r, +128) of B into its own shared memory
// (plain TMA loads, completing on the leader CTA's "full" barrier); the leader's single MMA thread issues
// 256 x 256 x 16 MMAs that read both CTAs' tiles; each CTA's TMEM holds its 128 rows x 256 columns.  Per CTA a
// k-block moves 32 KB for 4.2 MFLOP (vs 48 KB for the 1-CTA 128 x 256 tile), which is what keeps L2 -> SM traffic
// below the L2 bandwidth at full tensor rate.
// ----------------------------------------------------------------------------------------------------------------
constexpr int G2_BN = 256;               // N of the pair's tile; each CTA holds 128 columns of B
constexpr int G2_A_BYTES = 128 * 64 * 2; // 16 KB
constexpr int G2_B_BYTES = 128 * 64 * 2; // 16 KB
constexpr int G2_STAGE_BYTES = G2_A_BYTES + G2_B_BYTES;
constexpr int G2_STAGES = 6;
constexpr int G2_C_STAGE = 8192;         // TMA epilogue: per epilogue warp two 32 x 32 staging tiles (<= 4 KB each)
constexpr int G2_SMEM = G2_STAGES * G2_STAGE_BYTES + 4 * G2_C_STAGE + 1024;
constexpr int G2_TMEM_COLS = 512;        // two 256-column accumulators

template <bool A_MN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    gemm_tcgen05_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmC, GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[G2_STAGES];
  __shared__ __align__(8) uint64_t empty_bar[G2_STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
  const int num_m = (p.M + 255) / 256;
  const int num_n = (p.N + G2_BN - 1) / G2_BN;
  const bool syrk = p.syrk != 0;
  const int splits = (EPI == EPI_F32_ACC && p.splitk > 1) ? p.splitk : 1;
  const int tiles_per_batch = (syrk ? num_m * (num_m + 1) / 2 : num_m * num_n) * splits;
  const int num_tiles = tiles_per_batch * p.batch;
  const int num_kb_all = (p.K + GEMM_BK - 1) / GEMM_BK;
  const int kb_per_split = (num_kb_all + splits - 1) / splits;
  // split s of a tile covers k-blocks [s * kb_per_split, min(all, (s + 1) * kb_per_split))
  auto kb_range = [&](int r, int& kb0, int& kb1) {
    const int sp = r / (tiles_per_batch / splits);
    kb0 = sp * kb_per_split;
    kb1 = min(num_kb_all, kb0 + kb_per_split);
  };
  // tile index within a batch -> (row block, column block); symmetric mode: the lower triangle, row by row;
  // split-K: the split index varies slowest
  auto tile_mn = [&](int r, int& mt, int& nt) {
    r %= tiles_per_batch / splits;
    if (syrk) {
      int i = (int)((sqrtf(8.f * (float)r + 1.f) - 1.f) * 0.5f);
      while ((i + 1) * (i + 2) / 2 <= r) ++i;
      while (i * (i + 1) / 2 > r) --i;
      mt = i;
      nt = r - i * (i + 1) / 2;
    } else {
      mt = r / num_n;
      nt = r % num_n;
    }
  };

  // Tail split: the last p.tail_tiles tiles run as two 256 x 128 units each (half = 0 / 1), so a last wave that would
  // keep at most half of the pairs busy for a whole tile takes about half a tile's time. Units are dealt out
  // round-robin like the tiles; -1 marks a whole tile.
  const int n_whole = num_tiles - p.tail_tiles;
  const int num_units = num_tiles + p.tail_tiles;
  auto unit_tile = [&](int u, int& tile, int& half) {
    if (u < n_whole) {
      tile = u;
      half = -1;
    } else {
      tile = n_whole + (u - n_whole) / 2;
      half = (u - n_whole) & 1;
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < G2_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // leader only: one arrive.expect_tx for both CTAs' bytes
      mbar_init(&empty_bar[s], 1);  // both: the leader's multicast commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);  // both: the leader's multicast commit
      mbar_init(&tempty_bar[a], 8); // leader only: 4 epilogue warps x 2 CTAs
    }
    abort_sh = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_base_sh, G2_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // peer barriers initialised and TMEM allocated before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      for (int u = cluster; u < num_units && !abort_sh; u += n_clusters) {
        int tile, half;
        unit_tile(u, tile, half);
        const int b = tile / tiles_per_batch;
        int mt, nt, kb0, kb1;
        tile_mn(tile % tiles_per_batch, mt, nt);
        kb_range(tile % tiles_per_batch, kb0, kb1);
        // a half unit's CTA holds 64 columns of B: the 128-row box starting there brings 64 unused rows along
        const int m0 = mt * 256 + rank * 128;
        const int n0 = half < 0 ? nt * G2_BN + rank * 128 : nt * G2_BN + half * 128 + rank * 64;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_mode(&empty_bar[stage], phase ^ 1, p.err, ERR_MBAR_TIMEOUT_PRODUCER, (p.poll & 4) != 0)) {
            abort_sh = 1;
            break;
          }
          uint8_t* sa = smem + stage * G2_STAGE_BYTES;
          uint8_t* sb = sa + G2_A_BYTES;
          if (leader) mbar_expect_tx(&full_bar[stage], 2 * G2_STAGE_BYTES);
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
          const int k0 = kb * GEMM_BK;
          if constexpr (!A_MN) {
            tma_load_3d_pair(sa, &tmA, fb, k0, m0, b);
          } else {
            tma_load_3d_pair(sa, &tmA, fb, m0, k0, b);
            tma_load_3d_pair(sa + 8192, &tmA, fb, m0 + 64, k0, b);
          }
          if constexpr (!B_MN) {
            tma_load_3d_pair(sb, &tmB, fb, k0, n0, b);
          } else {
            tma_load_3d_pair(sb, &tmB, fb, n0, k0, b);
            tma_load_3d_pair(sb + 8192, &tmB, fb, n0 + 64, k0, b);
          }
          if (++stage == G2_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader CTA only) ----------------
      constexpr uint32_t idesc = EPI == EPI_I8 ? idesc_s8_s32(256, G2_BN) : idesc_bf16_f32(256, G2_BN, A_MN, B_MN);
      const uint64_t a_desc0 = A_MN ? sdesc_sw128(smem_u32(smem), 8192, 1024) : sdesc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t b_desc0 = B_MN ? sdesc_sw128(smem_u32(smem) + G2_A_BYTES, 8192, 1024)
                                    : sdesc_sw128(smem_u32(smem) + G2_A_BYTES, 16, 1024);
      constexpr uint64_t A_KSTEP = A_MN ? 128 : 2, B_KSTEP = B_MN ? 128 : 2;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      constexpr uint32_t idesc_half = EPI == EPI_I8 ? idesc_s8_s32(256, G2_BN / 2)
                                                     : idesc_bf16_f32(256, G2_BN / 2, A_MN, B_MN);
      for (int u = cluster; u < num_units && !abort_sh; u += n_clusters, ++local) {
        int tile, half;
        unit_tile(u, tile, half);
        const uint32_t id = half < 0 ? idesc : idesc_half;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_mode(&tempty_bar[acc], acc_phase ^ 1, p.err, ERR_MBAR_TIMEOUT_MMA, (p.poll & 1) != 0)) {
          abort_sh = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * G2_BN;
        bool ok = true;
        int kb0, kb1;
        kb_range(tile % tiles_per_batch, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_mode(&full_bar[stage], phase, p.err, ERR_MBAR_TIMEOUT_MMA, (p.poll & 1) != 0)) {
            abort_sh = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sdesc_add(a_desc0, stage * G2_STAGE_BYTES);
          const uint64_t bd = sdesc_add(b_desc0, stage * G2_STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            if constexpr (EPI == EPI_I8)
              umma_i8_pair(d_tmem, ad + k * A_KSTEP, bd + k * B_KSTEP, id, (kb != kb0 || k != 0) ? 1u : 0u);
            else
              umma_f16_pair(d_tmem, ad + k * A_KSTEP, bd + k * B_KSTEP, id, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit_pair_mc(&empty_bar[stage], 0x3);  // frees this stage in both CTAs
          if (++stage == G2_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(&tfull_bar[acc], 0x3);  // both CTAs' accumulators ready
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    const int q = warp & 3;
    const bool tma_c = p.c_tma != 0;
    uint8_t* const cstage = smem + G2_STAGES * G2_STAGE_BYTES + q * G2_C_STAGE;
    int cbuf = 0;
    // stage one 32 x 32 chunk and hand it to the TMA unit (the buffer's previous store must have read it)
    auto tma_chunk = [&](auto&& fill, int x, int y, int z) {
      uint8_t* buf = cstage + (cbuf & 1) * (G2_C_STAGE / 2);
      if (lane == 0) bulk_wait_group_read<1>();
      __syncwarp();
      fill(buf);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if constexpr (EPI == EPI_F32_ACC) tma_reduce_add_3d(&tmC, buf, x, y, z);
        else tma_store_3d(&tmC, buf, x, y, z);
        bulk_commit_group();
      }
      ++cbuf;
    };
    int local = 0;
    for (int u = cluster; u < num_units; u += n_clusters, ++local) {
      int tile, half;
      unit_tile(u, tile, half);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int ok = 1;
      if (lane == 0)
        ok = mbar_wait_mode(&tfull_bar[acc], acc_phase, p.err, ERR_MBAR_TIMEOUT_EPILOGUE, (p.poll & 2) != 0) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        abort_sh = 1;
        break;
      }
      __syncwarp();
      tc_fence_after();
      const int b = tile / tiles_per_batch;
      int mt, nt;
      tile_mn(tile % tiles_per_batch, mt, nt);
      const int m0 = mt * 256 + rank * 128, n0 = nt * G2_BN + (half < 0 ? 0 : half * 128);
      const int n_chunks = half < 0 ? G2_BN / 32 : G2_BN / 64;  // 32-column chunks of this unit
      const int row = m0 + q * 32 + lane;
      const uint32_t tbase = tmem_base + acc * G2_BN + ((uint32_t)(q * 32) << 16);
      if constexpr (EPI == EPI_BF16) {
        if (syrk) {  // the tile, and its mirror image above the diagonal
#pragma unroll 1
          for (int c = 0; c < G2_BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tbase + c * 32, v);
            tmem_ld_wait();
            float f[32];
            syrk_values(p, b, row, n0 + c * 32, v, f);
            tma_chunk([&](uint8_t* buf) { syrk_stage(buf, lane, f); }, n0 + c * 32, m0 + q * 32, b);
            if (mt != nt) tma_chunk([&](uint8_t* buf) { syrk_stage_t(buf, lane, f); }, m0 + q * 32, n0 + c * 32, b);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[acc]), 0));
          continue;
        }
      }
      if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < G2_BN / 64; ++c) {
          uint32_t gv[32], uv[32];
          tmem_ld_32x32b_x32(tbase + c * 32, gv);
          tmem_ld_32x32b_x32(tbase + G2_BN / 2 + c * 32, uv);
          tmem_ld_wait();
          if (tma_c)
            tma_chunk([&](uint8_t* buf) { gemm_stage_swiglu(buf, lane, gv, uv); }, n0 / 2 + c * 32, m0 + q * 32, b);
          else
            gemm_store_swiglu(p, b, row, n0 / 2 + c * 32, gv, uv);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < n_chunks; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tbase + c * 32, v);
          tmem_ld_wait();
          if constexpr (EPI == EPI_I8) {  // TMA epilogue only (the launcher requires C's tensor map)
            tma_chunk([&](uint8_t* buf) { gemm_stage_chunk_i8(p, row, n0 + c * 32, buf, lane, v); }, n0 + c * 32,
                      m0 + q * 32, b);
          } else if (tma_c) {
            tma_chunk([&](uint8_t* buf) { gemm_stage_chunk<EPI>(p, row, buf, lane, v); }, n0 + c * 32, m0 + q * 32, b);
          } else {
            gemm_store_chunk<EPI>(p, b, row, n0 + c * 32, v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[acc]), 0));
    }
    if (tma_c && lane == 0) bulk_wait_group_all();  // C written before the CTA retires
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA frees TMEM or exits while the pair still has MMAs / remote arrivals in flight
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, G2_TMEM_COLS);
  }
}

// ----------------------------------------------------------------------------------------------------------------
// Launch (tensor maps are encoded by the host wrapper in ops.cpp)
// ----------------------------------------------------------------------------------------------------------------
int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

static int g_gemm_poll = 0;
// Off by default: measured slower (8192 x 2048 x 2048 0.196 -> 0.235 ms, x 5504 0.506 -> 0.563 ms, qkv 0.576 ->
// 0.656 ms): a half unit still loads a full 128-row B box per CTA and all of A, so the last wave is bound by L2 -> SM
// traffic rather than by the tensor core, and takes about as long as a wave of whole tiles.
static bool g_gemm_tail = false;
cudaError_t gemm_set_tail_split(int on) {
  g_gemm_tail = on != 0;
  return cudaSuccess;
}
cudaError_t gemm_set_poll(int mask) {
  if (mask < 0 || mask > 7) return cudaErrorInvalidValue;
  g_gemm_poll = mask;
  return cudaSuccess;
}
static GemmParams with_poll(const GemmParams& p) {
  GemmParams q = p;
  q.poll = g_gemm_poll;
  return q;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
static cudaError_t launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t stream,
                               const CUtensorMap* tc = nullptr) {
  using Cfg = GemmCfg<BN>;
  static_assert(Cfg::SMEM + 1024 <= 232448, "GEMM: dynamic + static shared memory");
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    attr_set = true;
  }
  const int num_tiles = ((p.M + GEMM_BM - 1) / GEMM_BM) * ((p.N + BN - 1) / BN) * p.batch;
  const int grid = std::max(1, std::min(num_tiles, num_sms()));
  kern<<<grid, GEMM_THREADS, Cfg::SMEM, stream>>>(ta, tb, tc != nullptr ? *tc : ta, with_poll(p));
  return cudaGetLastError();
}

template <int BN, int EPI>
static cudaError_t dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                                  const GemmParams& p, cudaStream_t s,
                                   const CUtensorMap* tc) {
  if (!a_mn && !b_mn) return launch_gemm<BN, false, false, EPI>(ta, tb, p, s, tc);
  if (!a_mn && b_mn) return launch_gemm<BN, false, true, EPI>(ta, tb, p, s, tc);
  if (a_mn && !b_mn) return launch_gemm<BN, true, false, EPI>(ta, tb, p, s, tc);
  return launch_gemm<BN, true, true, EPI>(ta, tb, p, s, tc);
}

template <bool A_MN, bool B_MN, int EPI>
static cudaError_t launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                                    cudaStream_t stream, const CUtensorMap* tc) {
  static_assert(G2_SMEM + 1024 <= 232448, "2-CTA GEMM: dynamic + static shared memory");
  auto kern = gemm_tcgen05_pair_kernel<A_MN, B_MN, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G2_SMEM);
    attr_set = true;
  }
  const int nm = (p.M + 255) / 256;
  const int splits = (EPI == EPI_F32_ACC && p.splitk > 1) ? p.splitk : 1;
  const int num_tiles = (p.syrk ? nm * (nm + 1) / 2 : nm * ((p.N + G2_BN - 1) / G2_BN)) * p.batch * splits;
  const int pairs = num_sms() / 2;
  // tail split: when the tiles of the last wave would occupy at most half of the pairs, they run as half-width units
  GemmParams q = with_poll(p);
  q.tail_tiles = 0;
  if (g_gemm_tail && !p.syrk && splits == 1 && EPI != EPI_SWIGLU) {
    const int left = num_tiles % pairs;
    if (left > 0 && 2 * left <= pairs) q.tail_tiles = left;
  }
  const int units = num_tiles + q.tail_tiles;
  const int grid = std::max(2, std::min(2 * units, pairs * 2));
  kern<<<grid, GEMM_THREADS, G2_SMEM, stream>>>(ta, tb, tc != nullptr ? *tc : ta, q);
  return cudaGetLastError();
}

template <int EPI>
static cudaError_t dispatch_pair(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                                 const GemmParams& p, cudaStream_t s,
                                  const CUtensorMap* tc) {
  if (!a_mn && !b_mn) return launch_gemm_pair<false, false, EPI>(ta, tb, p, s, tc);
  if (!a_mn && b_mn) return launch_gemm_pair<false, true, EPI>(ta, tb, p, s, tc);
  if (a_mn && !b_mn) return launch_gemm_pair<true, false, EPI>(ta, tb, p, s, tc);
  return launch_gemm_pair<true, true, EPI>(ta, tb, p, s, tc);
}

template <bool B_MN, int PEER>
static cudaError_t launch_gemm_peer(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                                   cudaStream_t s) {
  using Cfg = GemmCfg<256>;
  auto kern = gemm_tcgen05_kernel<256, false, B_MN, EPI_BF16, PEER>;
  static bool set = false;
  if (!set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    set = true;
  }
  const int tiles = ((p.M + GEMM_BM - 1) / GEMM_BM) * ((p.N + 255) / 256) * p.batch;
  kern<<<std::min(tiles, num_sms()), GEMM_THREADS, Cfg::SMEM, s>>>(ta, tb, ta, with_poll(p));
  return cudaGetLastError();
}

cudaError_t gemm_grouped_launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, bool b_mn,
                                cudaStream_t s) {
  if (p.batch < 1 || p.batch > kMaxGroups || p.group_offsets == nullptr) return cudaErrorInvalidValue;
  using Cfg = GemmCfg<256>;
  auto kern = b_mn ? gemm_tcgen05_kernel<256, false, true, EPI_BF16, GROUPED>
                   : gemm_tcgen05_kernel<256, false, false, EPI_BF16, GROUPED>;
  static bool set[2] = {false, false};
  if (!set[b_mn]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    set[b_mn] = true;
  }
  // the tile count is known on the device only: a persistent grid, bounded by the worst case
  const long long worst = ((long long)(p.M + GEMM_BM - 1) / GEMM_BM + p.batch) * ((p.N + 255) / 256);
  const int grid = (int)std::max(1LL, std::min<long long>(worst, num_sms()));
  kern<<<grid, GEMM_THREADS, Cfg::SMEM, s>>>(ta, tb, ta, with_poll(p));
  return cudaGetLastError();
}

cudaError_t gemm_peer_launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, bool b_mn,
                             int peer_mode, cudaStream_t s) {
  if (p.peer.src_rows <= 0 || p.peer.src_rows % GEMM_BM != 0 || p.M % p.peer.src_rows != 0 ||
      p.M / p.peer.src_rows > kMaxPeers)
    return cudaErrorInvalidValue;
  if (peer_mode == PEER_WAIT_A) {
    if (p.peer.arrive == nullptr) return cudaErrorInvalidValue;
    return b_mn ? launch_gemm_peer<true, PEER_WAIT_A>(ta, tb, p, s) : launch_gemm_peer<false, PEER_WAIT_A>(ta, tb, p, s);
  }
  if (peer_mode == PEER_SCATTER_C) {
    if (p.peer.done_count == nullptr) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(p.peer.done_count, 0, sizeof(unsigned) * (p.M / p.peer.src_rows), s);
    if (e != cudaSuccess) return e;
    return b_mn ? launch_gemm_peer<true, PEER_SCATTER_C>(ta, tb, p, s)
                : launch_gemm_peer<false, PEER_SCATTER_C>(ta, tb, p, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int bn, bool a_mn,
                        bool b_mn, int epi, cudaStream_t s, const CUtensorMap* tc) {
  if (p.c_tma != 0 && tc == nullptr) return cudaErrorInvalidValue;  // TMA epilogue needs C's tensor map
  if (p.syrk != 0 && (bn != 0 || epi != EPI_BF16 || p.c_tma == 0 || p.M != p.N)) return cudaErrorInvalidValue;
  // split-K partial tiles must reduce-add (atomic in L2): 2-CTA kernel, fp32 accumulate through the tensor map
  if (p.splitk > 1 && (bn != 0 || epi != EPI_F32_ACC || p.c_tma == 0 || p.syrk != 0)) return cudaErrorInvalidValue;
  if (epi == EPI_I8) {  // int8 A [M, K] and B [N, K], both K-major; 2-CTA kernel with the TMA epilogue
    if (a_mn || b_mn || bn != 0 || p.c_tma == 0 || p.syrk != 0 || p.splitk > 1) return cudaErrorInvalidValue;
    return launch_gemm_pair<false, false, EPI_I8>(ta, tb, p, s, tc);
  }
  if (epi == EPI_SWIGLU) {  // forward only (A and B K-major), 256-column tiles
    if (a_mn || b_mn || (bn != 0 && bn != 256) || p.N % 256 != 0) return cudaErrorInvalidValue;
    return bn == 0 ? launch_gemm_pair<false, false, EPI_SWIGLU>(ta, tb, p, s, tc)
                   : launch_gemm<256, false, false, EPI_SWIGLU>(ta, tb, p, s);  // row stores (c_tma unused)
  }
  if (bn == 0) {  // 2-CTA kernel (tensor maps built with 128-row / 64-row boxes per CTA)
    if (epi == EPI_BF16) return dispatch_pair<EPI_BF16>(a_mn, b_mn, ta, tb, p, s, tc);
    if (epi == EPI_F32) return dispatch_pair<EPI_F32>(a_mn, b_mn, ta, tb, p, s, tc);
    return dispatch_pair<EPI_F32_ACC>(a_mn, b_mn, ta, tb, p, s, tc);
  }
  if (bn == 128) {
    if (epi == EPI_BF16) return dispatch_major<128, EPI_BF16>(a_mn, b_mn, ta, tb, p, s, tc);
    if (epi == EPI_F32) return dispatch_major<128, EPI_F32>(a_mn, b_mn, ta, tb, p, s, tc);
    return dispatch_major<128, EPI_F32_ACC>(a_mn, b_mn, ta, tb, p, s, tc);
  }
  if (epi == EPI_BF16) return dispatch_major<256, EPI_BF16>(a_mn, b_mn, ta, tb, p, s, tc);
  if (epi == EPI_F32) return dispatch_major<256, EPI_F32>(a_mn, b_mn, ta, tb, p, s, tc);
  return dispatch_major<256, EPI_F32_ACC>(a_mn, b_mn, ta, tb, p, s, tc);
}

}  // namespace tgo
