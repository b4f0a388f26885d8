// Flash attention forward / backward (bf16 in, fp32 softmax and accumulation), head dims 64 and 128.
//
//   O[b, t, h] = softmax(scale * Q[b, t, h] K[b, :, h / rep]^T  masked to keys < kv_len[b]) V[b, :, h / rep]
//
// Tensors are addressed as [batch][token][head][head_dim] with arbitrary (16-byte aligned) batch / token / head
// strides, so the kernels read q / k / v straight out of the fused qkv GEMM output and write O in the row layout
// the output projection consumes.  rep = Hq / Hkv gives grouped-query attention without repeating k / v.
// A key mask given as per-batch valid lengths covers the cross-attention key-padding mask and the text refiner's
// mask (captions are right-padded, reference aurora/model.py:121-132, :180-188).
//
// Replaces torch SDPA (reference aurora/model.py:16-21, :165, :187).  Tensor-core path: mma.sync m16n8k16 with
// ldmatrix from XOR-swizzled shared memory, cp.async double buffering.
#include "common.cuh"
#include "kernels.h"

namespace tgo {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------------------------------------------------------
// small PTX helpers
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void red_add_v2(float* addr, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b) : "memory");
}

// Tile of R rows x HD bf16 in shared memory; 16-byte chunk c of row r lives at chunk (c ^ (r & 7)).
template <int HD>
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  return (uint32_t)(row * (HD * 2) + ((chunk ^ (row & 7)) << 4));
}

// Copy rows [row0, row0 + R) of a [token][head_dim] matrix (token stride ld elements) into a swizzled tile;
// rows >= nrows are zero-filled.
template <int R, int HD, int NT>
__device__ __forceinline__ void load_tile(uint32_t smem, const bf16* g, long long ld, int row0, int nrows) {
  constexpr int CH = HD / 8;
  for (int i = threadIdx.x; i < R * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const bool ok = row0 + r < nrows;
    const bf16* src = g + (long long)(ok ? row0 + r : 0) * ld + c * 8;
    cp_async16(smem + tile_off<HD>(r, c), src, ok);
  }
}

// ------------------------------------------------------------------------------------------------------------------
// forward: CTA = 128 queries of one (batch, head), 8 warps x 16 rows; key tiles of 64, double buffered
// ------------------------------------------------------------------------------------------------------------------
constexpr int FA_BM = 128;
constexpr int FA_BN = 64;
constexpr int FA_FWD_THREADS = 256;

template <int HD>
__global__ void __launch_bounds__(FA_FWD_THREADS, 1) flash_fwd_kernel(AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + FA_BM * HD * 2;
  const uint32_t sV = sK + 2 * FA_BN * HD * 2;
  constexpr int KT = HD / 16;  // k-steps over the head dim
  constexpr int NO = HD / 8;   // n-tiles of the output

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.rep;
  const int warp = warp_id(), lane = lane_id();
  const int q0 = qb * FA_BM;
  int kv_end = p.Tk;
  if (p.kv_len != nullptr) kv_end = min(kv_end, p.kv_len[b]);

  const bf16* Qg = p.q + (long long)b * p.q_bs + (long long)h * p.q_hs;
  const bf16* Kg = p.k + (long long)b * p.k_bs + (long long)hk * p.k_hs;
  const bf16* Vg = p.v + (long long)b * p.v_bs + (long long)hk * p.v_hs;

  load_tile<FA_BM, HD, FA_FWD_THREADS>(sQ, Qg + (long long)q0 * p.q_ts, p.q_ts, 0, p.Tq - q0);
  const int n_tiles = (kv_end + FA_BN - 1) / FA_BN;
  if (n_tiles > 0) {
    load_tile<FA_BN, HD, FA_FWD_THREADS>(sK, Kg, p.k_ts, 0, kv_end);
    load_tile<FA_BN, HD, FA_FWD_THREADS>(sV, Vg, p.v_ts, 0, kv_end);
  }
  cp_async_commit();

  float o[NO][4];
#pragma unroll
  for (int i = 0; i < NO; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const float sl2 = p.scale * 1.4426950408889634f;  // scale * log2(e)
  uint32_t qf[KT][4];

  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_tiles) {
      const int nb = buf ^ 1;
      load_tile<FA_BN, HD, FA_FWD_THREADS>(sK + nb * FA_BN * HD * 2, Kg + (long long)(j + 1) * FA_BN * p.k_ts, p.k_ts,
                                           0, kv_end - (j + 1) * FA_BN);
      load_tile<FA_BN, HD, FA_FWD_THREADS>(sV + nb * FA_BN * HD * 2, Vg + (long long)(j + 1) * FA_BN * p.v_ts, p.v_ts,
                                           0, kv_end - (j + 1) * FA_BN);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = kk * 2 + (lane >> 4);
        ldsm_x4(sQ + tile_off<HD>(row, ch), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const uint32_t k_s = sK + buf * FA_BN * HD * 2, v_s = sV + buf * FA_BN * HD * 2;
    // S = Q K^T : 16 x 64 per warp
    float s[FA_BN / 8][4];
#pragma unroll
    for (int n = 0; n < FA_BN / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KT; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < FA_BN / 16; ++n2) {
        uint32_t b0, b1, b2, b3;
        const int row = n2 * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int ch = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(k_s + tile_off<HD>(row, ch), b0, b1, b2, b3);
        mma16816(s[2 * n2], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816(s[2 * n2 + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    // mask + online softmax (rows g and g + 8 of this warp's 16)
    const int kbase = j * FA_BN;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int n = 0; n < FA_BN / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kbase + n * 8 + (lane & 3) * 2 + (e & 1);
        float v = s[n][e] * sl2;
        if (key >= kv_end) v = -INFINITY;
        s[n][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      corr[r] = (m_r[r] == -INFINITY) ? 0.f : exp2f(m_r[r] - mx[r]);
      m_r[r] = mx[r];
    }
    uint32_t pf[FA_BN / 8][2];
#pragma unroll
    for (int n = 0; n < FA_BN / 8; ++n) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        pv[e] = (mm == -INFINITY) ? 0.f : exp2f(s[n][e] - mm);
      }
      // round P to bf16 once; the row sums use the rounded values (what the P V product sees)
      pf[n][0] = pack_bf16x2(pv[0], pv[1]);
      pf[n][1] = pack_bf16x2(pv[2], pv[3]);
      const __nv_bfloat162* h0 = reinterpret_cast<const __nv_bfloat162*>(&pf[n][0]);
      const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&pf[n][1]);
      const float2 f0 = __bfloat1622float2(*h0), f1 = __bfloat1622float2(*h1);
      rs[0] += f0.x + f0.y;
      rs[1] += f1.x + f1.y;
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_r[r] = l_r[r] * corr[r] + rs[r];
    }
#pragma unroll
    for (int i = 0; i < NO; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < FA_BN / 16; ++kk) {
      const uint32_t a0 = pf[2 * kk][0], a1 = pf[2 * kk][1], a2 = pf[2 * kk + 1][0], a3 = pf[2 * kk + 1][1];
#pragma unroll
      for (int n2 = 0; n2 < HD / 16; ++n2) {
        uint32_t b0, b1, b2, b3;
        const int row = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int ch = n2 * 2 + (lane >> 4);
        ldsm_x4_t(v_s + tile_off<HD>(row, ch), b0, b1, b2, b3);
        mma16816(o[2 * n2], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * n2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // this buffer is refilled two iterations later
  }
  // epilogue
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int t = q0 + warp * 16 + g + r * 8;
    if (t >= p.Tq) continue;
    const float inv = l_r[r] > 0.f ? 1.f / l_r[r] : 0.f;
    bf16* dst = p.o + (long long)b * p.o_bs + (long long)t * p.o_ts + (long long)h * p.o_hs + c * 2;
#pragma unroll
    for (int i = 0; i < NO; ++i)
      *reinterpret_cast<__nv_bfloat162*>(dst + i * 8) = __floats2bfloat162_rn(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
    if (c == 0 && p.lse != nullptr) {
      const float lse = l_r[r] > 0.f ? (m_r[r] + log2f(l_r[r])) * 0.6931471805599453f : INFINITY;
      p.lse[((long long)b * p.Hq + h) * p.Tq + t] = lse;
    }
  }
}

// ------------------------------------------------------------------------------------------------------------------
// backward preprocessing: delta[b, h, t] = sum_d dO * O
// ------------------------------------------------------------------------------------------------------------------
// HD / 8 lanes per (b, t, h) row, 16-byte loads, four rows per thread in flight (grid-stride), shuffle reduction
// inside each row's lane group.
template <int HD>
__global__ void __launch_bounds__(256, 4) flash_bwd_delta_kernel(AttnParams p, const bf16* __restrict__ dO,
                                                                 float* __restrict__ delta, float* __restrict__ lse2) {
  constexpr int LPR = HD / 8;  // lanes per row
  constexpr int U = 4;
  // 32-bit index arithmetic (the launcher checks B * Tq * Hq < 2^31): 64-bit divisions per row cost more than the
  // memory traffic of the row.  Four rows in flight per lane group, four CTAs per SM (64 registers).
  const int total = p.B * p.Tq * p.Hq;
  const int rows_per_pass = gridDim.x * (blockDim.x / LPR);
  const int first = blockIdx.x * (blockDim.x / LPR) + threadIdx.x / LPR;
  const int sub = threadIdx.x % LPR;
  for (int base = first; base < total; base += U * rows_per_pass) {
    uint4 a[U], d[U];
    int idx[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int item = base + u * rows_per_pass;
      a[u] = d[u] = make_uint4(0u, 0u, 0u, 0u);
      idx[u] = -1;
      if (item < total) {
        const int h = item % p.Hq, bt = item / p.Hq;
        const int b = bt / p.Tq, t = bt - b * p.Tq;
        const long long off = (long long)b * p.o_bs + (long long)t * p.o_ts + (long long)h * p.o_hs + sub * 8;
        a[u] = *reinterpret_cast<const uint4*>(p.o + off);
        d[u] = *reinterpret_cast<const uint4*>(dO + off);
        idx[u] = (b * p.Hq + h) * p.Tq + t;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a[u]);
      const __nv_bfloat162* hd = reinterpret_cast<const __nv_bfloat162*>(&d[u]);
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 x = __bfloat1622float2(ha[k]), y = __bfloat1622float2(hd[k]);
        s += x.x * y.x + x.y * y.y;
      }
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (sub == 0 && idx[u] >= 0) {
        delta[idx[u]] = s;
        if (lse2 != nullptr) lse2[idx[u]] = p.lse[idx[u]] * 1.4426950408889634f;  // log-sum-exp in base-2 units
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------------------------
// backward: CTA = 64 keys of one (batch, kv head), 4 warps x 16 keys; loops over the rep query heads of the group
// and over query tiles of 64.  dK, dV accumulate in registers; dQ accumulates in an fp32 buffer via red.add.
// ------------------------------------------------------------------------------------------------------------------
constexpr int FB_BN = 64;  // keys per CTA
constexpr int FB_BM = 64;  // queries per iteration
constexpr int FB_THREADS = 128;

template <int HD>
__global__ void __launch_bounds__(FB_THREADS, 1)
    flash_bwd_kernel(AttnParams p, const bf16* __restrict__ dO, const float* __restrict__ delta,
                     float* __restrict__ dq_acc, bf16* __restrict__ dk, long long dk_bs, long long dk_ts,
                     long long dk_hs, bf16* __restrict__ dv, long long dv_bs, long long dv_ts, long long dv_hs) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + FB_BN * HD * 2;
  const uint32_t sQ = sV + FB_BN * HD * 2;
  const uint32_t sdO = sQ + FB_BM * HD * 2;
  const uint32_t sdS = sdO + FB_BM * HD * 2;  // [64 keys][64 queries] bf16, 128-byte rows, swizzled
  float* s_lse = reinterpret_cast<float*>(smem + (sdS - sK) + FB_BN * FB_BM * 2);
  float* s_delta = s_lse + FB_BM;
  constexpr int KT = HD / 16;
  constexpr int NO = HD / 8;

  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int warp = warp_id(), lane = lane_id();
  const int g = lane >> 2, c = lane & 3;
  const int k0 = kb * FB_BN;
  int kv_end = p.Tk;
  if (p.kv_len != nullptr) kv_end = min(kv_end, p.kv_len[b]);
  const float sl2 = p.scale * 1.4426950408889634f;

  float dk_acc[NO][4], dv_acc[NO][4];
#pragma unroll
  for (int i = 0; i < NO; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk_acc[i][e] = dv_acc[i][e] = 0.f;

  const bf16* Kg = p.k + (long long)b * p.k_bs + (long long)hk * p.k_hs;
  const bf16* Vg = p.v + (long long)b * p.v_bs + (long long)hk * p.v_hs;
  if (k0 < kv_end) {
    load_tile<FB_BN, HD, FB_THREADS>(sK, Kg + (long long)k0 * p.k_ts, p.k_ts, 0, kv_end - k0);
    load_tile<FB_BN, HD, FB_THREADS>(sV, Vg + (long long)k0 * p.v_ts, p.v_ts, 0, kv_end - k0);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();

    const int n_qt = (p.Tq + FB_BM - 1) / FB_BM;
    for (int hr = 0; hr < p.rep; ++hr) {
      const int h = hk * p.rep + hr;
      const bf16* Qg = p.q + (long long)b * p.q_bs + (long long)h * p.q_hs;
      const bf16* dOg = dO + (long long)b * p.o_bs + (long long)h * p.o_hs;
      const float* lse_g = p.lse + ((long long)b * p.Hq + h) * p.Tq;
      const float* del_g = delta + ((long long)b * p.Hq + h) * p.Tq;
      for (int qt = 0; qt < n_qt; ++qt) {
        const int q0 = qt * FB_BM;
        load_tile<FB_BM, HD, FB_THREADS>(sQ, Qg + (long long)q0 * p.q_ts, p.q_ts, 0, p.Tq - q0);
        load_tile<FB_BM, HD, FB_THREADS>(sdO, dOg + (long long)q0 * p.o_ts, p.o_ts, 0, p.Tq - q0);
        cp_async_commit();
        for (int i = threadIdx.x; i < FB_BM; i += FB_THREADS) {
          const bool ok = q0 + i < p.Tq;
          s_lse[i] = ok ? lse_g[q0 + i] * 1.4426950408889634f : INFINITY;
          s_delta[i] = ok ? del_g[q0 + i] : 0.f;
        }
        cp_async_wait<0>();
        __syncthreads();

        // S^T (16 keys x 64 queries) = K_w Q^T ; dP^T = V_w dO^T
        float st[FB_BM / 8][4], dpt[FB_BM / 8][4];
#pragma unroll
        for (int n = 0; n < FB_BM / 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) st[n][e] = dpt[n][e] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KT; ++kk) {
          // this warp's K and V rows (16 keys) as A fragments for this k-step
          uint32_t kf[4], vf[4];
          {
            const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            const int ch = kk * 2 + (lane >> 4);
            ldsm_x4(sK + tile_off<HD>(row, ch), kf[0], kf[1], kf[2], kf[3]);
            ldsm_x4(sV + tile_off<HD>(row, ch), vf[0], vf[1], vf[2], vf[3]);
          }
#pragma unroll
          for (int n2 = 0; n2 < FB_BM / 16; ++n2) {
            const int row = n2 * 16 + (lane & 7) + ((lane >> 4) << 3);
            const int ch = kk * 2 + ((lane >> 3) & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(sQ + tile_off<HD>(row, ch), b0, b1, b2, b3);
            mma16816(st[2 * n2], kf[0], kf[1], kf[2], kf[3], b0, b1);
            mma16816(st[2 * n2 + 1], kf[0], kf[1], kf[2], kf[3], b2, b3);
            ldsm_x4(sdO + tile_off<HD>(row, ch), b0, b1, b2, b3);
            mma16816(dpt[2 * n2], vf[0], vf[1], vf[2], vf[3], b0, b1);
            mma16816(dpt[2 * n2 + 1], vf[0], vf[1], vf[2], vf[3], b2, b3);
          }
        }
        // P^T and dS^T (rows = keys g, g + 8 of this warp; columns = queries)
        uint32_t pt[FB_BM / 8][2], dst_[FB_BM / 8][2];
#pragma unroll
        for (int n = 0; n < FB_BM / 8; ++n) {
          float pv[4], ds[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = k0 + warp * 16 + g + (e >> 1) * 8;
            const int qi = n * 8 + c * 2 + (e & 1);
            float pr = exp2f(st[n][e] * sl2 - s_lse[qi]);
            if (key >= kv_end) pr = 0.f;
            pv[e] = pr;
            ds[e] = pr * (dpt[n][e] - s_delta[qi]);
          }
          pt[n][0] = pack_bf16x2(pv[0], pv[1]);
          pt[n][1] = pack_bf16x2(pv[2], pv[3]);
          dst_[n][0] = pack_bf16x2(ds[0], ds[1]);
          dst_[n][1] = pack_bf16x2(ds[2], ds[3]);
        }
        // dV_w += P^T dO ; dK_w += dS^T Q   (k = queries)
#pragma unroll
        for (int kk = 0; kk < FB_BM / 16; ++kk) {
#pragma unroll
          for (int n2 = 0; n2 < HD / 16; ++n2) {
            const int row = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
            const int ch = n2 * 2 + (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(sdO + tile_off<HD>(row, ch), b0, b1, b2, b3);
            mma16816(dv_acc[2 * n2], pt[2 * kk][0], pt[2 * kk][1], pt[2 * kk + 1][0], pt[2 * kk + 1][1], b0, b1);
            mma16816(dv_acc[2 * n2 + 1], pt[2 * kk][0], pt[2 * kk][1], pt[2 * kk + 1][0], pt[2 * kk + 1][1], b2, b3);
            ldsm_x4_t(sQ + tile_off<HD>(row, ch), b0, b1, b2, b3);
            mma16816(dk_acc[2 * n2], dst_[2 * kk][0], dst_[2 * kk][1], dst_[2 * kk + 1][0], dst_[2 * kk + 1][1], b0,
                     b1);
            mma16816(dk_acc[2 * n2 + 1], dst_[2 * kk][0], dst_[2 * kk][1], dst_[2 * kk + 1][0], dst_[2 * kk + 1][1],
                     b2, b3);
          }
        }
        // dS^T -> shared memory [key][query] (64 x 64 bf16, 8 chunks per row)
        {
          uint8_t* base = smem + (sdS - sK);
#pragma unroll
          for (int n = 0; n < FB_BM / 8; ++n) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              const int key = warp * 16 + g + r * 8;
              const int col = n * 8 + c * 2;
              const int ch = col >> 3;
              const uint32_t off = key * 128 + (((ch ^ (key & 7)) << 4)) + (col & 7) * 2;
              *reinterpret_cast<uint32_t*>(base + off) = dst_[n][r];
            }
          }
        }
        __syncthreads();
        // dQ (queries 16w..16w+15 of the tile) += dS K  (k = the 64 keys)
        {
          float dqp[NO][4];
#pragma unroll
          for (int i = 0; i < NO; ++i) dqp[i][0] = dqp[i][1] = dqp[i][2] = dqp[i][3] = 0.f;
#pragma unroll
          for (int kk = 0; kk < FB_BN / 16; ++kk) {
            uint32_t a0, a1, a2, a3;
            {
              // A = dS (m = query, k = key) from the [key][query] tile: transposed load
              const int row = kk * 16 + (lane & 7) + ((lane >> 4) << 3);
              const int chq = warp * 2 + ((lane >> 3) & 1);
              const uint32_t off = row * 128 + (((chq ^ (row & 7)) << 4));
              ldsm_x4_t(sdS + off, a0, a1, a2, a3);
            }
#pragma unroll
            for (int n2 = 0; n2 < HD / 16; ++n2) {
              const int row = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
              const int ch = n2 * 2 + (lane >> 4);
              uint32_t b0, b1, b2, b3;
              ldsm_x4_t(sK + tile_off<HD>(row, ch), b0, b1, b2, b3);
              mma16816(dqp[2 * n2], a0, a1, a2, a3, b0, b1);
              mma16816(dqp[2 * n2 + 1], a0, a1, a2, a3, b2, b3);
            }
          }
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int t = q0 + warp * 16 + g + r * 8;
            if (t < p.Tq) {
              float* dst = dq_acc + ((long long)b * p.Tq + t) * p.Hq * HD + (long long)h * HD + c * 2;
#pragma unroll
              for (int i = 0; i < NO; ++i) red_add_v2(dst + i * 8, dqp[i][2 * r] * p.scale, dqp[i][2 * r + 1] * p.scale);
            }
          }
        }
        __syncthreads();
      }
    }
  }
  // write dK (scaled), dV for this warp's 16 keys
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = k0 + warp * 16 + g + r * 8;
    if (key >= p.Tk) continue;
    bf16* kd = dk + (long long)b * dk_bs + (long long)key * dk_ts + (long long)hk * dk_hs + c * 2;
    bf16* vd = dv + (long long)b * dv_bs + (long long)key * dv_ts + (long long)hk * dv_hs + c * 2;
#pragma unroll
    for (int i = 0; i < NO; ++i) {
      *reinterpret_cast<__nv_bfloat162*>(kd + i * 8) =
          __floats2bfloat162_rn(dk_acc[i][2 * r] * p.scale, dk_acc[i][2 * r + 1] * p.scale);
      *reinterpret_cast<__nv_bfloat162*>(vd + i * 8) = __floats2bfloat162_rn(dv_acc[i][2 * r], dv_acc[i][2 * r + 1]);
    }
  }
}

// fp32 [B, Tq, Hq, HD] dQ accumulator -> bf16 strided dq
template <int HD>
__global__ void dq_convert_kernel(AttnParams p, const float* __restrict__ acc, bf16* __restrict__ dq, long long bs,
                                  long long ts, long long hs) {
  const long long n8 = (long long)p.B * p.Tq * p.Hq * (HD / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const int d8 = (int)(i % (HD / 8));
    long long r = i / (HD / 8);
    const int h = (int)(r % p.Hq);
    r /= p.Hq;
    const int t = (int)(r % p.Tq), b = (int)(r / p.Tq);
    const float4 a = *reinterpret_cast<const float4*>(acc + i * 8);
    const float4 c2 = *reinterpret_cast<const float4*>(acc + i * 8 + 4);
    uint4 u;
    u.x = pack_bf16x2(a.x, a.y);
    u.y = pack_bf16x2(a.z, a.w);
    u.z = pack_bf16x2(c2.x, c2.y);
    u.w = pack_bf16x2(c2.z, c2.w);
    *reinterpret_cast<uint4*>(dq + (long long)b * bs + (long long)t * ts + (long long)h * hs + d8 * 8) = u;
  }
}

// ------------------------------------------------------------------------------------------------------------------
// launchers
// ------------------------------------------------------------------------------------------------------------------
// delta kernel grid: 256 threads cover 256 / (hd / 8) rows per pass; at most 8 resident blocks per SM worth
static unsigned delta_grid(long long items, int hd) {  // items < 2^31 (checked by the callers)
  const long long rows_per_block = 256 / (hd / 8);
  const long long want = (items + rows_per_block - 1) / rows_per_block;
  return (unsigned)std::min<long long>(want, (long long)num_sms() * 16);
}

template <int HD>
static cudaError_t fwd_impl(const AttnParams& p, cudaStream_t s) {
  const int smem = (FA_BM + 4 * FA_BN) * HD * 2;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(flash_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    set = true;
  }
  dim3 grid((p.Tq + FA_BM - 1) / FA_BM, p.Hq, p.B);
  flash_fwd_kernel<HD><<<grid, FA_FWD_THREADS, smem, s>>>(p);
  return cudaGetLastError();
}

cudaError_t attention_fwd_launch(const AttnParams& p, cudaStream_t s) {
  if (p.hd == 128) return fwd_impl<128>(p, s);
  if (p.hd == 64) return fwd_impl<64>(p, s);
  return cudaErrorInvalidValue;
}

template <int HD>
static cudaError_t bwd_impl(const AttnParams& p, const bf16* dO, float* delta, float* dq_acc, bf16* dq, long long dq_bs,
                            long long dq_ts, long long dq_hs, bf16* dk, long long dk_bs, long long dk_ts,
                            long long dk_hs, bf16* dv, long long dv_bs, long long dv_ts, long long dv_hs,
                            cudaStream_t s) {
  {
    const long long items = (long long)p.B * p.Tq * p.Hq;
    if (items >= (1ll << 31)) return cudaErrorInvalidValue;
    flash_bwd_delta_kernel<HD><<<delta_grid(items, HD), 256, 0, s>>>(p, dO, delta, nullptr);
  }
  cudaError_t e = cudaMemsetAsync(dq_acc, 0, sizeof(float) * (size_t)p.B * p.Tq * p.Hq * HD, s);
  if (e != cudaSuccess) return e;
  const int smem = (2 * FB_BN + 2 * FB_BM) * HD * 2 + FB_BN * FB_BM * 2 + 2 * FB_BM * 4;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(flash_bwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    set = true;
  }
  dim3 grid((p.Tk + FB_BN - 1) / FB_BN, p.Hkv, p.B);
  flash_bwd_kernel<HD><<<grid, FB_THREADS, smem, s>>>(p, dO, delta, dq_acc, dk, dk_bs, dk_ts, dk_hs, dv, dv_bs,
                                                       dv_ts, dv_hs);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (dq != nullptr) {
    const long long n8 = (long long)p.B * p.Tq * p.Hq * (HD / 8);
    const int grid2 = (int)std::min<long long>((n8 + 255) / 256, (long long)num_sms() * 16);
    dq_convert_kernel<HD><<<grid2, 256, 0, s>>>(p, dq_acc, dq, dq_bs, dq_ts, dq_hs);
  }
  return cudaGetLastError();
}

// delta = rowsum(dO * O) and a zeroed dQ accumulator (shared by both backward kernels)
cudaError_t attention_bwd_prep_launch(const AttnParams& p, const bf16* dO, float* delta, float* dq_acc, cudaStream_t s,
                                      float* lse2) {
  const long long items = (long long)p.B * p.Tq * p.Hq;
  if (items >= (1ll << 31)) return cudaErrorInvalidValue;
  if (p.hd == 128) flash_bwd_delta_kernel<128><<<delta_grid(items, 128), 256, 0, s>>>(p, dO, delta, lse2);
  else if (p.hd == 64) flash_bwd_delta_kernel<64><<<delta_grid(items, 64), 256, 0, s>>>(p, dO, delta, lse2);
  else return cudaErrorInvalidValue;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || dq_acc == nullptr) return e;
  return cudaMemsetAsync(dq_acc, 0, sizeof(float) * (size_t)p.B * p.Tq * p.Hq * p.hd, s);
}

cudaError_t attention_dq_convert_launch(const AttnParams& p, const float* dq_acc, bf16* dq, long long bs, long long ts,
                                        long long hs, cudaStream_t s) {
  const long long n8 = (long long)p.B * p.Tq * p.Hq * (p.hd / 8);
  const int grid = (int)std::min<long long>((n8 + 255) / 256, (long long)num_sms() * 16);
  if (p.hd == 128) dq_convert_kernel<128><<<grid, 256, 0, s>>>(p, dq_acc, dq, bs, ts, hs);
  else if (p.hd == 64) dq_convert_kernel<64><<<grid, 256, 0, s>>>(p, dq_acc, dq, bs, ts, hs);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t attention_bwd_launch(const AttnParams& p, const bf16* dO, float* delta, float* dq_acc, bf16* dq,
                                 long long dq_bs, long long dq_ts, long long dq_hs, bf16* dk, long long dk_bs,
                                 long long dk_ts, long long dk_hs, bf16* dv, long long dv_bs, long long dv_ts,
                                 long long dv_hs, cudaStream_t s) {
  if (p.hd == 128)
    return bwd_impl<128>(p, dO, delta, dq_acc, dq, dq_bs, dq_ts, dq_hs, dk, dk_bs, dk_ts, dk_hs, dv, dv_bs, dv_ts,
                         dv_hs, s);
  if (p.hd == 64)
    return bwd_impl<64>(p, dO, delta, dq_acc, dq, dq_bs, dq_ts, dq_hs, dk, dk_bs, dk_ts, dk_hs, dv, dv_bs, dv_ts,
                        dv_hs, s);
  return cudaErrorInvalidValue;
}

}  // namespace tgo
