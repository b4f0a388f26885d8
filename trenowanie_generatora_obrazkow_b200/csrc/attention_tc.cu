// Flash attention forward on the 5th-generation tensor cores (tcgen05 + TMEM), head dims 64 and 128.
//
// CTA = 128 query rows of one (batch, head); 192 threads:
//   warp 0        TMA loads: Q once, then K / V tiles of 64 keys into a 2-stage ring
//   warp 1        TMEM allocation (256 columns) and the single MMA-issuing thread:
//                   S_j = Q K_j^T  (M 128, N 64, K hd)  -> TMEM, double buffered (columns 0 / 64)
//                   O  += P_j V_j  (M 128, N hd, K 64)  -> TMEM columns 128 .. 128 + hd
//   warps 2-5     softmax: thread = query row = TMEM lane; reads its S row (tcgen05.ld), online softmax in
//                 exp2 form, writes P (bf16) into a 128-byte-swizzled shared tile the next MMA reads as its A
//                 operand; rescales its O row in TMEM only when its running max grew by more than 2^8 (the
//                 stale max is used consistently, so the result is exact); final O / l and log-sum-exp.
// S_{j+1} is issued before P_j V_j, so the tensor core works on the next tile while the softmax warps work on
// this one; two CTAs per SM (112 KB shared, 256 TMEM columns each) interleave as well.
// Key masking by per-sample valid length; grouped-query attention by head mapping. Output and LSE layout match
// the mma.sync kernel in attention.cu, so the backward there consumes them unchanged.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tgo {

namespace {

constexpr int TQ = 128;      // query rows per CTA
constexpr int TK = 64;       // keys per tile
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 256;
constexpr int S_COL = 0;     // S buffers at columns 0 and 64
constexpr int O_COL = 128;   // O at columns 128 .. 128 + hd
constexpr float kRescaleThreshold = 8.f;  // log2 units

__device__ __forceinline__ float ex2(float x) {  // hardware 2^x (MUFU)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int HD>
struct FwdSmem {
  static constexpr int Q_BYTES = TQ * HD * 2;          // HD / 64 blocks of 128 rows x 128 B
  static constexpr int KV_BYTES = TK * HD * 2;         // HD / 64 blocks of 64 rows x 128 B
  static constexpr int P_BYTES = TQ * TK * 2;          // 128 rows x 128 B
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * KV_BYTES;
  static constexpr int P_OFF = V_OFF + 2 * KV_BYTES;
  static constexpr int BAR_OFF = P_OFF + P_BYTES;
  static constexpr int TOTAL = BAR_OFF + 256;
};

struct FwdBars {
  uint64_t q_full;
  uint64_t kv_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t p_full;
  uint64_t pv_done;
  uint32_t tmem_base;
  int abort_flag;
};

}  // namespace

template <int HD>
__global__ void __launch_bounds__(THREADS, 2)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, AttnParams p, int* err) {
  using L = FwdSmem<HD>;
  extern __shared__ __align__(1024) uint8_t smem[];
  FwdBars* bars = reinterpret_cast<FwdBars*>(smem + L::BAR_OFF);
  const int warp = warp_id(), lane = lane_id();
  if ((smem_u32(smem) & 1023) != 0) {  // the swizzled tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) record_error(err, ERR_BAD_ARGS);
    return;
  }
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.rep;
  const int q0 = qb * TQ;
  int kv_end = p.Tk;
  if (p.kv_len != nullptr) kv_end = min(kv_end, p.kv_len[b]);
  const int n_tiles = max(0, (kv_end + TK - 1) / TK);

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->kv_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_empty[i], 128);
    }
    mbar_init(&bars->p_full, 128);
    mbar_init(&bars->pv_done, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      // ---------------- TMA loads ----------------
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_expect_tx(&bars->q_full, L::Q_BYTES);
#pragma unroll
      for (int blk = 0; blk < HD / 64; ++blk)
        tma_load_4d(smem + L::Q_OFF + blk * TQ * 128, &tmQ, &bars->q_full, blk * 64, q0, h, b);
      for (int j = 0; j < n_tiles && !*abort_flag; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&bars->kv_empty[st], ((j >> 1) & 1) ^ 1, err, ERR_MBAR_TIMEOUT_PRODUCER)) {
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&bars->kv_full[st], 2 * L::KV_BYTES);
#pragma unroll
        for (int blk = 0; blk < HD / 64; ++blk) {
          tma_load_4d(smem + L::K_OFF + st * L::KV_BYTES + blk * TK * 128, &tmK, &bars->kv_full[st], blk * 64,
                      j * TK, hk, b);
          tma_load_4d(smem + L::V_OFF + st * L::KV_BYTES + blk * TK * 128, &tmV, &bars->kv_full[st], blk * 64,
                      j * TK, hk, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {
      // ---------------- MMA issue ----------------
      constexpr uint32_t idesc_s = idesc_bf16_f32(TQ, TK, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(TQ, HD, false, true);
      const uint32_t sq = smem_u32(smem + L::Q_OFF);
      const uint32_t sp = smem_u32(smem + L::P_OFF);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&bars->kv_full[st], (j >> 1) & 1, err, ERR_MBAR_TIMEOUT_MMA)) return false;
        if (!mbar_wait(&bars->s_empty[st], ((j >> 1) & 1) ^ 1, err, ERR_MBAR_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + L::K_OFF + st * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t blk = kk >> 2, sub = (kk & 3) * 32;
          umma_f16(tmem + S_COL + st * TK, sdesc_sw128(sq + blk * TQ * 128 + sub, 16, 1024),
                   sdesc_sw128(sk + blk * TK * 128 + sub, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[st]);
        return true;
      };
      bool ok = mbar_wait(&bars->q_full, 0, err, ERR_MBAR_TIMEOUT_MMA) && issue_s(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&bars->p_full, j & 1, err, ERR_MBAR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + L::V_OFF + (j & 1) * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk)
          umma_f16(tmem + O_COL, sdesc_sw128(sp + kk * 32, 16, 1024), sdesc_sw128(sv + kk * 2048, TK * 128, 1024),
                   idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bars->kv_empty[j & 1]);
        umma_commit(&bars->pv_done);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- softmax / epilogue ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane == query row within the tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    uint8_t* prow = smem + L::P_OFF + row * 128;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      int w_ok = 1;
      if (lane == 0) w_ok = mbar_wait(&bars->s_full[st], (j >> 1) & 1, err, ERR_MBAR_TIMEOUT_EPILOGUE) ? 1 : 0;
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
      if (!w_ok) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld_32x32b_x32(tmem + lane_base + S_COL + st * TK, sr[0]);
      tmem_ld_32x32b_x32(tmem + lane_base + S_COL + st * TK + 32, sr[1]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&bars->s_empty[st]);
      const int kbase = j * TK;
      float smax = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = kbase + c * 32 + i;
          float v = __uint_as_float(sr[c][i]) * sl2;
          if (key >= kv_end) v = -INFINITY;
          sr[c][i] = __float_as_uint(v);
          smax = fmaxf(smax, v);
        }
      // PV_{j-1} must be complete before P is overwritten and before O is touched
      if (j > 0) {
        if (lane == 0) w_ok = mbar_wait(&bars->pv_done, (j - 1) & 1, err, ERR_MBAR_TIMEOUT_EPILOGUE) ? 1 : 0;
        w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
        if (!w_ok) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
      }
      const float m_new = fmaxf(m, smax);
      const bool need = (j > 0) && (m_new > m + kRescaleThreshold);
      if (__any_sync(0xffffffffu, need)) {
        // rescale this warp's O rows to the new running max
        const float corr = (m == -INFINITY) ? 0.f : ex2(m - m_new);
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tmem + lane_base + O_COL + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
          tmem_st_32x32b_x32(tmem + lane_base + O_COL + c * 32, o);
        }
        tmem_st_wait();
        l *= corr;
        m = m_new;
      } else if (j == 0) {
        m = m_new;
      }
      const float mu = (m == -INFINITY) ? 0.f : m;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {  // 8 keys -> one 16-byte chunk
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float a = ex2(__uint_as_float(sr[c][ch * 8 + 2 * e]) - mu);
            const float bq = ex2(__uint_as_float(sr[c][ch * 8 + 2 * e + 1]) - mu);
            __nv_bfloat162 pr = __floats2bfloat162_rn(a, bq);
            const float2 back = __bfloat1622float2(pr);
            rs += back.x + back.y;
            pk[e] = *reinterpret_cast<uint32_t*>(&pr);
          }
          const int chunk = c * 4 + ch;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ (row & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
      l += rs;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_full);
    }
    // epilogue: O / l -> bf16, log-sum-exp
    if (ok && n_tiles > 0) {
      int w_ok = 1;
      if (lane == 0) w_ok = mbar_wait(&bars->pv_done, (n_tiles - 1) & 1, err, ERR_MBAR_TIMEOUT_EPILOGUE) ? 1 : 0;
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
      ok = w_ok != 0;
      __syncwarp();
      tc_fence_after();
    }
    const int t = q0 + row;
    const float inv = (l > 0.f) ? 1.f / l : 0.f;
    if (ok) {
      __nv_bfloat16* dst = p.o + (long long)b * p.o_bs + (long long)t * p.o_ts + (long long)h * p.o_hs;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        if (n_tiles > 0) {
          tmem_ld_32x32b_x32(tmem + lane_base + O_COL + c * 32, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (t < p.Tq) {
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(o[v4 * 8 + 0]) * inv, __uint_as_float(o[v4 * 8 + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(o[v4 * 8 + 2]) * inv, __uint_as_float(o[v4 * 8 + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(o[v4 * 8 + 4]) * inv, __uint_as_float(o[v4 * 8 + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(o[v4 * 8 + 6]) * inv, __uint_as_float(o[v4 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + v4 * 8) = u;
          }
        }
      }
      if (t < p.Tq && p.lse != nullptr)
        p.lse[((long long)b * p.Hq + h) * p.Tq + t] =
            (l > 0.f) ? (m + log2f(l)) * 0.6931471805599453f : INFINITY;
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int HD>
static cudaError_t fwd_tc_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                               const AttnParams& p, int* err, cudaStream_t s) {
  using L = FwdSmem<HD>;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(flash_fwd_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
    set = true;
  }
  dim3 grid((p.Tq + TQ - 1) / TQ, p.Hq, p.B);
  flash_fwd_tc_kernel<HD><<<grid, THREADS, L::TOTAL, s>>>(tq, tk, tv, p, err);
  return cudaGetLastError();
}

cudaError_t attention_fwd_tc_launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                    const AttnParams& p, int* err, cudaStream_t s) {
  if (p.hd == 128) return fwd_tc_impl<128>(tq, tk, tv, p, err, s);
  if (p.hd == 64) return fwd_tc_impl<64>(tq, tk, tv, p, err, s);
  return cudaErrorInvalidValue;
}


// ==================================================================================================================
// Backward on tcgen05 (head dim 128).
//
// CTA = 128 keys of one (batch, kv head); loops over the rep query heads of the group and over query tiles of 64.
// Per iteration (Q_i, dO_i: 64 queries):
//   MMA1  S^T  = K Q_i^T          M 128 keys, N 64, K 128      TMEM cols   0 ..  63
//   MMA2  dP^T = V dO_i^T         M 128 keys, N 64, K 128      TMEM cols  64 .. 127
//   softmax warps (thread = key): P^T = 2^(S^T scale log2e - lse log2e), dS^T = P^T (dP^T - delta) -> bf16 tiles
//   MMA3  dV  += P^T dO_i         M 128 keys, N 128, K 64      TMEM cols 256 .. 383
//   MMA4  dK  += dS^T Q_i         M 128 keys, N 128, K 64      TMEM cols 384 .. 511
//   MMA5  dQ^T = K^T dS^T         M 128 (head dim), N 64, K 128 keys   TMEM cols 128 .. 191
//   dQ warps (thread = head-dim lane): dQ^T row -> scale -> red.global.add into the fp32 dQ accumulator
// Operand majors: K / V / Q / dO tiles are TMA-loaded once in the [token][head_dim] layout and read K-major or
// MN-major as each product needs; P^T / dS^T are written K-major (queries contiguous) and double buffered, so the
// softmax of iteration i+1 overlaps MMA3-5 of iteration i, and MMA1/2 of iteration i+1 overlap the softmax of i.
// Warps: 0 TMA, 1 MMA (+ TMEM), 2-5 softmax + final dK / dV, 6-9 dQ drain.
// ==================================================================================================================
namespace {

constexpr int BK_KEYS = 128;
constexpr int BQ = 64;
constexpr int BWD_THREADS = 320;

struct BwdSmem {  // head dim 128
  static constexpr int K_OFF = 0;                              // 2 blocks x 128 rows x 128 B
  static constexpr int V_OFF = K_OFF + 32768;
  static constexpr int Q_OFF = V_OFF + 32768;                  // 2 stages x (2 blocks x 64 rows x 128 B)
  static constexpr int DO_OFF = Q_OFF + 2 * 16384;
  static constexpr int PT_OFF = DO_OFF + 2 * 16384;            // 2 buffers x 128 rows x 128 B
  static constexpr int DS_OFF = PT_OFF + 2 * 16384;
  static constexpr int STAT_OFF = DS_OFF + 2 * 16384;          // lse / delta: 2 slots x 2 x 64 floats
  static constexpr int BAR_OFF = STAT_OFF + 1024;
  static constexpr int TOTAL = BAR_OFF + 256;
};

struct BwdBars {
  uint64_t kv_full;
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t s_full;
  uint64_t s_empty;
  uint64_t p_full[2];
  uint64_t p_empty[2];
  uint64_t dq_full;
  uint64_t dq_empty;
  uint64_t acc_done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void softmax_group_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  int ok = 1;
  if (lane_id() == 0) ok = mbar_wait(bar, parity, err, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

}  // namespace

__global__ void __launch_bounds__(BWD_THREADS, 1)
    flash_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                        AttnParams p, const float* __restrict__ delta, float* __restrict__ dq_acc,
                        __nv_bfloat16* __restrict__ dk, long long dk_bs, long long dk_ts, long long dk_hs,
                        __nv_bfloat16* __restrict__ dv, long long dv_bs, long long dv_ts, long long dv_hs, int* err) {
  constexpr int HD = 128;
  using L = BwdSmem;
  extern __shared__ __align__(1024) uint8_t smem[];
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + L::BAR_OFF);
  float* stat = reinterpret_cast<float*>(smem + L::STAT_OFF);  // [slot][0: lse*log2e | 1: delta][64]
  const int warp = warp_id(), lane = lane_id();
  if ((smem_u32(smem) & 1023) != 0) {
    if (threadIdx.x == 0) record_error(err, ERR_BAD_ARGS);
    return;
  }
  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int k0 = kb * BK_KEYS;
  int kv_end = p.Tk;
  if (p.kv_len != nullptr) kv_end = min(kv_end, p.kv_len[b]);
  const bool active = k0 < kv_end;
  const int n_qt = (p.Tq + BQ - 1) / BQ;
  const int n_it = active ? p.rep * n_qt : 0;

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->q_full[i], 1);
      mbar_init(&bars->q_empty[i], 1);
      mbar_init(&bars->p_full[i], 128);
      mbar_init(&bars->p_empty[i], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->s_empty, 128);
    mbar_init(&bars->dq_full, 1);
    mbar_init(&bars->dq_empty, 128);
    mbar_init(&bars->acc_done, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    if (lane == 0 && n_it > 0) {
      // ---------------- TMA loads ----------------
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmdO);
      mbar_expect_tx(&bars->kv_full, 2 * 32768);
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        tma_load_4d(smem + L::K_OFF + blk * 16384, &tmK, &bars->kv_full, blk * 64, k0, hk, b);
        tma_load_4d(smem + L::V_OFF + blk * 16384, &tmV, &bars->kv_full, blk * 64, k0, hk, b);
      }
      for (int i = 0; i < n_it && !*abort_flag; ++i) {
        const int st = i & 1;
        const int h = hk * p.rep + i / n_qt, q0 = (i % n_qt) * BQ;
        if (!mbar_wait(&bars->q_empty[st], ((i >> 1) & 1) ^ 1, err, ERR_MBAR_TIMEOUT_PRODUCER)) {
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&bars->q_full[st], 2 * 16384);
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          tma_load_4d(smem + L::Q_OFF + st * 16384 + blk * 8192, &tmQ, &bars->q_full[st], blk * 64, q0, h, b);
          tma_load_4d(smem + L::DO_OFF + st * 16384 + blk * 8192, &tmdO, &bars->q_full[st], blk * 64, q0, h, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      // ---------------- MMA issue ----------------
      constexpr uint32_t id_s = idesc_bf16_f32(128, BQ, false, false);   // S^T, dP^T
      constexpr uint32_t id_kv = idesc_bf16_f32(128, HD, false, true);   // dV, dK
      constexpr uint32_t id_q = idesc_bf16_f32(128, BQ, true, true);     // dQ^T
      const uint32_t sK = smem_u32(smem + L::K_OFF), sV = smem_u32(smem + L::V_OFF);
      auto issue_s = [&](int i) -> bool {
        const int st = i & 1;
        if (!mbar_wait(&bars->q_full[st], (i >> 1) & 1, err, ERR_MBAR_TIMEOUT_MMA)) return false;
        if (i > 0 && !mbar_wait(&bars->s_empty, (i - 1) & 1, err, ERR_MBAR_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t sQ = smem_u32(smem + L::Q_OFF + st * 16384), sdO = smem_u32(smem + L::DO_OFF + st * 16384);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t blk = kk >> 2, sub = (kk & 3) * 32;
          umma_f16(tmem + 0, sdesc_sw128(sK + blk * 16384 + sub, 16, 1024),
                   sdesc_sw128(sQ + blk * 8192 + sub, 16, 1024), id_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t blk = kk >> 2, sub = (kk & 3) * 32;
          umma_f16(tmem + 64, sdesc_sw128(sV + blk * 16384 + sub, 16, 1024),
                   sdesc_sw128(sdO + blk * 8192 + sub, 16, 1024), id_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full);
        return true;
      };
      bool ok = mbar_wait(&bars->kv_full, 0, err, ERR_MBAR_TIMEOUT_MMA) && issue_s(0);
      for (int i = 0; i < n_it && ok; ++i) {
        const int st = i & 1;
        if (i + 1 < n_it && !issue_s(i + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&bars->p_full[st], (i >> 1) & 1, err, ERR_MBAR_TIMEOUT_MMA) ||
            !mbar_wait(&bars->dq_empty, (i & 1) ^ 1, err, ERR_MBAR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sQ = smem_u32(smem + L::Q_OFF + st * 16384), sdO = smem_u32(smem + L::DO_OFF + st * 16384);
        const uint32_t sPT = smem_u32(smem + L::PT_OFF + st * 16384), sDS = smem_u32(smem + L::DS_OFF + st * 16384);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dV += P^T dO
          umma_f16(tmem + 256, sdesc_sw128(sPT + kk * 32, 16, 1024), sdesc_sw128(sdO + kk * 2048, 8192, 1024), id_kv,
                   (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dK += dS^T Q
          umma_f16(tmem + 384, sdesc_sw128(sDS + kk * 32, 16, 1024), sdesc_sw128(sQ + kk * 2048, 8192, 1024), id_kv,
                   (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < BK_KEYS / 16; ++kk)  // dQ^T = K^T dS^T
          umma_f16(tmem + 128, sdesc_sw128(sK + kk * 2048, 16384, 1024), sdesc_sw128(sDS + kk * 2048, 8192, 1024),
                   id_q, kk > 0 ? 1u : 0u);
        umma_commit(&bars->p_empty[st]);
        umma_commit(&bars->q_empty[st]);
        umma_commit(&bars->dq_full);
      }
      if (ok) umma_commit(&bars->acc_done);
      else *abort_flag = 1;
    }
  } else if (warp < 6) {
    // ---------------- softmax (thread = key row), final dK / dV ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int tid = threadIdx.x - 64;  // 0..127
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale * 1.4426950408889634f;
    const bool key_ok = k0 + r < kv_end;
    bool ok = true;
    for (int i = 0; i < n_it; ++i) {
      const int st = i & 1;
      const int h = hk * p.rep + i / n_qt, q0 = (i % n_qt) * BQ;
      {  // stage lse (pre-scaled by log2 e) and delta of this query tile
        float* slot = stat + st * 128;
        const int q = tid & 63;
        const bool in = q0 + q < p.Tq;
        const long long idx = ((long long)b * p.Hq + h) * p.Tq + q0 + q;
        if (tid < 64) slot[q] = in ? p.lse[idx] * 1.4426950408889634f : INFINITY;
        else slot[64 + q] = in ? delta[idx] : 0.f;
      }
      softmax_group_sync();
      if (!warp_wait(&bars->s_full, i & 1, err, ERR_MBAR_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[2][32], dp[2][32];
      tmem_ld_32x32b_x32(tmem + lane_base + 0, sv[0]);
      tmem_ld_32x32b_x32(tmem + lane_base + 32, sv[1]);
      tmem_ld_32x32b_x32(tmem + lane_base + 64, dp[0]);
      tmem_ld_32x32b_x32(tmem + lane_base + 96, dp[1]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&bars->s_empty);
      if (!warp_wait(&bars->p_empty[st], ((i >> 1) & 1) ^ 1, err, ERR_MBAR_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      const float* slot = stat + st * 128;
      uint8_t* pt_row = smem + L::PT_OFF + st * 16384 + r * 128;
      uint8_t* ds_row = smem + L::DS_OFF + st * 16384 + r * 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t pk[4], dk4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float pv[2], dsv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int qi = c * 32 + ch * 8 + 2 * e + u;
              float pr = ex2(__uint_as_float(sv[c][ch * 8 + 2 * e + u]) * sl2 - slot[qi]);
              pr = key_ok ? pr : 0.f;
              pv[u] = pr;
              dsv[u] = pr * (__uint_as_float(dp[c][ch * 8 + 2 * e + u]) - slot[64 + qi]);
            }
            pk[e] = pack_bf16x2(pv[0], pv[1]);
            dk4[e] = pack_bf16x2(dsv[0], dsv[1]);
          }
          const int chunk = c * 4 + ch;
          const int off = (chunk ^ (r & 7)) << 4;
          *reinterpret_cast<uint4*>(pt_row + off) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(ds_row + off) = make_uint4(dk4[0], dk4[1], dk4[2], dk4[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_full[st]);
    }
    if (ok && n_it > 0) ok = warp_wait(&bars->acc_done, 0, err, ERR_MBAR_TIMEOUT_EPILOGUE);
    tc_fence_after();
    const int key = k0 + r;
    if (ok) {
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {  // 0: dV, 1: dK (scaled)
        __nv_bfloat16* dst = which == 0 ? dv + (long long)b * dv_bs + (long long)key * dv_ts + (long long)hk * dv_hs
                                        : dk + (long long)b * dk_bs + (long long)key * dk_ts + (long long)hk * dk_hs;
        const float mul = which == 0 ? 1.f : p.scale;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          if (n_it > 0) {
            tmem_ld_32x32b_x32(tmem + lane_base + 256 + which * 128 + c * 32, o);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0u;
          }
          if (key < p.Tk) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              uint4 u;
              u.x = pack_bf16x2(__uint_as_float(o[v4 * 8 + 0]) * mul, __uint_as_float(o[v4 * 8 + 1]) * mul);
              u.y = pack_bf16x2(__uint_as_float(o[v4 * 8 + 2]) * mul, __uint_as_float(o[v4 * 8 + 3]) * mul);
              u.z = pack_bf16x2(__uint_as_float(o[v4 * 8 + 4]) * mul, __uint_as_float(o[v4 * 8 + 5]) * mul);
              u.w = pack_bf16x2(__uint_as_float(o[v4 * 8 + 6]) * mul, __uint_as_float(o[v4 * 8 + 7]) * mul);
              *reinterpret_cast<uint4*>(dst + c * 32 + v4 * 8) = u;
            }
          }
        }
      }
    } else {
      *abort_flag = 1;
    }
  } else {
    // ---------------- dQ drain (thread = head-dim lane) ----------------
    const int quarter = warp & 3;
    const int d = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    for (int i = 0; i < n_it; ++i) {
      const int h = hk * p.rep + i / n_qt, q0 = (i % n_qt) * BQ;
      if (!warp_wait(&bars->dq_full, i & 1, err, ERR_MBAR_TIMEOUT_EPILOGUE)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      uint32_t v[2][32];
      tmem_ld_32x32b_x32(tmem + lane_base + 128, v[0]);
      tmem_ld_32x32b_x32(tmem + lane_base + 160, v[1]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&bars->dq_empty);
      float* base = dq_acc + ((long long)b * p.Tq) * p.Hq * HD + (long long)h * HD + d;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll 8
        for (int q = 0; q < 32; ++q) {
          const int t = q0 + c * 32 + q;
          if (t < p.Tq) atomicAdd(base + (long long)t * p.Hq * HD, __uint_as_float(v[c][q]) * p.scale);
        }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

cudaError_t attention_bwd_tc_launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                    const CUtensorMap& tdo, const AttnParams& p, const float* delta, float* dq_acc,
                                    __nv_bfloat16* dk, long long dk_bs, long long dk_ts, long long dk_hs,
                                    __nv_bfloat16* dv, long long dv_bs, long long dv_ts, long long dv_hs, int* err,
                                    cudaStream_t s) {
  if (p.hd != 128) return cudaErrorInvalidValue;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(flash_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdSmem::TOTAL);
    set = true;
  }
  dim3 grid((p.Tk + BK_KEYS - 1) / BK_KEYS, p.Hkv, p.B);
  flash_bwd_tc_kernel<<<grid, BWD_THREADS, BwdSmem::TOTAL, s>>>(tq, tk, tv, tdo, p, delta, dq_acc, dk, dk_bs, dk_ts,
                                                               dk_hs, dv, dv_bs, dv_ts, dv_hs, err);
  return cudaGetLastError();
}

}  // namespace tgo
