// Flash attention forward on the 5th-generation tensor cores (tcgen05 + TMEM), head dims 64 and 128.
//
// Persistent CTA (one per SM, 320 threads) walking work items = two tiles of 128 query rows of one (batch, head):
//   warp 0        TMA loads: both Q tiles of an item, then K and V tiles of 128 keys; K into a 3-stage ring one
//                 tile ahead of V (2-stage ring): a K tile is free once S of both Q tiles is computed, a V tile
//                 only after both P V products
//   warp 1        TMEM allocation (512 columns) and the single MMA-issuing thread, per K / V tile j:
//                   S_g(j+1) = Q_g K_{j+1}^T  (M 128, N 128, K hd) -> TMEM columns g * 128
//                   O_g += P_g(j) V_j          (M 128, N hd, K 128) -> TMEM 256 + g * hd, P read from TMEM
//   warps 2-5/6-9 softmax of Q tile 0 / 1: thread = query row = TMEM lane; reads its S row (tcgen05.ld), online
//                 softmax in exp2 form with packed f32x2 arithmetic and 3-input max, a fraction of the
//                 exponentials as FMA-pipe polynomials (the MUFU unit alone cannot keep up with the tensor core at
//                 head dim 128), writes P (bf16 pairs) back over the first 64 columns of its S buffer (tcgen05.st),
//                 where the P V MMA reads it as its A operand; rescales its O row in TMEM only when its running
//                 max grew by more than 2^8 (the stale max is used consistently, so the result is exact); before
//                 writing P it waits for the previous P V of the other tile (see the note at the store);
//                 final O / l and log-sum-exp.
// Key masking by per-sample valid length; grouped-query attention by head mapping. Output and LSE layout match
// the mma.sync kernel in attention.cu, so the backward there consumes them unchanged.
// Packed variable-length sequences (cu_seqlens) and causal masking serve the frozen caption LM (inference): a CTA
// reads its sequence's offset, loads its Q / K / V tiles from there, masks keys past the sequence (and, when
// causal, keys after each row's query) and stores only its sequence's rows; a causal CTA stops at its diagonal.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tgo {

namespace {

constexpr int TQ = 128;      // query rows per Q tile (one softmax warpgroup)
constexpr int NQ = 2;        // Q tiles per CTA
constexpr int TK = 128;      // keys per K / V tile
constexpr int K_STAGES = 3;  // K ring (loaded one tile ahead of V)
constexpr int V_STAGES = 2;  // V ring
constexpr int THREADS = 320; // warp 0 TMA, warp 1 MMA, warps 2-5 softmax of Q tile 0, warps 6-9 of Q tile 1
constexpr int TMEM_COLS = 512;
constexpr int O_COL = 256;   // Q tile g: S / P at g * 128 (P: bf16 pairs in the first 64 columns); O at 256 + g * hd
constexpr float kRescaleThreshold = 8.f;  // log2 units
constexpr int kDefaultFwdEmu = 2;         // key pairs (in eighths) whose exponentials use the FMA pipe

// Optional per-phase timeline of one CTA (clock64 per event and iteration), for profiling the pipelines: off
// unless attention_set_trace() installed a buffer. Slot = event * 64 + (iteration & 63).
struct TraceCfg {
  long long* buf;
  int cta;
};
__device__ TraceCfg g_attn_trace;
// The buffer pointer is read once per CTA (trace_buffer) so that recording an event is one clock read and one
// store: reloading a __device__ variable after every asm with a memory clobber distorted the timeline.
__device__ __forceinline__ long long* trace_buffer() {
  const TraceCfg t = g_attn_trace;
  return (t.buf != nullptr && (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)) == t.cta)
             ? t.buf
             : nullptr;
}
#define ATTN_TRACE(on, ev, it)                                                  \
  do {                                                                          \
    if (on) trace_buf[(ev) * 64 + ((it) & 63)] = (long long)clock64();          \
  } while (0)

__device__ __forceinline__ float ex2(float x) {  // hardware 2^x (MUFU)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 f32x2 instructions: one issue slot for two lanes of work) and the 3-input max.
__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x of two values on the FMA pipe (relieves the MUFU unit, whose exponential rate equals the tensor core's
// consumption of probabilities at head dim 128). x = j + f with j = round(x), taken from the low mantissa bits of
// x + 1.5 * 2^23; 2^f on [-0.5, 0.5] by a degree-3 polynomial fitted here for minimum maximum relative error
// (Lawson's iteratively reweighted least squares; max relative error 7.5e-5, far below the bf16 rounding of P);
// 2^j enters as an integer add to the exponent field. Inputs are clamped to -126 (2^f >= 0.707 keeps the
// exponent field non-negative there; the result is then a denormal of at most 2^-126, where ex2.ftz gives 0).
__device__ __forceinline__ void ex2_fma2(uint64_t x2, float& ya, float& yb) {
  float xa, xb;
  f2_split(x2, xa, xb);
  const uint64_t x = f2(fmaxf(xa, -126.f), fmaxf(xb, -126.f));
  const uint64_t shifter = f2(12582912.f, 12582912.f);
  const uint64_t t = f2_add(x, shifter);
  const uint64_t f = f2_sub(x, f2_sub(t, shifter));
  uint64_t q = f2_fma(f2(0.05517143f, 0.05517143f), f, f2(0.24261081f, 0.24261081f));
  q = f2_fma(q, f, f2(0.69326097f, 0.69326097f));
  q = f2_fma(q, f, f2(0.9999281f, 0.9999281f));
  float qa, qb, ta, tb;
  f2_split(q, qa, qb);
  f2_split(t, ta, tb);
  ya = __int_as_float(__float_as_int(qa) + (__float_as_int(ta) << 23));
  yb = __int_as_float(__float_as_int(qb) + (__float_as_int(tb) << 23));
}

template <int HD>
struct FwdSmem {
  static constexpr int Q_BYTES = TQ * HD * 2;          // per Q tile: HD / 64 blocks of 128 rows x 128 B
  static constexpr int KV_BYTES = TK * HD * 2;         // HD / 64 blocks of 128 rows x 128 B
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + NQ * Q_BYTES;
  static constexpr int V_OFF = K_OFF + K_STAGES * KV_BYTES;
  static constexpr int BAR_OFF = V_OFF + V_STAGES * KV_BYTES;
  static constexpr int TOTAL = BAR_OFF + 512;
};

struct FwdBars {
  uint64_t q_full, q_empty;                        // Q tiles of the current item loaded / read by its last S
  uint64_t k_full[K_STAGES], k_empty[K_STAGES];    // K tile free once S of both Q tiles is computed
  uint64_t v_full[V_STAGES], v_empty[V_STAGES];    // V tile free once P V of both Q tiles is computed
  uint64_t s_full[NQ];                             // S_g(j) in TMEM (and, by issue order, P_g(j-1) V done)
  uint64_t p_full[NQ];                             // softmax wrote P_g(j) over S_g(j): one arrival per warp
  uint64_t pv_done[NQ];                            // one phase per P_g(j) V_j
  uint64_t o_free[NQ];                             // the epilogue read O_g of the item: 128 arrivals
  uint64_t turn[NQ];                               // ping-pong: softmax group g may run its exponentials
  uint32_t tmem_base;
  int abort_flag;
};

// One work item: two 128-row query tiles of one (batch, head); its key range and KV tile count.
struct FwdItem {
  int h, b, hk, q0, seq0, tb, q_len, kv_end, n_tiles;
};
__device__ __forceinline__ FwdItem fwd_item(const AttnParams& p, int item, int n_qb) {
  FwdItem w;
  const int qb = item % n_qb, r = item / n_qb;
  w.h = r % p.Hq;
  w.b = r / p.Hq;
  w.hk = w.h / p.rep;
  w.q0 = qb * (NQ * TQ);
  // varlen: sequence b occupies tokens [seq0, seq0 + len) of the packed axis (batch coordinate 0 of the maps)
  w.seq0 = 0;
  w.tb = w.b;
  w.q_len = p.Tq;
  w.kv_end = p.Tk;
  if (p.cu_seqlens != nullptr) {
    w.seq0 = p.cu_seqlens[w.b];
    w.q_len = w.kv_end = p.cu_seqlens[w.b + 1] - w.seq0;
    w.tb = 0;
  }
  if (p.kv_len != nullptr) w.kv_end = min(w.kv_end, p.kv_len[w.b]);
  if (p.causal) w.kv_end = min(w.kv_end, w.q0 + NQ * TQ);  // no key after the item's last query row
  if (w.q0 >= w.q_len) w.kv_end = 0;
  w.n_tiles = max(0, (w.kv_end + TK - 1) / TK);
  return w;
}

}  // namespace

// Persistent: one CTA per SM walks the work items (query block fastest, so neighbouring CTAs share K / V in L2).
// Barrier phases run on across items (a global KV-tile counter), so the TMA loads, MMAs and softmax of the next
// item start while the softmax warps still write the previous item's output: short-key items (cross-attention
// against 128 text tokens) are no longer one prologue and one epilogue per CTA.
// Schedule (one MMA-issuing thread, tensor-pipe order):  S_0(0) S_1(0) | PV_0(0) S_0(1) PV_1(0) S_1(1) | PV_0(1) ...
// S_g(j+1) is issued right after P_g(j) V_j, into the same TMEM columns: the tensor pipe runs them in order, so when
// S_g(j+1) is complete the P V that read P_g(j) is complete too. The softmax of Q tile g therefore rescales O_g and
// overwrites S_g with P_g without waiting for its own P V; while it works, the tensor core runs the other tile's
// P V and next S. Before a tcgen05.st into TMEM the softmax waits for the other tile's P V that may still be
// reading its A operand from TMEM (a tcgen05.st into TMEM lanes under an in-flight TS-MMA gave wrong products on
// B200); in the steady state that P V finished long before the exponentials do.
template <int HD, int EMU>
__global__ void __launch_bounds__(THREADS, 1)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, AttnParams p, int* err, int flags) {
  const int pingpong = flags & 1;
  const bool poll_mma = (flags & 2) != 0, poll_sm = (flags & 4) != 0, poll_ld = (flags & 8) != 0;
  using L = FwdSmem<HD>;
  static_assert(sizeof(FwdBars) <= 512, "barrier block");
  extern __shared__ __align__(1024) uint8_t smem[];
  FwdBars* bars = reinterpret_cast<FwdBars*>(smem + L::BAR_OFF);
  const int warp = warp_id(), lane = lane_id();
  if ((smem_u32(smem) & 1023) != 0) {  // the swizzled tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) record_error(err, ERR_BAD_ARGS);
    return;
  }
  const int n_qb = (p.Tq + NQ * TQ - 1) / (NQ * TQ);
  const int n_items = n_qb * p.Hq * p.B;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int i = 0; i < K_STAGES; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
    }
    for (int i = 0; i < V_STAGES; ++i) {
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
    }
    for (int g = 0; g < NQ; ++g) {
      mbar_init(&bars->s_full[g], 1);
      mbar_init(&bars->p_full[g], 4);
      mbar_init(&bars->pv_done[g], 1);
      mbar_init(&bars->o_free[g], 128);
      mbar_init(&bars->turn[g], 4);
    }
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
  long long* const trace_buf = trace_buffer();
  const bool tr = trace_buf != nullptr;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA loads: per item both Q tiles, then K_j and V_j into 2-stage rings ----------------
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      bool ok = true;
      int items = 0, gt = 0;  // non-empty items loaded, global KV tile counter
      for (int item = blockIdx.x; item < n_items && ok && !*abort_flag; item += gridDim.x) {
        const FwdItem w = fwd_item(p, item, n_qb);
        if (w.n_tiles == 0) continue;
        if (items > 0 && !mbar_wait_mode(&bars->q_empty, (items - 1) & 1, err, ERR_MBAR_TIMEOUT_PRODUCER, poll_ld)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&bars->q_full, NQ * L::Q_BYTES);
#pragma unroll
        for (int g = 0; g < NQ; ++g)
#pragma unroll
          for (int blk = 0; blk < HD / 64; ++blk)
            tma_load_4d(smem + L::Q_OFF + g * L::Q_BYTES + blk * TQ * 128, &tmQ, &bars->q_full, blk * 64,
                        w.seq0 + w.q0 + g * TQ, w.h, w.tb);
        // K_j of global tile t goes to ring slot t % K_STAGES; within an item K runs one tile ahead of V
        auto load_k = [&](int t, int jj) -> bool {
          const int st = t % K_STAGES, ph = (t / K_STAGES) & 1;
          if (!mbar_wait_mode(&bars->k_empty[st], ph ^ 1, err, ERR_MBAR_TIMEOUT_PRODUCER, poll_ld)) return false;
          mbar_expect_tx(&bars->k_full[st], L::KV_BYTES);
#pragma unroll
          for (int blk = 0; blk < HD / 64; ++blk)
            tma_load_4d(smem + L::K_OFF + st * L::KV_BYTES + blk * TK * 128, &tmK, &bars->k_full[st], blk * 64,
                        w.seq0 + jj * TK, w.hk, w.tb);
          return true;
        };
        if (!load_k(gt, 0)) {
          ok = false;
          break;
        }
        for (int j = 0; j < w.n_tiles && ok; ++j, ++gt) {
          if (j + 1 < w.n_tiles && !load_k(gt + 1, j + 1)) {
            ok = false;
            break;
          }
          const int st = gt % V_STAGES, ph = (gt / V_STAGES) & 1;
          if (!mbar_wait_mode(&bars->v_empty[st], ph ^ 1, err, ERR_MBAR_TIMEOUT_PRODUCER, poll_ld)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bars->v_full[st], L::KV_BYTES);
#pragma unroll
          for (int blk = 0; blk < HD / 64; ++blk)
            tma_load_4d(smem + L::V_OFF + st * L::KV_BYTES + blk * TK * 128, &tmV, &bars->v_full[st], blk * 64,
                        w.seq0 + j * TK, w.hk, w.tb);
        }
        ++items;
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issue ----------------
      constexpr uint32_t idesc_s = idesc_bf16_f32(TQ, TK, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(TQ, HD, false, true);
      const uint64_t q_desc0 = sdesc_sw128(smem_u32(smem + L::Q_OFF), 16, 1024);
      const uint64_t k_desc0 = sdesc_sw128(smem_u32(smem + L::K_OFF), 16, 1024);
      const uint64_t v_desc0 = sdesc_sw128(smem_u32(smem + L::V_OFF), TK * 128, 1024);
      auto issue_s = [&](int g, int gtile, bool last_s) {  // S_g = Q_g K^T into TMEM columns g * 128
        const int ks = gtile % K_STAGES;
        const uint64_t kd = sdesc_add(k_desc0, ks * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t blk = kk >> 2, sub = (kk & 3) * 32;
          umma_f16(tmem + g * 128, sdesc_add(q_desc0, g * L::Q_BYTES + blk * TQ * 128 + sub),
                   sdesc_add(kd, blk * TK * 128 + sub), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[g]);
        if (g == NQ - 1) {
          umma_commit(&bars->k_empty[ks]);        // K read by both Q tiles
          if (last_s) umma_commit(&bars->q_empty);  // the item's Q tiles are read for the last time
        }
      };
      bool ok = true;
      int items = 0, gt = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const FwdItem w = fwd_item(p, item, n_qb);
        const int n = w.n_tiles;
        if (n == 0) continue;
        ok = mbar_wait_mode(&bars->q_full, items & 1, err, ERR_MBAR_TIMEOUT_MMA, poll_mma) &&
             mbar_wait_mode(&bars->k_full[gt % K_STAGES], (gt / K_STAGES) & 1, err, ERR_MBAR_TIMEOUT_MMA, poll_mma);
        if (!ok) break;
        tc_fence_after();
        issue_s(0, gt, false);  // after the previous item's last P_0 V in tensor-pipe order (same TMEM columns)
        issue_s(1, gt, n == 1);
        ATTN_TRACE(tr, 20, gt);
        for (int j = 0; j < n && ok; ++j) {
          const int gj = gt + j;
          const int vs = gj % V_STAGES, vph = (gj / V_STAGES) & 1;
          const int kn = (gj + 1) % K_STAGES, knph = ((gj + 1) / K_STAGES) & 1;
          if (!mbar_wait_mode(&bars->v_full[vs], vph, err, ERR_MBAR_TIMEOUT_MMA, poll_mma)) {
            ok = false;
            break;
          }
          const uint64_t vd = sdesc_add(v_desc0, vs * L::KV_BYTES);
#pragma unroll
          for (int g = 0; g < NQ && ok; ++g) {
            if (!mbar_wait_mode(&bars->p_full[g], gj & 1, err, ERR_MBAR_TIMEOUT_MMA, poll_mma)) {
              ok = false;
              break;
            }
            // the first P V of an item overwrites O_g: the previous item's epilogue must have read it
            if (j == 0 && items > 0 &&
                !mbar_wait_mode(&bars->o_free[g], (items - 1) & 1, err, ERR_MBAR_TIMEOUT_MMA, poll_mma)) {
              ok = false;
              break;
            }
            ATTN_TRACE(tr, 21 + g, gj);
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < TK / 16; ++kk)  // O_g += P_g V_j, P read from TMEM (8 columns per 16 keys)
              umma_f16_tmem_a(tmem + O_COL + g * HD, tmem + g * 128 + kk * 8, sdesc_add(vd, kk * 2048), idesc_o,
                              (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&bars->pv_done[g]);
            if (g == NQ - 1) umma_commit(&bars->v_empty[vs]);  // V_j read by both Q tiles
            if (j + 1 < n) {
              if (g == 0 && !mbar_wait_mode(&bars->k_full[kn], knph, err, ERR_MBAR_TIMEOUT_MMA, poll_mma)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_s(g, gj + 1, j + 2 == n);  // same TMEM columns as P_g(j): after the P V above in pipe order
            }
          }
          ATTN_TRACE(tr, 20, gj + 1);
        }
        gt += n;
        ++items;
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- softmax / epilogue of Q tile g ----------------
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;         // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;  // TMEM lane == query row within the tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_base = tmem + lane_base + g * 128;
    const uint32_t o_base = tmem + lane_base + O_COL + g * HD;
    const float sl2 = p.scale * 1.4426950408889634f;
    const bool tw = tr && (threadIdx.x == 64 + g * 128);
    const bool tw4 = tr && threadIdx.x == 128, tw5 = tr && threadIdx.x == 160;  // the other SMSPs' warps of tile 0
    bool ok = true;
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
      int w_ok = 1;
      if (lane == 0) w_ok = mbar_wait_mode(bar, parity, err, ERR_MBAR_TIMEOUT_EPILOGUE, poll_sm) ? 1 : 0;
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
      __syncwarp();
      return w_ok != 0;
    };
    // output row of this thread for an item (recomputed where needed: fewer live registers in the tile loop)
    auto out_row = [&](const FwdItem& w, int qpos) {
      return p.o + (long long)w.tb * p.o_bs + (long long)(w.seq0 + qpos) * p.o_ts + (long long)w.h * p.o_hs;
    };
    auto lse_index = [&](const FwdItem& w, int qpos) {
      return p.cu_seqlens != nullptr ? (long long)w.h * p.total + w.seq0 + qpos
                                     : ((long long)w.b * p.Hq + w.h) * p.Tq + qpos;
    };
    int gt = 0;
    // Ping-pong (optional): the two softmax groups take turns for their exponential phases (turn[g] completes when
    // the other group finished its phase; group 1 hands group 0 the first turn), so each phase runs with the MUFU
    // and issue slots of its SM sub-partitions to itself instead of interleaved with the other group's.
    int turns = 0;
    if (pingpong && g == 1 && lane == 0) mbar_arrive(&bars->turn[0]);
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      int n, key_lim;
      {
        const FwdItem w = fwd_item(p, item, n_qb);
        n = w.n_tiles;
        const int qpos = w.q0 + g * TQ + row;                       // query index within the sequence
        key_lim = p.causal ? min(w.kv_end, qpos + 1) : w.kv_end;    // this row's keys: [0, key_lim)
        if (n == 0) {  // no keys (kv_len 0): zero rows; no barrier takes part
          if (qpos < w.q_len) {
            __nv_bfloat16* dst = out_row(w, qpos);
            for (int c = 0; c < HD; c += 8) *reinterpret_cast<uint4*>(dst + c) = make_uint4(0u, 0u, 0u, 0u);
            if (p.lse != nullptr) p.lse[lse_index(w, qpos)] = INFINITY;
          }
          continue;
        }
      }
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        const int gj = gt + j;
        if (!warp_wait(&bars->s_full[g], gj & 1)) {
          ok = false;
          break;
        }
        ATTN_TRACE(tw, 23 + 4 * g, gj);
        tc_fence_after();
        // raw logits: the running max m is kept in log2 units (sl2 > 0, so max and scaling commute) and
        // p = 2^(s sl2 - m) is one FFMA + ex2 per element; keys past key_lim exist only in the last tile (and,
        // when causal, in the tiles that cross the diagonal). The four TMEM loads of the row are issued together
        // (one wait: a tcgen05.ld round trip is long while the tensor core works on TMEM), and P is packed in
        // place over the consumed S registers (element pair e of a chunk -> register e).
        const int kbase = j * TK;
        const bool full_tile = kbase + TK <= key_lim;
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(s_base + c * 32, sr[c]);
        tmem_ld_wait();
        ATTN_TRACE(tw, 24 + 4 * g, gj);
        if (!full_tile) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (kbase + c * 32 + i >= key_lim) sr[c][i] = __float_as_uint(-INFINITY);
        }
        float mx[4];  // 3-input max, 4 partial maxima (short dependency chains), then a tree
#pragma unroll
        for (int k = 0; k < 4; ++k) mx[k] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; i += 2)
            mx[(i >> 1) & 3] = max3(mx[(i >> 1) & 3], __uint_as_float(sr[c][i]), __uint_as_float(sr[c][i + 1]));
        const float smax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl2;
        const float m_new = fmaxf(m, smax);
        const bool rescale = (j > 0) && (m_new > m + kRescaleThreshold);
        const float corr = rescale ? ((m == -INFINITY) ? 0.f : ex2(m - m_new)) : 1.f;
        if (rescale || j == 0) m = m_new;
        const float mu = (m == -INFINITY) ? 0.f : m;
        // per key pair: one packed FMA (scale, subtract the max), two exponentials (MUFU, or the FMA-pipe
        // polynomial for EMU of every 8 pairs), one packed add into the row sum, one bf16x2 pack
        if (pingpong) {
          if (!warp_wait(&bars->turn[g], turns & 1)) {
            ok = false;
            break;
          }
          ++turns;
        }
        const uint64_t sl2x2 = f2(sl2, sl2), nmu2 = f2(-mu, -mu);
        uint64_t rs2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const uint64_t x2 = f2_fma(f2(__uint_as_float(sr[c][2 * e]), __uint_as_float(sr[c][2 * e + 1])),
                                       sl2x2, nmu2);
            float a, bq;
            if ((e & 7) >= 8 - EMU) {
              ex2_fma2(x2, a, bq);
            } else {
              float xa, xb;
              f2_split(x2, xa, xb);
              a = ex2(xa);
              bq = ex2(xb);
            }
            rs2[e & 1] = f2_add(rs2[e & 1], f2(a, bq));
            sr[c][e] = pack_bf16x2(a, bq);  // e <= 2e: the pair was read above
          }
        }
        float r0, r1, r2, r3;
        f2_split(rs2[0], r0, r1);
        f2_split(rs2[1], r2, r3);
        l = l * corr + ((r0 + r1) + (r2 + r3));
        if (pingpong) {  // hand the exponential unit to the other group
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->turn[1 - g]);
        }
        ATTN_TRACE(tw, 25 + 4 * g, gj);
        ATTN_TRACE(tw5, 16, gj);
        // the other Q tile's P V may still read its A operand from TMEM: let it finish before any tcgen05.st here
        // (tile 0 waits for the P_1 V of the previous KV tile, tile 1 for the P_0 V of this one; the later P V of
        // that tile cannot start before this tile's P is written, so the barrier cannot be a phase ahead)
        const int oj = (g == 0) ? gj - 1 : gj;
        if (oj >= 0 && !warp_wait(&bars->pv_done[1 - g], oj & 1)) {
          ok = false;
          break;
        }
        ATTN_TRACE(tw, 17 + g, gj);
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
          // O_g is stable: P_g(j-1) V completed before S_g(j) (tensor-pipe order), P_g(j) V is not issued yet
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(o_base + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
            tmem_st_32x32b_x32(o_base + c * 32, o);
          }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)  // P_g(j): 128 keys as bf16 pairs, chunk c in columns c * 16 .. + 15
          tmem_st_32x32b_x16(s_base + c * 16, *reinterpret_cast<const uint32_t(*)[16]>(&sr[c][0]));
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        ATTN_TRACE(tw, 26 + 4 * g, gj);
        ATTN_TRACE(tw5, 19, gj);
        ATTN_TRACE(tw4, 31, gj);
        if (lane == 0) mbar_arrive(&bars->p_full[g]);  // one arrival per warp, after its stores completed
      }
      if (!ok) break;
      // epilogue: O / l -> bf16, log-sum-exp; then O_g is released to the next item's first P V
      if (!warp_wait(&bars->pv_done[g], (gt + n - 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      const FwdItem w = fwd_item(p, item, n_qb);
      const int qpos = w.q0 + g * TQ + row;
      __nv_bfloat16* dst = out_row(w, qpos);
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(o_base + c * 32, o);
        tmem_ld_wait();
        if (qpos < w.q_len) {
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
      tc_fence_before();
      mbar_arrive(&bars->o_free[g]);
      if (qpos < w.q_len && p.lse != nullptr)
        p.lse[lse_index(w, qpos)] = (l > 0.f) ? (m + log2f(l)) * 0.6931471805599453f : INFINITY;
      gt += n;
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

static int g_fwd_pingpong = 0;  // softmax groups alternate their exponential phases
// barrier waits that poll (test_wait) instead of suspending: bit 0 the MMA thread, bit 1 the softmax / drain
// warps, bit 2 the TMA producer
static int g_attn_poll_fwd = 3, g_attn_poll_bwd = 1;

template <int HD, int EMU>
static cudaError_t fwd_tc_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                               const AttnParams& p, int* err, cudaStream_t s) {
  using L = FwdSmem<HD>;
  static_assert(L::TOTAL <= 232448, "shared memory");
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(flash_fwd_tc_kernel<HD, EMU>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
    set = true;
  }
  const long long items = (long long)((p.Tq + NQ * TQ - 1) / (NQ * TQ)) * p.Hq * p.B;
  if (items <= 0) return cudaSuccess;
  if (items >= (1ll << 31)) return cudaErrorInvalidValue;
  const int grid = (int)std::min<long long>(items, num_sms());
  flash_fwd_tc_kernel<HD, EMU><<<grid, THREADS, L::TOTAL, s>>>(tq, tk, tv, p, err,
                                                                g_fwd_pingpong | (g_attn_poll_fwd << 1));
  return cudaGetLastError();
}

// Exponentials computed on the FMA pipe, in eighths of the key pairs (0: all on the MUFU unit).
static int g_fwd_emu = kDefaultFwdEmu;

cudaError_t attention_set_fwd_split(int wpq) { return wpq == 1 ? cudaSuccess : cudaErrorInvalidValue; }

cudaError_t attention_set_fwd_pingpong(int on) {
  g_fwd_pingpong = on ? 1 : 0;
  return cudaSuccess;
}

cudaError_t attention_set_fwd_emu(int eighths) {  // -1: the built-in default
  if (eighths == -1) eighths = kDefaultFwdEmu;
  if (eighths < 0 || eighths > 4) return cudaErrorInvalidValue;
  g_fwd_emu = eighths;
  return cudaSuccess;
}

template <int HD>
static cudaError_t fwd_tc_dispatch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                   const AttnParams& p, int* err, cudaStream_t s) {
  switch (g_fwd_emu) {
    case 1: return fwd_tc_impl<HD, 1>(tq, tk, tv, p, err, s);
    case 2: return fwd_tc_impl<HD, 2>(tq, tk, tv, p, err, s);
    case 3: return fwd_tc_impl<HD, 3>(tq, tk, tv, p, err, s);
    case 4: return fwd_tc_impl<HD, 4>(tq, tk, tv, p, err, s);
    default: return fwd_tc_impl<HD, 0>(tq, tk, tv, p, err, s);
  }
}

cudaError_t attention_fwd_tc_launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                    const AttnParams& p, int* err, cudaStream_t s) {
  if (p.hd == 128) return fwd_tc_dispatch<128>(tq, tk, tv, p, err, s);
  if (p.hd == 64) return fwd_tc_dispatch<64>(tq, tk, tv, p, err, s);
  return cudaErrorInvalidValue;
}


// ==================================================================================================================
// Backward on tcgen05 (head dim 128).
//
// CTA = 128 keys of one (batch, kv head); loops over the rep query heads of the group and over query tiles of 64.
// Per iteration (Q_i, dO_i: 64 queries):
//   MMA1  S^T  = K Q_i^T          M 128 keys, N 64, K 128      TMEM cols   0 ..  63
//   MMA2  dP^T = V dO_i^T         M 128 keys, N 64, K 128      TMEM cols  64 .. 127
//   softmax warps (thread = key): P^T = 2^(S^T scale log2e - lse log2e) -> bf16 pairs into TMEM (cols 192 + 32 b),
//                                 dS^T = P^T (dP^T - delta) -> bf16 K-major shared tile (double buffered)
//   MMA3  dV  += P^T dO_i         M 128 keys, N 128, K 64      A from TMEM, TMEM cols 256 .. 383
//   MMA4  dK  += dS^T Q_i         M 128 keys, N 128, K 64      TMEM cols 384 .. 511
//   MMA5  dQ^T = K^T dS^T         M 128 (head dim), N 64, K 128 keys   TMEM cols 128 .. 191
//   dQ warps (thread = head-dim lane): dQ^T -> scale -> fp32 [query][head dim] shared tiles -> TMA reduce-add into
//                                      the fp32 dQ accumulator (cp.reduce.async.bulk.tensor, two 32-query halves)
// Q / dO tiles (and the tile's lse / delta rows, bulk-copied) stream through a 3-stage ring released by MMA3-5, so the
// loads run two iterations ahead. The softmax of iteration i+1 overlaps MMA3-5 of iteration i, except for its
// P^T store, which waits for them (a tcgen05.st into the TMEM lanes that an in-flight MMA reads its A operand from
// gave wrong products on B200; see the forward kernel). MMA1/2 of iteration i+1 are issued before MMA3-5 of i.
// Warps: 0 TMA, 1 MMA (+ TMEM), 2-9 softmax (two warps per TMEM lane quarter, 32 queries each) + final dV / dK,
// 10-13 dQ drain. The softmax reads lse in base-2 units (lse2 = lse log2 e, written by the delta kernel).
// ==================================================================================================================
namespace {

constexpr int BK_KEYS = 128;
constexpr int BQ = 64;
constexpr int BWD_THREADS = 448;  // warp 0 TMA, 1 MMA, 2-9 softmax (two per TMEM lane quarter), 10-13 dQ
constexpr int QST = 3;  // Q / dO ring stages

struct BwdSmem {  // head dim 128
  static constexpr int K_OFF = 0;                              // 2 blocks x 128 rows x 128 B
  static constexpr int V_OFF = K_OFF + 32768;
  static constexpr int Q_OFF = V_OFF + 32768;                  // QST stages x (2 blocks x 64 rows x 128 B)
  static constexpr int DO_OFF = Q_OFF + QST * 16384;
  static constexpr int DS_OFF = DO_OFF + QST * 16384;          // 2 buffers x 128 rows x 128 B
  static constexpr int DQ_OFF = DS_OFF + 2 * 16384;            // 2 halves x 32 queries x 128 fp32
  static constexpr int STAT_OFF = DQ_OFF + 32768;              // QST slots x (lse[64], delta[64]) fp32
  static constexpr int BAR_OFF = STAT_OFF + QST * 512;
  static constexpr int TOTAL = BAR_OFF + 256;
};

struct BwdBars {
  uint64_t kv_full;
  uint64_t q_full[QST];
  uint64_t q_empty[QST];
  uint64_t s_full;
  uint64_t s_empty;
  uint64_t p_full;      // softmax wrote P^T (TMEM) and dS^T (shared): 128 arrivals
  uint64_t mma_done;    // MMA3-5 of an iteration completed (one phase per iteration)
  uint64_t dq_full;
  uint64_t dq_empty;
  uint64_t acc_done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void softmax_group_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ void drain_group_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code, bool poll) {
  int ok = 1;
  if (lane_id() == 0) ok = mbar_wait_mode(bar, parity, err, code, poll) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

}  // namespace

__global__ void __launch_bounds__(BWD_THREADS, 1)
    flash_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                        const __grid_constant__ CUtensorMap tmdQ, AttnParams p, const float* __restrict__ delta,
                        const float* __restrict__ lse2, __nv_bfloat16* __restrict__ dk, long long dk_bs, long long dk_ts, long long dk_hs,
                        __nv_bfloat16* __restrict__ dv, long long dv_bs, long long dv_ts, long long dv_hs, int* err,
                        int flags, int dq_mode) {
  constexpr int HD = 128;
  const bool poll_mma = (flags & 2) != 0, poll_sm = (flags & 4) != 0, poll_ld = (flags & 8) != 0;
  using L = BwdSmem;
  static_assert(L::TOTAL <= 232448, "shared memory");
  extern __shared__ __align__(1024) uint8_t smem[];
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + L::BAR_OFF);
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
  const bool bulk_stats = (p.Tq % 4) == 0;  // 16-byte aligned rows: lse / delta arrive with the Q tile

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    for (int i = 0; i < QST; ++i) {
      mbar_init(&bars->q_full[i], 1);
      mbar_init(&bars->q_empty[i], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->s_empty, 256);
    mbar_init(&bars->p_full, 256);
    mbar_init(&bars->mma_done, 1);
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
  long long* const trace_buf = trace_buffer();
  const bool tr = trace_buf != nullptr;

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
        const int st = i % QST;
        const int h = hk * p.rep + i / n_qt, q0 = (i % n_qt) * BQ;
        if (!mbar_wait_mode(&bars->q_empty[st], ((i / QST) & 1) ^ 1, err, ERR_MBAR_TIMEOUT_PRODUCER, poll_ld)) {
          *abort_flag = 1;
          break;
        }
        ATTN_TRACE(tr, 0, i);
        const int nq = min(BQ, p.Tq - q0);
        const uint32_t stat_bytes = bulk_stats ? (uint32_t)nq * 4u : 0u;
        mbar_expect_tx(&bars->q_full[st], 2 * 16384 + 2 * stat_bytes);
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          tma_load_4d(smem + L::Q_OFF + st * 16384 + blk * 8192, &tmQ, &bars->q_full[st], blk * 64, q0, h, b);
          tma_load_4d(smem + L::DO_OFF + st * 16384 + blk * 8192, &tmdO, &bars->q_full[st], blk * 64, q0, h, b);
        }
        if (bulk_stats) {
          const long long row = ((long long)b * p.Hq + h) * p.Tq + q0;
          bulk_load(smem + L::STAT_OFF + st * 512, lse2 + row, stat_bytes, &bars->q_full[st]);
          bulk_load(smem + L::STAT_OFF + st * 512 + 256, delta + row, stat_bytes, &bars->q_full[st]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      // ---------------- MMA issue ----------------
      constexpr uint32_t id_s = idesc_bf16_f32(128, BQ, false, false);   // S^T, dP^T
      constexpr uint32_t id_kv = idesc_bf16_f32(128, HD, false, true);   // dV, dK
      constexpr uint32_t id_q = idesc_bf16_f32(128, BQ, true, true);     // dQ^T
      // precomputed descriptors; stage and k offsets are added per MMA
      const uint64_t dK_km = sdesc_sw128(smem_u32(smem + L::K_OFF), 16, 1024);      // K as K-major A (S^T)
      const uint64_t dV_km = sdesc_sw128(smem_u32(smem + L::V_OFF), 16, 1024);      // V as K-major A (dP^T)
      const uint64_t dK_mn = sdesc_sw128(smem_u32(smem + L::K_OFF), 16384, 1024);   // K as MN-major A (dQ^T)
      const uint64_t dQ_km = sdesc_sw128(smem_u32(smem + L::Q_OFF), 16, 1024);      // Q as K-major B (S^T)
      const uint64_t dQ_mn = sdesc_sw128(smem_u32(smem + L::Q_OFF), 8192, 1024);   // Q as MN-major B (dK)
      const uint64_t dO_km = sdesc_sw128(smem_u32(smem + L::DO_OFF), 16, 1024);     // dO as K-major B (dP^T)
      const uint64_t dO_mn = sdesc_sw128(smem_u32(smem + L::DO_OFF), 8192, 1024);   // dO as MN-major B (dV)
      const uint64_t dS_km = sdesc_sw128(smem_u32(smem + L::DS_OFF), 16, 1024);     // dS^T as K-major A (dK)
      const uint64_t dS_mn = sdesc_sw128(smem_u32(smem + L::DS_OFF), 8192, 1024);   // dS^T as MN-major B (dQ^T)
      auto issue_s = [&](int i) -> bool {
        const int st = i % QST;
        if (!mbar_wait_mode(&bars->q_full[st], (i / QST) & 1, err, ERR_MBAR_TIMEOUT_MMA, poll_mma)) return false;
        ATTN_TRACE(tr, 2, i);
        if (i > 0 && !mbar_wait_mode(&bars->s_empty, (i - 1) & 1, err, ERR_MBAR_TIMEOUT_MMA, poll_mma)) return false;
        ATTN_TRACE(tr, 3, i);
        tc_fence_after();
        const uint32_t so = st * 16384;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t blk = kk >> 2, sub = (kk & 3) * 32;
          umma_f16(tmem + 0, sdesc_add(dK_km, blk * 16384 + sub), sdesc_add(dQ_km, so + blk * 8192 + sub), id_s,
                   kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t blk = kk >> 2, sub = (kk & 3) * 32;
          umma_f16(tmem + 64, sdesc_add(dV_km, blk * 16384 + sub), sdesc_add(dO_km, so + blk * 8192 + sub), id_s,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full);
        ATTN_TRACE(tr, 4, i);
        return true;
      };
      bool ok = mbar_wait_mode(&bars->kv_full, 0, err, ERR_MBAR_TIMEOUT_MMA, poll_mma) && issue_s(0);
      for (int i = 0; i < n_it && ok; ++i) {
        const int st = i % QST, pb = i & 1;
        if (i + 1 < n_it && !issue_s(i + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait_mode(&bars->p_full, i & 1, err, ERR_MBAR_TIMEOUT_MMA, poll_mma)) {
          ok = false;
          break;
        }
        ATTN_TRACE(tr, 5, i);
        tc_fence_after();
        const uint32_t so = st * 16384, dso = pb * 16384;
        // dV and dK need only this iteration's P^T / dS^T: they run while the dQ drain may still read dQ^T(i-1)
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dV += P^T dO, P^T read from TMEM (8 columns per 16 queries)
          umma_f16_tmem_a(tmem + 256, tmem + 192 + pb * 32 + kk * 8, sdesc_add(dO_mn, so + kk * 2048), id_kv,
                          (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dK += dS^T Q
          umma_f16(tmem + 384, sdesc_add(dS_km, dso + kk * 32), sdesc_add(dQ_mn, so + kk * 2048), id_kv,
                   (i > 0 || kk > 0) ? 1u : 0u);
        if (!mbar_wait_mode(&bars->dq_empty, (i & 1) ^ 1, err, ERR_MBAR_TIMEOUT_MMA, poll_mma)) {
          ok = false;
          break;
        }
        ATTN_TRACE(tr, 6, i);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BK_KEYS / 16; ++kk)  // dQ^T = K^T dS^T
          umma_f16(tmem + 128, sdesc_add(dK_mn, kk * 2048), sdesc_add(dS_mn, dso + kk * 2048), id_q,
                   kk > 0 ? 1u : 0u);
        umma_commit(&bars->q_empty[st]);
        umma_commit(&bars->mma_done);
        umma_commit(&bars->dq_full);
        ATTN_TRACE(tr, 7, i);
      }
      if (ok) umma_commit(&bars->acc_done);
      else *abort_flag = 1;
    }
  } else if (warp < 10) {
    // ---------------- softmax (thread = key row, one half of the 64 queries), final dV (half 0) / dK (half 1) ----
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const int tid = threadIdx.x - 64;  // 0..255
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale * 1.4426950408889634f;
    const bool key_ok = k0 + r < kv_end;
    const bool tw = tr && threadIdx.x == 64;
    bool ok = true;
    for (int i = 0; i < n_it; ++i) {
      const int st = i % QST, pb = i & 1;
      const int h = hk * p.rep + i / n_qt, q0 = (i % n_qt) * BQ;
      const int nq = min(BQ, p.Tq - q0);
      float* slot = reinterpret_cast<float*>(smem + L::STAT_OFF + st * 512);  // lse * log2 e [64], delta [64]
      if (!bulk_stats) {  // staged by the threads; out-of-range queries get P = 0
        if (tid < 128) {
          const int q = tid & 63;
          const bool in = q < nq;
          const long long idx = ((long long)b * p.Hq + h) * p.Tq + q0 + q;
          if (tid < 64) slot[q] = in ? lse2[idx] : INFINITY;
          else slot[64 + q] = in ? delta[idx] : 0.f;
        }
        softmax_group_sync();
      } else {
        if (!warp_wait(&bars->q_full[st], (i / QST) & 1, err, ERR_MBAR_TIMEOUT_EPILOGUE, poll_sm)) {
          ok = false;  // the bulk-copied rows of this stage have landed
          break;
        }
        if (nq < BQ) {  // tail tile: pad the rows past the end
          if (tid < BQ - nq) {
            slot[nq + tid] = INFINITY;
            slot[64 + nq + tid] = 0.f;
          }
          softmax_group_sync();
        }
      }
      ATTN_TRACE(tw, 8, i);
      if (!warp_wait(&bars->s_full, i & 1, err, ERR_MBAR_TIMEOUT_EPILOGUE, poll_sm)) {
        ok = false;
        break;
      }
      ATTN_TRACE(tw, 9, i);
      tc_fence_after();
      uint32_t sv[32], dp[32];
      tmem_ld_32x32b_x32(tmem + lane_base + half * 32, sv);
      tmem_ld_32x32b_x32(tmem + lane_base + 64 + half * 32, dp);
      tmem_ld_wait();
      ATTN_TRACE(tw, 10, i);
      tc_fence_before();
      mbar_arrive(&bars->s_empty);
      // P^T and dS^T of this thread's 32 queries, packed in registers before waiting for the previous MMA3-5
      uint32_t pk[16], dk4[16];
      const float* ls = slot + half * 32;
      const float* dl = slot + 64 + half * 32;
      if (key_ok) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = ex2(__uint_as_float(sv[2 * e]) * sl2 - ls[2 * e]);
          const float p1 = ex2(__uint_as_float(sv[2 * e + 1]) * sl2 - ls[2 * e + 1]);
          pk[e] = pack_bf16x2(p0, p1);
          dk4[e] = pack_bf16x2(p0 * (__uint_as_float(dp[2 * e]) - dl[2 * e]),
                               p1 * (__uint_as_float(dp[2 * e + 1]) - dl[2 * e + 1]));
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = dk4[e] = 0u;
      }
      // MMA3-5 of iteration i-1 must be done: they read this dS^T buffer's other use and the P^T TMEM lanes
      if (i > 0 && !warp_wait(&bars->mma_done, (i - 1) & 1, err, ERR_MBAR_TIMEOUT_EPILOGUE, poll_sm)) {
        ok = false;
        break;
      }
      ATTN_TRACE(tw, 11, i);
      tc_fence_after();
      uint8_t* ds_row = smem + L::DS_OFF + pb * 16384 + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int chunk = half * 4 + c;
        *reinterpret_cast<uint4*>(ds_row + ((chunk ^ (r & 7)) << 4)) =
            make_uint4(dk4[4 * c], dk4[4 * c + 1], dk4[4 * c + 2], dk4[4 * c + 3]);
      }
      tmem_st_32x32b_x16(tmem + lane_base + 192 + pb * 32 + half * 16, pk);
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      ATTN_TRACE(tw, 12, i);
      mbar_arrive(&bars->p_full);
    }
    if (ok && n_it > 0) ok = warp_wait(&bars->acc_done, 0, err, ERR_MBAR_TIMEOUT_EPILOGUE, poll_sm);
    tc_fence_after();
    const int key = k0 + r;
    if (ok) {
      const int which = half;  // 0: dV, 1: dK (scaled)
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
    } else {
      *abort_flag = 1;
    }
  } else {
    // ---------------- dQ drain (thread = head-dim lane): TMEM -> shared fp32 tile -> TMA reduce-add ----------------
    const int quarter = warp & 3;
    const int d = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const bool leader = threadIdx.x == 320;
    float* stage = reinterpret_cast<float*>(smem + L::DQ_OFF);  // [2 halves][32 queries][128]
    if (dq_mode != 0 && !active && kb == 0) {
      // stored dQ and no key for this sample (kv_len 0): nothing else writes its rows, so they are stored as zeros
      for (int i = threadIdx.x - 320; i < 2 * 32 * HD; i += 128) stage[i] = 0.f;
      fence_proxy_async_smem();
      drain_group_sync();
      if (leader) {
        for (int i = 0; i < p.rep * n_qt; ++i) {
          const int h = hk * p.rep + i / n_qt, q0 = (i % n_qt) * BQ;
          for (int half = 0; half < 2 && q0 + half * 32 < p.Tq; ++half) {
            tma_store_4d(&tmdQ, stage + half * 32 * HD, 0, h, q0 + half * 32, b);
            bulk_commit_group();
          }
        }
      }
    }
    for (int i = 0; i < n_it; ++i) {
      const int h = hk * p.rep + i / n_qt, q0 = (i % n_qt) * BQ;
      if (!warp_wait(&bars->dq_full, i & 1, err, ERR_MBAR_TIMEOUT_EPILOGUE, poll_sm)) {
        *abort_flag = 1;
        break;
      }
      ATTN_TRACE(tr && leader, 13, i);
      tc_fence_after();
      uint32_t v[2][32];
      tmem_ld_32x32b_x32(tmem + lane_base + 128, v[0]);
      tmem_ld_32x32b_x32(tmem + lane_base + 160, v[1]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&bars->dq_empty);
      ATTN_TRACE(tr && leader, 14, i);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        if (q0 + half * 32 >= p.Tq) break;
        if (leader) bulk_wait_group_read<1>();  // this half's reduce from the previous iteration has read smem
        drain_group_sync();
        if (dq_mode == 2) {  // the only key block: dQ stored as bf16, [32 queries][128] tile
          __nv_bfloat16* dstb = reinterpret_cast<__nv_bfloat16*>(stage) + half * 32 * HD + d;
#pragma unroll
          for (int q = 0; q < 32; ++q) dstb[q * HD] = __float2bfloat16_rn(__uint_as_float(v[half][q]) * p.scale);
        } else {
          float* dst = stage + half * 32 * HD + d;
#pragma unroll
          for (int q = 0; q < 32; ++q) dst[q * HD] = __uint_as_float(v[half][q]) * p.scale;
        }
        fence_proxy_async_smem();
        drain_group_sync();
        if (leader) {
          if (dq_mode == 0) {
            tma_reduce_add_4d(&tmdQ, stage + half * 32 * HD, 0, h, q0 + half * 32, b);
          } else {
            const void* src = dq_mode == 2 ? static_cast<const void*>(reinterpret_cast<__nv_bfloat16*>(stage) +
                                                                      half * 32 * HD)
                                           : static_cast<const void*>(stage + half * 32 * HD);
            tma_store_4d(&tmdQ, src, 0, h, q0 + half * 32, b);
          }
          bulk_commit_group();
        }
      }
      ATTN_TRACE(tr && leader, 15, i);
    }
    if (leader) bulk_wait_group_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

cudaError_t attention_set_poll(int fwd_mask, int bwd_mask) {
  if (fwd_mask < 0 || fwd_mask > 7 || bwd_mask < 0 || bwd_mask > 7) return cudaErrorInvalidValue;
  g_attn_poll_fwd = fwd_mask;
  g_attn_poll_bwd = bwd_mask;
  return cudaSuccess;
}

cudaError_t attention_set_trace(long long* buf, int cta) {
  TraceCfg t{buf, cta};
  return cudaMemcpyToSymbol(g_attn_trace, &t, sizeof(t));
}

cudaError_t attention_bwd_tc_launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                    const CUtensorMap& tdo, const CUtensorMap& tdq, const AttnParams& p,
                                    const float* delta, const float* lse2, __nv_bfloat16* dk, long long dk_bs,
                                    long long dk_ts,
                                    long long dk_hs, __nv_bfloat16* dv, long long dv_bs, long long dv_ts,
                                    long long dv_hs, int* err, cudaStream_t s, int dq_mode) {
  if (p.hd != 128) return cudaErrorInvalidValue;
  // dq_mode 1 / 2 store the dQ tile (fp32 / bf16) instead of reduce-adding it: only when one key block covers every key
  if (dq_mode < 0 || dq_mode > 2 || (dq_mode != 0 && p.Tk > BK_KEYS)) return cudaErrorInvalidValue;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(flash_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdSmem::TOTAL);
    set = true;
  }
  dim3 grid((p.Tk + BK_KEYS - 1) / BK_KEYS, p.Hkv, p.B);
  flash_bwd_tc_kernel<<<grid, BWD_THREADS, BwdSmem::TOTAL, s>>>(tq, tk, tv, tdo, tdq, p, delta, lse2, dk, dk_bs,
                                                               dk_ts, dk_hs, dv, dv_bs, dv_ts, dv_hs, err,
                                                               g_attn_poll_bwd << 1, dq_mode);
  return cudaGetLastError();
}

}  // namespace tgo
