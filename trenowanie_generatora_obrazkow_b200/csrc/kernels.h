// Launch interfaces of the sm_100a kernels.  Plain CUDA types only: the torch-facing argument checks live in
// ops.cpp, so the .cu files compile without the torch headers.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tgo {

int num_sms();

constexpr int kMaxPeers = 8;

// ---------------------------------------------------------------- GEMM (gemm.cu)
// Expert-parallel MoE exchange inside the GEMM (all zero: off). The A rows of every batch come from the source
// ranks in blocks of src_rows (a multiple of the 128-row tile): with `arrive`, the producer waits until
// arrive[s] == epoch before loading an A tile of source s (the rows were stored into this GPU by the source's
// dispatch kernel). With `out`, the epilogue stores row m of batch b into source s = m / src_rows at
// out[s] + ((b_base + b) * src_rows + m % src_rows) * ldc (that source's [experts, src_rows, N] combine buffer),
// counts its finished tile warps in done_count[s] (local, zeroed before the launch) and the warp that completes
// source s sets *done_flag[s] = epoch there.
struct GemmPeer {
  int src_rows;
  uint32_t epoch;
  const uint32_t* arrive;
  __nv_bfloat16* out[kMaxPeers];
  int b_base;
  unsigned* done_count;
  uint32_t* done_flag[kMaxPeers];
  unsigned tile_warps_per_src;
  unsigned long long timeout_ns;
};
struct GemmParams {
  int M, N, K, batch;
  void* C;
  long long ldc, bsc;  // elements
  const __nv_bfloat16* D;
  long long ldd, bsd;
  float alpha, beta;
  int* err;
  GemmPeer peer;
  int c_tma;  // 1: the kernel writes C through the tensor map it is given (TMA store / reduce-add)
  // grouped mode (gemm_grouped_launch): A rows [offsets[g], offsets[g + 1]) use B batch g; C rows as A's
  const int* group_offsets;            // device [batch + 1], batch = groups (<= kMaxGroups)
  const float* row_scale;              // optional [M]: output row r scaled by row_scale[r]
  const float* col_scale;              // int8 GEMM (EPI_I8): output column n scaled by col_scale[n]
  // symmetric product (2-CTA kernel, bf16 C through its tensor map, M == N, A and B the same operand): only the
  // 256-row tile blocks on or below the diagonal are computed; each off-diagonal tile is stored twice (as itself
  // and transposed). Valid when alpha A B^T + beta D is symmetric (D symmetric or absent).
  int syrk;
  // split-K (2-CTA kernel, fp32 accumulate through the TMA reduce-add epilogue only): each output tile is computed
  // as `splitk` partial products over consecutive K ranges, all reduce-added into C (atomic in L2)
  int splitk;
  // barrier waits that poll (test_wait) instead of suspending: bit 0 the MMA thread, bit 1 the epilogue, bit 2 the
  // TMA producer (set by the launchers from gemm_set_poll)
  int poll;
  // 2-CTA kernel: how many of the last tiles run as two 256 x 128 halves (set by its launcher; 0 = none)
  int tail_tiles;
};
cudaError_t gemm_set_tail_split(int on);
constexpr int kMaxGroups = 256;
cudaError_t gemm_set_poll(int mask);
// epi: 0 = bf16 store, 1 = fp32 store, 2 = fp32 accumulate (C += alpha * A B^T)
// tc: tensor map of C ({N, M, batch}, box {32, 32, 1}; bf16 with 64-byte or fp32 with 128-byte swizzle) for the
// TMA epilogue when p.c_tma is set (not for the SwiGLU epilogue of the 1-CTA kernel).
cudaError_t gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int bn, bool a_mn,
                        bool b_mn, int epi, cudaStream_t s, const CUtensorMap* tc = nullptr);
// Grouped GEMM with a device-side tile schedule (no host synchronisation on the group sizes): bf16 output,
// A [M, K] K-major with the rows of group g at [offsets[g], offsets[g + 1]), B [groups, N, K] (or, b_mn, [groups, K, N]).
cudaError_t gemm_grouped_launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, bool b_mn,
                                cudaStream_t s);
// MoE exchange GEMM (bf16 output, A K-major, 128 x 256 tiles): peer_mode 1 = wait for A rows (p.peer.arrive),
// 2 = scatter C rows to the sources (p.peer.out)
cudaError_t gemm_peer_launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, bool b_mn,
                             int peer_mode, cudaStream_t s);


// ---------------------------------------------------------------- norms (norm.cu)
struct AdaNormFwdParams {
  const __nv_bfloat16* x;
  const __nv_bfloat16* y;      // optional residual branch
  const __nv_bfloat16* gate;   // optional [B, D] (batch stride gate_bs)
  long long gate_bs;
  const float* w;
  const __nv_bfloat16* shift;  // optional [B, D] (batch stride mod_bs)
  const __nv_bfloat16* scale;
  long long mod_bs;
  __nv_bfloat16* x_out;        // x + gate * y (when y is given)
  __nv_bfloat16* h;
  float* rstd;
  int M, D, T, rows_per_cta;
  float eps;
};
struct AdaNormBwdParams {
  const __nv_bfloat16* dh;
  const __nv_bfloat16* dxe;    // optional extra gradient into x_new
  const __nv_bfloat16* xn;     // x_new
  const float* rstd;
  const float* w;
  const __nv_bfloat16* scale;
  long long mod_bs;
  const __nv_bfloat16* y;
  const __nv_bfloat16* gate;
  long long gate_bs;
  __nv_bfloat16* dx;
  __nv_bfloat16* dy;
  float* partial;              // scratch [B][chunks][4][D]
  int M, D, T, chunks, rows_per_cta;
};
cudaError_t adanorm_fwd_launch(const AdaNormFwdParams& p, cudaStream_t s);
cudaError_t adanorm_set_bwd_rows(int rows);  // rows per block reduction of the backward: 1 or 2 (default)
cudaError_t adanorm_bwd_launch(const AdaNormBwdParams& p, float* dshift, float* dscale, float* dgate, float* dw,
                               cudaStream_t s);

struct QKNormRopeParams {
  const __nv_bfloat16* qkv;    // [M, ld_qkv]: hq query heads, then hkv key heads (then values, untouched)
  long long ld_qkv;
  const float* q_w;            // optional per-head RMSNorm weights [hd]
  const float* k_w;
  const float* cos;            // optional [B?][T][hd] (batch stride rope_bs, 0 = shared)
  const float* sin;
  long long rope_bs;
  __nv_bfloat16* q_out;        // [M, ld_q]
  long long ld_q;
  __nv_bfloat16* k_out;
  long long ld_k;
  float* rstd_q;               // [M, hq]
  float* rstd_k;               // [M, hkv]
  int M, T, hq, hkv, hd;
  float eps;
};
cudaError_t qknorm_rope_fwd_launch(const QKNormRopeParams& p, cudaStream_t s);
cudaError_t qknorm_rope_bwd_launch(const QKNormRopeParams& p, const void* dq, long long ld_dq, bool dq_f32,
                                   const __nv_bfloat16* dk, long long ld_dk, __nv_bfloat16* dqkv, long long ld_dqkv,
                                   float* dwq, float* dwk, cudaStream_t s);

cudaError_t qknorm_set_bwd_unroll(int u);     // 2 or 4 heads in flight per lane group (A/B runs)
cudaError_t swiglu_fwd_launch(const __nv_bfloat16* ab, __nv_bfloat16* g, long long M, int H, cudaStream_t s);
cudaError_t swiglu_bwd_launch(const __nv_bfloat16* ab, const __nv_bfloat16* dg, __nv_bfloat16* dab, long long M,
                              int H, cudaStream_t s);


// ---------------------------------------------------------------- attention (attention.cu)
struct AttnParams {
  const __nv_bfloat16* q;  // [B][Tq][Hq][hd] with strides (elements)
  long long q_bs, q_ts, q_hs;
  const __nv_bfloat16* k;  // [B][Tk][Hkv][hd]
  long long k_bs, k_ts, k_hs;
  const __nv_bfloat16* v;
  long long v_bs, v_ts, v_hs;
  __nv_bfloat16* o;        // [B][Tq][Hq][hd] (also the layout of dO)
  long long o_bs, o_ts, o_hs;
  float* lse;              // [B][Hq][Tq] natural-log sum-exp of the scaled logits
  const int* kv_len;       // optional [B] valid key count (prefix mask)
  int B, Tq, Tk, Hq, Hkv, rep, hd;
  float scale;
  // Packed variable-length sequences (tcgen05 forward only): cu_seqlens [B + 1] token offsets of the B sequences
  // along one packed token axis (the tensors' batch extent is 1, Tq = Tk = the longest sequence, lse is
  // [Hq][total]).  causal: key index <= query index, both counted from the start of the sequence.
  const int* cu_seqlens;
  int total, causal;
};
cudaError_t attention_fwd_launch(const AttnParams& p, cudaStream_t s);
// dq_acc: scratch fp32 [B][Tq][Hq][hd] (zeroed here); delta: scratch fp32 [B][Hq][Tq]; dq (bf16) optional.
cudaError_t attention_bwd_launch(const AttnParams& p, const __nv_bfloat16* dO, float* delta, float* dq_acc,
                                 __nv_bfloat16* dq, long long dq_bs, long long dq_ts, long long dq_hs,
                                 __nv_bfloat16* dk, long long dk_bs, long long dk_ts, long long dk_hs,
                                 __nv_bfloat16* dv, long long dv_bs, long long dv_ts, long long dv_hs, cudaStream_t s);

// lse2 (optional, [B][Hq][Tq]): receives lse * log2(e) for the tcgen05 backward; dq_acc nullptr: nothing zeroed
cudaError_t attention_bwd_prep_launch(const AttnParams& p, const __nv_bfloat16* dO, float* delta, float* dq_acc,
                                      cudaStream_t s, float* lse2 = nullptr);
cudaError_t attention_dq_convert_launch(const AttnParams& p, const float* dq_acc, __nv_bfloat16* dq, long long bs,
                                        long long ts, long long hs, cudaStream_t s);
// tcgen05 backward (head dim 128); delta (and, dq_mode 0, the zeroed dq_acc) from attention_bwd_prep_launch. tdq:
// 4-D map of dQ {hd, Hq, Tq, B} with a {128, 1, 32, 1} box, no swizzle. dq_mode 0: fp32 accumulator, the dQ tiles of
// every key block are TMA reduce-added into it; 1 / 2 (one key block covers all keys, Tk <= 128): each dQ tile is
// final and is stored, fp32 / bf16, so nothing needs zeroing or converting.
cudaError_t attention_bwd_tc_launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                    const CUtensorMap& tdo, const CUtensorMap& tdq, const AttnParams& p,
                                    const float* delta, const float* lse2, __nv_bfloat16* dk, long long dk_bs, long long dk_ts,
                                    long long dk_hs, __nv_bfloat16* dv, long long dv_bs, long long dv_ts,
                                    long long dv_hs, int* err, cudaStream_t s, int dq_mode = 0);
// tcgen05 forward (attention_tc.cu); tensor maps: 4-D {hd, T, H, B}, boxes {64, 128 | 64, 1, 1}, 128-byte swizzle
cudaError_t attention_fwd_tc_launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                    const AttnParams& p, int* err, cudaStream_t s);

// ---------------------------------------------------------------- elementwise (elementwise.cu)
cudaError_t euler_cfg_launch(const __nv_bfloat16* out, float* z, int B, int T, int C, float dt, float w,
                             cudaStream_t s);
// flow-matching input (bf16) and target (fp32), token-major [B, T, C], from fp32 x0 / eps [B, C, T] and t [B]
// per-row int8 quantisation: q = round(x / scale), scale[m] = max |x[m, :]| / 127; K % 8 == 0
cudaError_t quantize_rows_i8_launch(const __nv_bfloat16* x, int8_t* q, float* scale, int M, int K, cudaStream_t s);
cudaError_t fm_inputs_launch(const float* x0, const float* eps, const float* t, __nv_bfloat16* z_tok, float* target,
                             int B, int T, int C, cudaStream_t s);

// ---------------------------------------------------------------- peer-memory collectives (comm.cu)
struct PeerAllReduceParams {
  float* grads;                        // local fp32 gradients [n], averaged in place
  long long n, slice;                  // slice = per-rank share (multiple of 8); buffers hold world * slice
  int rank, world;
  __nv_bfloat16* staging[kMaxPeers];   // every rank's bf16 staging buffer (peer addresses from CUDA IPC)
  __nv_bfloat16* result[kMaxPeers];    // every rank's bf16 result buffer
  uint32_t* flags[kMaxPeers];          // every rank's flag array: C (phase 0) + world * C (phase 1) words
  uint32_t epoch;
  float scale;
  unsigned long long timeout_ns;
  int* err;
};
cudaError_t allreduce_bf16_launch(const PeerAllReduceParams& p, int blocks, cudaStream_t s);
cudaError_t peer_copy_launch(void* dst, const void* src, long long nbytes, uint32_t* dst_version,
                             unsigned long long* counter, uint32_t version, int blocks, cudaStream_t s);


// Sharded Muon over peer memory (muon_comm.cu). Flag arrays: RS 2 x world x blocks words per rank (ready, done),
// AG world x blocks words per rank; blocks x world <= kMuonMaxFlags.
constexpr int kMuonMaxFlags = 1024;
struct MuonRSParams {
  const float* grads;                  // this rank's fp32 gradient bucket [n] (16-byte aligned)
  long long n;
  __nv_bfloat16* staging[kMaxPeers];   // every rank's bf16 staging (>= n elements)
  uint32_t* flags[kMaxPeers];          // every rank's RS flag array
  const long long* segs;               // [nsegs][3]: (bucket offset, owned-buffer offset, length) of my segments
  int nsegs;
  long long owned;                     // sum of the segment lengths
  float* g_owned;                      // fp32 reduced gradients of my matrices
  float scale;                         // 1 / world
  float* sumsq;                        // += sum of squares of the reduced values (may be null)
  int rank, world;
  uint32_t epoch, prev_epoch;          // prev_epoch 0: no earlier launch to wait for
  unsigned long long timeout_ns;
  int* err;
};
struct MuonMomentumParams {
  const float* g;                      // reduced gradients [n]
  long long n;
  float* buf_f32;                      // momentum, fp32 ...
  __nv_bfloat16* buf_bf16;             // ... or bf16 with stochastic rounding (exactly one is non-null)
  __nv_bfloat16* x_out;                // Newton-Schulz input [n]
  const float* coef;                   // gradient-clip coefficient (device scalar: no host round trip)
  float mu;                            // momentum
  int nesterov;
  unsigned long long seed;
};
// Single-owner Muon step (the optimizer's local path; same flat, bucket-major Muon space as the sharded path).
struct MuonSegMomentumParams {
  const long long* segs;               // [nsegs][3]: (fp32 gradient ptr, offset in the Muon space, length)
  int nsegs;
  float* buf_f32;                      // flat momentum, fp32 ...
  __nv_bfloat16* buf_bf16;             // ... or bf16 with stochastic rounding (exactly one is non-null)
  __nv_bfloat16* x_out;                // flat Newton-Schulz input
  const float* coef;                   // gradient-clip coefficient (device scalar)
  float mu;
  int nesterov;
  unsigned long long seed;
};
struct MuonApplyParams {
  const __nv_bfloat16* upd;            // flat orthogonalised updates (the whole Muon space)
  const long long* segs;               // [nsegs][5]: (fp32 param ptr, bf16 shadow ptr or 0, offset, length,
                                       //              fp32 EMA ptr or 0)
  const float* coefs;                  // [nsegs][2]: (alpha, decay): p = p * decay + alpha * U
  int nsegs;
  float ema_rate;                      // EMA: e += ema_rate * (p - e) after the update
};
struct MuonAGParams {
  __nv_bfloat16* upd[kMaxPeers];       // every rank's update buffer (the whole Muon space)
  uint32_t* flags[kMaxPeers];          // every rank's AG flag array
  const long long* own;                // [nown][2]: (offset, length) of my owned ranges in the Muon space
  int nown;
  long long owned;
  const long long* segs;               // [nsegs][5]: (fp32 param ptr, bf16 shadow ptr or 0, offset, length,
                                       //              fp32 EMA ptr or 0)
  const float* coefs;                  // [nsegs][2]: (alpha, decay): p = p * decay + alpha * U
  int nsegs;
  float ema_rate;
  int rank, world;
  uint32_t epoch;
  unsigned long long timeout_ns;
  int* err;
};
// MoE dispatch / combine over peer memory (moe_comm.cu). Static capacity: this rank's dispatch holds C rows per
// expert; expert e = r * local + j lives on rank r, whose receive buffer is [local][world][C][D] (source-major
// within an expert, so an expert's rows from source s are one contiguous block of C rows).
struct MoEDispatchParams {
  const __nv_bfloat16* x;              // [N, D] token rows (forward) or output gradients (backward)
  const int* src_tok;                  // [E * C] token of each of this rank's slots (-1: empty slot -> zeros)
  const float* scale;                  // optional [E * C] row scale (routing weight, backward)
  __nv_bfloat16* recv[kMaxPeers];      // every rank's receive buffer
  uint32_t* arrive[kMaxPeers];         // every rank's arrive flags [world]: word `rank` is set on the owner
  const uint32_t* free_flags;          // optional local [world]: owner r released its receive rows for epoch - 1
  unsigned* counter;                   // local [world] finished-CTA counters (zeroed before the launch)
  int E, local, C, D, rank, world;
  uint32_t epoch;
  unsigned long long timeout_ns;
  int* err;
};
struct MoECombineParams {
  const __nv_bfloat16* ybuf;           // local [E * C, D] rows written by the owners
  const int* slot;                     // [N, k] slot of every assignment (-1: dropped)
  const float* w;                      // optional [N, k] weights (forward combine)
  const uint32_t* done;                // local [world] flags set by the owners
  __nv_bfloat16* out;                  // [N, D]
  int N, k, D, world;
  uint32_t epoch;
  unsigned long long timeout_ns;
  int* err;
};
cudaError_t moe_dispatch_launch(const MoEDispatchParams& p, int blocks_per_owner, cudaStream_t s);
cudaError_t moe_combine_launch(const MoECombineParams& p, cudaStream_t s);
// owner side: tell every source that this rank's receive rows may be overwritten (free_peer[s][rank] = epoch)
cudaError_t moe_release_launch(uint32_t* const* free_peer, int rank, int world, uint32_t epoch, cudaStream_t s);

cudaError_t attention_set_trace(long long* buf, int cta);  // profiling timeline (null: off)
cudaError_t attention_set_fwd_split(int wpq);  // softmax warps per TMEM lane quarter in the forward (1 or 2)
cudaError_t attention_set_fwd_emu(int eighths);
// attention barrier waits that poll instead of suspending, per kernel: bit 0 MMA thread, 1 softmax / drain, 2 TMA
cudaError_t attention_set_poll(int fwd_mask, int bwd_mask);
cudaError_t attention_set_fwd_pingpong(int on);  // forward softmax groups alternate their exponential phases  // forward exponentials on the FMA pipe: 0, 2, 3 or 4 eighths
cudaError_t muon_rs_launch(const MuonRSParams& p, int blocks, cudaStream_t s);
cudaError_t muon_seg_momentum_launch(const MuonSegMomentumParams& p, int blocks, cudaStream_t s);
cudaError_t muon_apply_launch(const MuonApplyParams& p, int blocks, cudaStream_t s);

// Optimizer tail (optim.cu): global gradient norm + clip coefficient in one launch, multi-tensor AdamW with the
// clip coefficient, the bf16 shadow refresh and the EMA update fused in.
struct GradNormParams {
  const long long* segs;               // [nsegs][2]: (fp32 gradient ptr, length)
  int nsegs;
  float* acc;                          // [1] running sum of squares (zero between launches; the last CTA resets it)
  unsigned int* counter;               // [1] finished-CTA counter (zero between launches)
  const float* extra_sumsq;            // optional [1]: squares of gradients counted elsewhere (added to the total)
  float clip;                          // max norm (<= 0: no clipping, coef = 1)
  float* gnorm;                        // [1] out: the global norm
  float* coef;                         // [1] out: min(1, clip / (norm + 1e-6))
};
struct AdamWParams {
  const long long* segs;               // [nsegs][8]: (param, grad, exp_avg, exp_avg_sq fp32 ptrs, bf16 shadow ptr or 0,
                                       //              fp32 EMA ptr or 0, length, group)
  int nsegs;
  const float* hyper;                  // [groups][6]: decay (1 - lr wd), step size (lr / bc1), 1 / sqrt(bc2), eps,
                                       //              beta1, beta2
  const float* coef;                   // gradient scale (clip coefficient, device scalar) or null
  float ema_rate;
};
cudaError_t grad_norm_launch(const GradNormParams& p, int blocks, cudaStream_t s);
cudaError_t adamw_launch(const AdamWParams& p, int blocks, cudaStream_t s);
cudaError_t muon_momentum_launch(const MuonMomentumParams& p, cudaStream_t s);
cudaError_t muon_ag_apply_launch(const MuonAGParams& p, int blocks, cudaStream_t s);

}  // namespace tgo
