// Torch-facing wrappers of the sm_100a kernels: argument checks, TMA descriptor encoding, launches on the current
// stream.  Exposed as the extension module trenowanie_generatora_obrazkow_b200._C.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "kernels.h"

#include <atomic>

namespace tgo {

// Number of kernels this extension has launched (for the benchmark's launch accounting).
static std::atomic<long long> g_launches{0};
long long launch_count() { return g_launches.load(); }

#define TGO_CHECK_LAUNCH_N(expr, n)                                                        \
  do {                                                                                     \
    cudaError_t _e = (expr);                                                               \
    TORCH_CHECK(_e == cudaSuccess, "kernel launch failed: ", cudaGetErrorString(_e));      \
    g_launches += (n);                                                                     \
  } while (0)
#define TGO_CHECK_LAUNCH(expr) TGO_CHECK_LAUNCH_N(expr, 1)

// The driver's tensor-map encoder needs a current context. A thread whose first CUDA work is this extension (an
// autograd worker thread whose first backward node is ours, a server thread) has none yet: the device guard is a
// no-op when the thread's device index already matches, so cudaSetDevice binds the primary context here, once per
// thread.
static void bind_context() {
  thread_local bool bound = false;
  if (!bound) {
    int dev = 0;
    TORCH_CHECK(cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess, "cudaSetDevice failed");
    bound = true;
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  bind_context();
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && ptr != nullptr && q == cudaDriverEntryPointSuccess,
                "cuTensorMapEncodeTiled entry point not found");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 3-D bf16 tensor map {inner, rows, batch} with a {64, box_rows, 1} box and 128-byte swizzle.
static CUtensorMap make_tmap_bf16_sw128(const void* base, uint64_t inner, uint64_t rows, uint64_t batch,
                                        uint64_t row_stride, uint64_t batch_stride, uint32_t box_rows) {
  CUtensorMap m;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK((row_stride * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  if (batch <= 1) batch_stride = row_stride * rows;
  TORCH_CHECK((batch_stride * 2) % 16 == 0, "TMA batch stride must be a multiple of 16 bytes");
  cuuint64_t dims[3] = {inner, rows, batch};
  cuuint64_t strides[2] = {row_stride * 2, batch_stride * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = tmap_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return m;
}

// 3-D map of a GEMM output C {N, M, batch} for the GEMM kernels' TMA epilogue: box {32, 32, 1}; bf16 rows of the
// box are 64 bytes (64-byte swizzle), fp32 rows 128 bytes (128-byte swizzle). Returns false (no map) when C's base
// or strides are not 16-byte aligned, in which case the kernel stores rows directly.
static bool make_tmap_c(CUtensorMap* m, void* base, bool f32, uint64_t N, uint64_t M, uint64_t batch,
                        uint64_t ldc, uint64_t bsc) {
  const uint64_t es = f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ldc * es) % 16 != 0) return false;
  if (batch <= 1) bsc = ldc * M;
  if ((bsc * es) % 16 != 0) return false;
  cuuint64_t dims[3] = {N, M, batch};
  cuuint64_t strides[2] = {ldc * es, bsc * es};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = tmap_encoder()(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base,
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}
static bool g_gemm_tma_c = true;  // GEMM epilogue through TMA stores / reduce-adds
void set_gemm_tma_epilogue(bool on) { g_gemm_tma_c = on; }

// 4-D fp32 map of the dQ accumulator [B][Tq][Hq][hd] as {hd, Hq, Tq, B}, box {hd, 1, 32, 1}, no swizzle: the
// backward kernel reduce-adds 32-query x hd tiles into it.
static CUtensorMap make_tmap_dq(const float* base, uint64_t hd, uint64_t H, uint64_t T, uint64_t B) {
  CUtensorMap m;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  cuuint64_t dims[4] = {hd, H, T, B};
  cuuint64_t strides[3] = {hd * 4, H * hd * 4, T * H * hd * 4};
  cuuint32_t box[4] = {(cuuint32_t)hd, 1, 32, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = tmap_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (dQ accumulator) failed with code ", (int)r);
  return m;
}

// 4-D bf16 map of a dQ output [B][Tq][Hq][hd] with element strides (bs, ts, hs) as {hd, Hq, Tq, B}, box
// {hd, 1, 32, 1}, no swizzle: the backward stores final 32-query dQ tiles into it (one key block covers all keys).
static CUtensorMap make_tmap_dq_bf16(const void* base, uint64_t hd, uint64_t H, uint64_t T, uint64_t B, uint64_t hs,
                                     uint64_t ts, uint64_t bs) {
  CUtensorMap m;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0 && (hs * 2) % 16 == 0 && (ts * 2) % 16 == 0 &&
                  (bs * 2) % 16 == 0, "dQ tensor map: 16-byte aligned base and strides");
  cuuint64_t dims[4] = {hd, H, T, B};
  cuuint64_t strides[3] = {(H > 1 ? hs : hd) * 2, ts * 2, (B > 1 ? bs : ts * T) * 2};
  cuuint32_t box[4] = {(cuuint32_t)hd, 1, 32, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = tmap_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (dQ bf16) failed with code ", (int)r);
  return m;
}

// 4-D bf16 tensor map {hd, T, H, B} (strides in elements) with a {64, box_rows, 1, 1} box, 128-byte swizzle.
static CUtensorMap make_tmap_bhtd(const void* base, uint64_t hd, uint64_t T, uint64_t H, uint64_t B, uint64_t ts,
                                  uint64_t hs, uint64_t bs, uint32_t box_rows) {
  CUtensorMap m;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK(ts % 8 == 0 && hs % 8 == 0 && bs % 8 == 0, "TMA strides must be multiples of 16 bytes");
  cuuint64_t dims[4] = {hd, T, H, B};
  cuuint64_t strides[3] = {ts * 2, (H > 1 ? hs : ts * T) * 2, (B > 1 ? bs : ts * T * H) * 2};
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = tmap_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (4-D) failed with code ", (int)r);
  return m;
}

static bool g_attention_tc = true;
static bool g_attention_dq_store = true;  // one key block: store final dQ tiles (off: zeroed accumulator, for A/B)
void set_attention_dq_store(bool on) { g_attention_dq_store = on; }
void set_attention_tc(bool on) { g_attention_tc = on; }
void set_attention_fwd_split(int64_t wpq) {
  TORCH_CHECK(attention_set_fwd_split((int)wpq) == cudaSuccess, "attention forward split: 1 or 2");
}
void set_attention_fwd_pingpong(bool on) { attention_set_fwd_pingpong(on ? 1 : 0); }
void set_attention_poll(int64_t fwd_mask, int64_t bwd_mask) {
  TORCH_CHECK(attention_set_poll((int)fwd_mask, (int)(bwd_mask < 0 ? fwd_mask : bwd_mask)) == cudaSuccess,
              "set_attention_poll: masks 0..7");
}
void set_attention_fwd_emu(int64_t eighths) {
  TORCH_CHECK(attention_set_fwd_emu((int)eighths) == cudaSuccess, "attention forward FMA exponentials: 0 .. 4 eighths (-1: default)");
}

static bool g_gemm_pair_enabled = true;  // 256 x 256 CTA-pair tiles: 3-6 % faster on the training shapes
void set_gemm_pair(bool on) { g_gemm_pair_enabled = on; }
static bool g_gemm_syrk = true;  // symmetric mode of gemm_syrk (off: the full product, for A/B runs)
void set_gemm_syrk(bool on) { g_gemm_syrk = on; }
static bool g_gemm_splitk = true;  // split-K of the fp32-accumulating GEMMs (off: one unit per tile, for A/B runs)
void set_gemm_splitk(bool on) { g_gemm_splitk = on; }
void set_adanorm_bwd_rows(int64_t rows) {
  TORCH_CHECK(adanorm_set_bwd_rows((int)rows) == cudaSuccess, "set_adanorm_bwd_rows: 1 or 2");
}
void set_gemm_tail_split(bool on) { gemm_set_tail_split(on ? 1 : 0); }
void set_gemm_poll(int64_t mask) { TORCH_CHECK(gemm_set_poll((int)mask) == cudaSuccess, "set_gemm_poll: mask 0..7"); }

// Smallest split count whose units fill the CTA pairs in waves at >= 92 % (at least 32 k-blocks of 64 per split,
// at most 16 splits); every split non-empty (the count is derived from the k-blocks per split).
static int choose_splitk(int64_t tiles, int64_t K) {
  const int64_t pairs = num_sms() / 2, nkb = (K + 63) / 64;
  for (int s = 1; s <= 16; ++s) {
    if (nkb / s < 32) break;
    const int64_t units = tiles * s, waves = (units + pairs - 1) / pairs;
    if ((double)units / (double)(waves * pairs) >= 0.92) {
      const int64_t per = (nkb + s - 1) / s;
      return (int)((nkb + per - 1) / per);
    }
  }
  return 1;
}

static int* err_ptr(const at::Tensor& err) {
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt && err.numel() >= 1, "err must be a CUDA int32 tensor");
  return err.data_ptr<int>();
}

// A: [batch,] rowsA x colsA (colsA contiguous); !a_mn: rowsA = M, colsA = K; a_mn: rowsA = K, colsA = M.
// B: [batch,] rowsB x colsB;                    !b_mn: rowsB = N, colsB = K; b_mn: rowsB = K, colsB = N.
// C: [batch,] M x N, last dim contiguous; bf16, or fp32 (overwrite, or += when accumulate).
// D (optional, bf16 output only): [batch,] M x N added as beta * D.
void gemm(at::Tensor A, at::Tensor B, at::Tensor C, bool a_mn, bool b_mn, c10::optional<at::Tensor> D, double alpha,
          double beta, bool accumulate, at::Tensor err) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm: CUDA tensors expected");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: A and B must be bf16");
  TORCH_CHECK(A.dim() == B.dim() && A.dim() == C.dim() && (A.dim() == 2 || A.dim() == 3), "gemm: rank mismatch");
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1 && C.stride(-1) == 1, "gemm: inner dim must be contiguous");
  const c10::cuda::CUDAGuard guard(A.device());
  const bool batched = A.dim() == 3;
  const int64_t batch = batched ? A.size(0) : 1;
  if (batched) TORCH_CHECK(B.size(0) == batch && C.size(0) == batch, "gemm: batch mismatch");
  const int64_t M = a_mn ? A.size(-1) : A.size(-2);
  const int64_t K = a_mn ? A.size(-2) : A.size(-1);
  const int64_t N = b_mn ? B.size(-1) : B.size(-2);
  const int64_t Kb = b_mn ? B.size(-2) : B.size(-1);
  TORCH_CHECK(K == Kb, "gemm: contraction mismatch ", K, " vs ", Kb);
  TORCH_CHECK(C.size(-2) == M && C.size(-1) == N, "gemm: output shape mismatch");
  TORCH_CHECK(A.size(-1) % 8 == 0 && B.size(-1) % 8 == 0 && N % 8 == 0, "gemm: contiguous dims and N must be multiples of 8");
  const bool out_f32 = C.scalar_type() == at::kFloat;
  TORCH_CHECK(out_f32 || C.scalar_type() == at::kBFloat16, "gemm: C must be bf16 or fp32");
  TORCH_CHECK(!accumulate || out_f32, "gemm: accumulate needs an fp32 C");
  if (M == 0 || N == 0 || batch == 0) return;
  if (K == 0) {
    if (!accumulate) C.zero_();
    return;
  }
  // 2-CTA kernel (256 x 256 tiles over a CTA pair) when there are enough such tiles to fill the GPU; otherwise
  // the 1-CTA kernel with 128 x 256 (or 128 x 128 for N <= 128) tiles.
  const int64_t pair_tiles = ((M + 255) / 256) * ((N + 255) / 256) * batch;
  const bool has_d = D.has_value() && D->defined();
  TORCH_CHECK(C.stride(-2) % 8 == 0 && reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0, "gemm: C alignment");
  // C's tensor map first: the TMA epilogue (and split-K, which needs its reduce-add) depend on it
  CUtensorMap tc;
  const bool c_tma = g_gemm_tma_c && !has_d &&
                     make_tmap_c(&tc, C.data_ptr(), out_f32, N, M, batch, C.stride(-2), batched ? C.stride(0) : 0);
  // split-K for the fp32-accumulating GEMMs (weight gradients): partial tiles reduce-add into C (atomic in L2), so
  // the 2-CTA kernel's work units can fill the 74 CTA pairs in near-whole waves (one wave of 64 tiles uses 86 % of
  // them, 176 tiles over 3 waves 79 %)
  const int splitk = (out_f32 && accumulate && c_tma && g_gemm_splitk && g_gemm_pair_enabled && M >= 256 &&
                      N >= 256) ? choose_splitk(pair_tiles, K) : 1;
  const bool use_pair = g_gemm_pair_enabled && M >= 256 && N >= 256 && (pair_tiles >= num_sms() / 2 || splitk > 1);
  const int bn = use_pair ? 0 : (N <= 128 ? 128 : 256);
  const uint64_t bsA = batched ? A.stride(0) : 0, bsB = batched ? B.stride(0) : 0;
  CUtensorMap ta = make_tmap_bf16_sw128(A.data_ptr(), A.size(-1), A.size(-2), batch, A.stride(-2), bsA,
                                        a_mn ? 64 : 128);
  CUtensorMap tb = make_tmap_bf16_sw128(B.data_ptr(), B.size(-1), B.size(-2), batch, B.stride(-2), bsB,
                                        b_mn ? 64 : (use_pair ? 128 : bn));
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = (int)batch;
  p.C = C.data_ptr();
  p.ldc = C.stride(-2);
  p.bsc = batched ? C.stride(0) : 0;
  p.D = nullptr;
  p.ldd = 0;
  p.bsd = 0;
  if (has_d) {
    TORCH_CHECK(!out_f32 && D->scalar_type() == at::kBFloat16 && D->stride(-1) == 1, "gemm: D must be bf16");
    TORCH_CHECK(D->dim() == C.dim() && D->size(-2) == M && D->size(-1) == N, "gemm: D shape mismatch");
    TORCH_CHECK(D->stride(-2) % 8 == 0 && reinterpret_cast<uintptr_t>(D->data_ptr()) % 16 == 0, "gemm: D align");
    p.D = reinterpret_cast<const __nv_bfloat16*>(D->data_ptr());
    p.ldd = D->stride(-2);
    p.bsd = batched ? D->stride(0) : 0;
  }
  p.alpha = (float)alpha;
  p.beta = (float)beta;
  p.err = err_ptr(err);
  const int epi = out_f32 ? (accumulate ? 2 : 1) : 0;
  p.c_tma = c_tma ? 1 : 0;
  p.splitk = splitk;
  TGO_CHECK_LAUNCH(gemm_launch(ta, tb, p, bn, a_mn, b_mn, epi, at::cuda::getCurrentCUDAStream(),
                               p.c_tma ? &tc : nullptr));
}


// Symmetric product C = alpha A A^T + beta D (D symmetric or absent), A [batch,] M x K K-major, C / D [batch,] M x M
// bf16: the 2-CTA kernel computes only the tile blocks on and below the diagonal and stores each off-diagonal block
// twice (csrc/gemm.cu, GemmParams::syrk); shapes too small for the 2-CTA kernel run the full product.
// int8 GEMM (W8A8): C[M, N] (bf16) = (A[M, K] int8 . B[N, K]^T int8, int32) * a_scale[m] * b_scale[n] on the 2-CTA
// kind::i8 kernel. The int8 rows go through the bf16 data path as K / 2 bf16 pairs (the bytes TMA moves and the
// shared-memory layout are identical; only the MMA kind and the epilogue differ).
void gemm_i8(at::Tensor A, at::Tensor B, at::Tensor C, at::Tensor a_scale, at::Tensor b_scale, at::Tensor err) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm_i8: CUDA tensors");
  TORCH_CHECK(A.scalar_type() == at::kChar && B.scalar_type() == at::kChar && C.scalar_type() == at::kBFloat16,
              "gemm_i8: A, B int8, C bf16");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 &&
                  C.stride(1) == 1, "gemm_i8: 2-D with a contiguous inner dim");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && C.size(0) == M && C.size(1) == N, "gemm_i8: shapes");
  TORCH_CHECK(K % 16 == 0 && A.stride(0) % 16 == 0 && B.stride(0) % 16 == 0, "gemm_i8: K and row strides multiples of 16");
  TORCH_CHECK(a_scale.scalar_type() == at::kFloat && a_scale.is_contiguous() && a_scale.numel() == M &&
                  b_scale.scalar_type() == at::kFloat && b_scale.is_contiguous() && b_scale.numel() == N,
              "gemm_i8: fp32 scales [M] and [N]");
  const c10::cuda::CUDAGuard guard(A.device());
  if (M == 0 || N == 0) return;
  CUtensorMap ta = make_tmap_bf16_sw128(A.data_ptr(), K / 2, M, 1, A.stride(0) / 2, 0, 128);
  CUtensorMap tb = make_tmap_bf16_sw128(B.data_ptr(), K / 2, N, 1, B.stride(0) / 2, 0, 128);
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)(K / 2);
  p.batch = 1;
  p.C = C.data_ptr();
  p.ldc = C.stride(0);
  p.alpha = 1.f;
  p.row_scale = a_scale.data_ptr<float>();
  p.col_scale = b_scale.data_ptr<float>();
  p.err = err_ptr(err);
  p.splitk = 1;
  CUtensorMap tc;
  TORCH_CHECK(make_tmap_c(&tc, C.data_ptr(), false, N, M, 1, p.ldc, 0), "gemm_i8: C must be 16-byte aligned");
  p.c_tma = 1;
  TGO_CHECK_LAUNCH(gemm_launch(ta, tb, p, 0, false, false, 4 /* EPI_I8 */, at::cuda::getCurrentCUDAStream(), &tc));
}

// Per-row int8 quantisation of bf16 activations: returns (q int8 [M, K], scale fp32 [M]).
std::vector<at::Tensor> quantize_rows_i8(at::Tensor x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
              "quantize_rows_i8: contiguous bf16 [M, K]");
  TORCH_CHECK(x.size(1) % 8 == 0, "quantize_rows_i8: K must be a multiple of 8");
  const c10::cuda::CUDAGuard guard(x.device());
  auto q = at::empty(x.sizes(), x.options().dtype(at::kChar));
  auto s = at::empty({x.size(0)}, x.options().dtype(at::kFloat));
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  TGO_CHECK_LAUNCH(quantize_rows_i8_launch(xb, q.data_ptr<int8_t>(), s.data_ptr<float>(), (int)x.size(0), (int)x.size(1),
                                           at::cuda::getCurrentCUDAStream()));
  return {q, s};
}

void gemm_syrk(at::Tensor A, at::Tensor C, c10::optional<at::Tensor> D, double alpha, double beta, at::Tensor err) {
  TORCH_CHECK(A.is_cuda() && C.is_cuda() && A.scalar_type() == at::kBFloat16 && C.scalar_type() == at::kBFloat16,
              "gemm_syrk: bf16 CUDA tensors");
  TORCH_CHECK(A.dim() == C.dim() && (A.dim() == 2 || A.dim() == 3), "gemm_syrk: rank mismatch");
  TORCH_CHECK(A.stride(-1) == 1 && C.stride(-1) == 1, "gemm_syrk: inner dim must be contiguous");
  const c10::cuda::CUDAGuard guard(A.device());
  const bool batched = A.dim() == 3;
  const int64_t batch = batched ? A.size(0) : 1;
  const int64_t M = A.size(-2), K = A.size(-1);
  TORCH_CHECK(C.size(-2) == M && C.size(-1) == M && (!batched || C.size(0) == batch), "gemm_syrk: C shape");
  TORCH_CHECK(K % 8 == 0 && M % 8 == 0, "gemm_syrk: dims must be multiples of 8");
  const int64_t tri = ((M + 255) / 256) * ((M + 255) / 256 + 1) / 2 * batch;
  const bool use_pair = g_gemm_syrk && g_gemm_pair_enabled && g_gemm_tma_c && M >= 256 && tri >= num_sms() / 2;
  if (!use_pair) {
    gemm(A, A, C, false, false, D, alpha, beta, false, err);
    return;
  }
  const uint64_t bsA = batched ? A.stride(0) : 0;
  CUtensorMap ta = make_tmap_bf16_sw128(A.data_ptr(), K, M, batch, A.stride(-2), bsA, 128);
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)M;
  p.K = (int)K;
  p.batch = (int)batch;
  p.C = C.data_ptr();
  p.ldc = C.stride(-2);
  p.bsc = batched ? C.stride(0) : 0;
  if (D.has_value() && D->defined()) {
    TORCH_CHECK(D->scalar_type() == at::kBFloat16 && D->stride(-1) == 1 && D->dim() == C.dim() &&
                D->size(-2) == M && D->size(-1) == M, "gemm_syrk: D must be bf16 like C");
    TORCH_CHECK(D->stride(-2) % 8 == 0 && reinterpret_cast<uintptr_t>(D->data_ptr()) % 16 == 0, "gemm_syrk: D align");
    p.D = reinterpret_cast<const __nv_bfloat16*>(D->data_ptr());
    p.ldd = D->stride(-2);
    p.bsd = batched ? D->stride(0) : 0;
  }
  TORCH_CHECK(p.ldc % 8 == 0 && reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0, "gemm_syrk: C alignment");
  p.alpha = (float)alpha;
  p.beta = (float)beta;
  p.err = err_ptr(err);
  p.syrk = 1;
  CUtensorMap tc;
  if (!make_tmap_c(&tc, C.data_ptr(), false, M, M, batch, p.ldc, p.bsc)) {
    gemm(A, A, C, false, false, D, alpha, beta, false, err);
    return;
  }
  p.c_tma = 1;
  TGO_CHECK_LAUNCH(gemm_launch(ta, ta, p, 0, false, false, 0, at::cuda::getCurrentCUDAStream(), &tc));
}


// ------------------------------------------------------------------------------------------------ helpers
static const __nv_bfloat16* bf16_ptr_or_null(const c10::optional<at::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_cuda(), "expected a bf16 CUDA tensor");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "bf16 operand must be 16-byte aligned");
  return reinterpret_cast<const __nv_bfloat16*>(t->data_ptr());
}
static const float* f32_ptr_or_null(const c10::optional<at::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_cuda() && t->is_contiguous(), "expected a contiguous fp32 CUDA tensor");
  return t->data_ptr<float>();
}
static __nv_bfloat16* bfp(const at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
// [B, D] per-batch row vector (possibly a strided view of a [B, 6, D] modulation tensor): batch stride
static long long row_vec_stride(const c10::optional<at::Tensor>& t, int64_t D) {
  if (!t.has_value() || !t->defined()) return 0;
  TORCH_CHECK(t->dim() == 2 && t->size(1) == D && t->stride(1) == 1, "per-batch vector must be [B, D] contiguous in D");
  TORCH_CHECK(t->stride(0) % 8 == 0, "per-batch vector batch stride must be a multiple of 8");
  return t->stride(0);
}

// Up projection + SwiGLU in one GEMM: A [M, K] bf16, B [2H, K] bf16 with the gate / up rows interleaved in blocks
// of 128 (gate block k at rows 256 k .. 256 k + 127, up block k right after), C [M, H] = silu(A Wg^T) * (A Wu^T).
void gemm_swiglu(at::Tensor A, at::Tensor B, at::Tensor C, at::Tensor err) {
  TORCH_CHECK(A.is_cuda() && A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 &&
                  C.scalar_type() == at::kBFloat16, "gemm_swiglu: bf16 CUDA tensors");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1,
              "gemm_swiglu: 2-D row-major operands");
  const c10::cuda::CUDAGuard guard(A.device());
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && N % 256 == 0 && C.size(0) == M && C.size(1) * 2 == N, "gemm_swiglu: shapes");
  TORCH_CHECK(K % 8 == 0 && A.stride(0) % 8 == 0 && C.stride(0) % 8 == 0, "gemm_swiglu: alignment");
  if (M == 0) return;
  const int64_t pair_tiles = ((M + 255) / 256) * (N / 256);
  const bool use_pair = g_gemm_pair_enabled && M >= 256 && pair_tiles >= num_sms() / 2;
  CUtensorMap ta = make_tmap_bf16_sw128(A.data_ptr(), K, M, 1, A.stride(0), 0, 128);
  CUtensorMap tb = make_tmap_bf16_sw128(B.data_ptr(), K, N, 1, B.stride(0), 0, use_pair ? 128 : 256);
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = 1;
  p.C = C.data_ptr();
  p.ldc = C.stride(0);
  p.alpha = 1.f;
  p.err = err_ptr(err);
  TORCH_CHECK(reinterpret_cast<uintptr_t>(p.C) % 16 == 0, "gemm_swiglu: C alignment");
  CUtensorMap tc;
  p.c_tma = (use_pair && g_gemm_tma_c && make_tmap_c(&tc, p.C, false, N / 2, M, 1, p.ldc, 0)) ? 1 : 0;
  TGO_CHECK_LAUNCH(gemm_launch(ta, tb, p, use_pair ? 0 : 256, false, false, 3, at::cuda::getCurrentCUDAStream(),
                               p.c_tma ? &tc : nullptr));
}

// Expert GEMM of the peer-memory MoE exchange (A [batch, M, K] K-major bf16 = the local receive buffer or local
// activations; B [batch, N, K] or, b_mn, [batch, K, N]). mode 1: wait for the A rows of each source (arrive flags
// at `arrive`), output to C. mode 2: scatter the output rows to the sources' combine buffers `out_ptrs` (row stride
// N), raising their done flags `done_flag_ptrs` when a source's rows are complete.
void gemm_peer(at::Tensor A, at::Tensor B, c10::optional<at::Tensor> C, bool b_mn, int64_t mode, int64_t src_rows,
               int64_t epoch, int64_t arrive, std::vector<int64_t> out_ptrs, int64_t b_base,
               c10::optional<at::Tensor> done_count, std::vector<int64_t> done_flag_ptrs, int64_t timeout_ns,
               at::Tensor err) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16,
              "gemm_peer: bf16 CUDA operands");
  TORCH_CHECK(A.dim() == 3 && B.dim() == 3 && A.size(0) == B.size(0), "gemm_peer: [batch, rows, cols] operands");
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1, "gemm_peer: inner dim must be contiguous");
  const c10::cuda::CUDAGuard guard(A.device());
  const int64_t batch = A.size(0), M = A.size(1), K = A.size(2);
  const int64_t N = b_mn ? B.size(2) : B.size(1);
  TORCH_CHECK((b_mn ? B.size(1) : B.size(2)) == K, "gemm_peer: contraction mismatch");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0 && B.size(-1) % 8 == 0, "gemm_peer: dims must be multiples of 8");
  TORCH_CHECK(src_rows > 0 && src_rows % 128 == 0 && M % src_rows == 0 && M / src_rows <= kMaxPeers,
              "gemm_peer: src_rows must be a multiple of 128 dividing M");
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = (int)batch;
  p.alpha = 1.f;
  p.err = err_ptr(err);
  p.peer.src_rows = (int)src_rows;
  p.peer.epoch = (uint32_t)epoch;
  p.peer.timeout_ns = (unsigned long long)timeout_ns;
  if (mode == 1) {
    TORCH_CHECK(C.has_value() && C->defined() && C->scalar_type() == at::kBFloat16 && C->dim() == 3 &&
                    C->size(0) == batch && C->size(1) == M && C->size(2) == N && C->stride(-1) == 1,
                "gemm_peer: C [batch, M, N] bf16");
    TORCH_CHECK(arrive != 0, "gemm_peer: arrive flags");
    p.C = C->data_ptr();
    p.ldc = C->stride(1);
    p.bsc = C->stride(0);
    TORCH_CHECK(p.ldc % 8 == 0 && reinterpret_cast<uintptr_t>(p.C) % 16 == 0, "gemm_peer: C alignment");
    p.peer.arrive = reinterpret_cast<const uint32_t*>(arrive);
  } else {
    TORCH_CHECK(mode == 2, "gemm_peer: mode 1 (wait) or 2 (scatter)");
    const int64_t nsrc = M / src_rows;
    TORCH_CHECK((int64_t)out_ptrs.size() == nsrc && (int64_t)done_flag_ptrs.size() == nsrc, "gemm_peer: one "
                "output buffer and one done flag per source");
    TORCH_CHECK(done_count.has_value() && done_count->is_cuda() && done_count->scalar_type() == at::kInt &&
                    done_count->numel() >= nsrc, "gemm_peer: done_count int32 [sources]");
    p.ldc = N;
    for (int64_t s = 0; s < nsrc; ++s) {
      p.peer.out[s] = reinterpret_cast<__nv_bfloat16*>(out_ptrs[s]);
      p.peer.done_flag[s] = reinterpret_cast<uint32_t*>(done_flag_ptrs[s]);
      TORCH_CHECK(out_ptrs[s] % 16 == 0, "gemm_peer: output buffers must be 16-byte aligned");
    }
    p.peer.b_base = (int)b_base;
    p.peer.done_count = reinterpret_cast<unsigned*>(done_count->data_ptr<int>());
    p.peer.tile_warps_per_src = (unsigned)((src_rows / 128) * ((N + 255) / 256) * batch * 4);
  }
  CUtensorMap ta = make_tmap_bf16_sw128(A.data_ptr(), K, M, batch, A.stride(1), A.stride(0), 128);
  CUtensorMap tb = make_tmap_bf16_sw128(B.data_ptr(), B.size(2), B.size(1), batch, B.stride(1), B.stride(0),
                                        b_mn ? 64 : 256);
  TGO_CHECK_LAUNCH(gemm_peer_launch(ta, tb, p, b_mn, (int)mode, at::cuda::getCurrentCUDAStream()));
}

// Grouped GEMM (device-side schedule): A [M, K] bf16 rows sorted by group, offsets int32 [G + 1] on the device,
// B [G, N, K] (or, b_mn, [G, K, N]) bf16, C [M, N] bf16; optional row_scale fp32 [M] multiplies output rows.
void gemm_grouped(at::Tensor A, at::Tensor B, at::Tensor offsets, at::Tensor C, bool b_mn,
                  c10::optional<at::Tensor> row_scale, at::Tensor err) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda() && A.scalar_type() == at::kBFloat16 &&
                  B.scalar_type() == at::kBFloat16 && C.scalar_type() == at::kBFloat16, "gemm_grouped: bf16 CUDA");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 3 && C.dim() == 2 && A.stride(1) == 1 && B.stride(2) == 1 &&
                  C.stride(1) == 1, "gemm_grouped: A [M, K], B [G, ., .], C [M, N], inner dims contiguous");
  TORCH_CHECK(offsets.is_cuda() && offsets.scalar_type() == at::kInt && offsets.is_contiguous() &&
                  offsets.numel() == B.size(0) + 1, "gemm_grouped: offsets int32 [G + 1] on the device");
  const c10::cuda::CUDAGuard guard(A.device());
  const int64_t M = A.size(0), K = A.size(1), G = B.size(0);
  const int64_t N = b_mn ? B.size(2) : B.size(1);
  TORCH_CHECK((b_mn ? B.size(1) : B.size(2)) == K, "gemm_grouped: contraction mismatch");
  TORCH_CHECK(C.size(0) == M && C.size(1) == N, "gemm_grouped: C shape");
  TORCH_CHECK(G >= 1 && G <= kMaxGroups, "gemm_grouped: 1 .. 256 groups");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0 && B.size(2) % 8 == 0 && C.stride(0) % 8 == 0 && A.stride(0) % 8 == 0,
              "gemm_grouped: dims / strides must be multiples of 8");
  if (M == 0) return;
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = (int)G;
  p.C = C.data_ptr();
  p.ldc = C.stride(0);
  p.alpha = 1.f;
  p.err = err_ptr(err);
  p.group_offsets = offsets.data_ptr<int>();
  p.row_scale = f32_ptr_or_null(row_scale);
  if (p.row_scale != nullptr) TORCH_CHECK(row_scale->numel() == M, "gemm_grouped: row_scale [M]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(p.C) % 16 == 0, "gemm_grouped: C alignment");
  CUtensorMap ta = make_tmap_bf16_sw128(A.data_ptr(), K, M, 1, A.stride(0), 0, 128);
  CUtensorMap tb = make_tmap_bf16_sw128(B.data_ptr(), B.size(2), B.size(1), G, B.stride(1), B.stride(0),
                                        b_mn ? 64 : 256);
  TGO_CHECK_LAUNCH(gemm_grouped_launch(ta, tb, p, b_mn, at::cuda::getCurrentCUDAStream()));
}

void moe_dispatch(at::Tensor x, at::Tensor src_tok, c10::optional<at::Tensor> scale, std::vector<int64_t> recv_ptrs,
                  std::vector<int64_t> arrive_ptrs, int64_t free_flags, at::Tensor counter, int64_t E, int64_t local,
                  int64_t C, int64_t rank, int64_t epoch, int64_t timeout_ns, int64_t blocks, at::Tensor err) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2,
              "moe_dispatch: x [N, D] bf16 contiguous");
  TORCH_CHECK(src_tok.is_cuda() && src_tok.scalar_type() == at::kInt && src_tok.numel() == E * C &&
                  src_tok.is_contiguous(), "moe_dispatch: src_tok int32 [E * C]");
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == at::kInt, "moe_dispatch: counter int32");
  const c10::cuda::CUDAGuard guard(x.device());
  const int world = (int)recv_ptrs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxPeers && (int)arrive_ptrs.size() == world && counter.numel() >= world,
              "moe_dispatch: one receive buffer and arrive flag array per rank");
  MoEDispatchParams p{};
  p.x = bfp(x);
  p.src_tok = src_tok.data_ptr<int>();
  p.scale = f32_ptr_or_null(scale);
  if (p.scale != nullptr) TORCH_CHECK(scale->numel() == E * C, "moe_dispatch: scale [E * C]");
  for (int r = 0; r < world; ++r) {
    p.recv[r] = reinterpret_cast<__nv_bfloat16*>(recv_ptrs[r]);
    p.arrive[r] = reinterpret_cast<uint32_t*>(arrive_ptrs[r]);
    TORCH_CHECK(recv_ptrs[r] % 16 == 0, "moe_dispatch: receive buffers must be 16-byte aligned");
  }
  p.free_flags = reinterpret_cast<const uint32_t*>(free_flags);
  p.counter = reinterpret_cast<unsigned*>(counter.data_ptr<int>());
  p.E = (int)E;
  p.local = (int)local;
  p.C = (int)C;
  p.D = (int)x.size(1);
  p.rank = (int)rank;
  p.world = world;
  p.epoch = (uint32_t)epoch;
  p.timeout_ns = (unsigned long long)timeout_ns;
  p.err = err_ptr(err);
  TGO_CHECK_LAUNCH(moe_dispatch_launch(p, (int)blocks, at::cuda::getCurrentCUDAStream()));
}

void moe_combine(int64_t ybuf, at::Tensor slot, c10::optional<at::Tensor> w, int64_t done, at::Tensor out,
                 int64_t world, int64_t epoch, int64_t timeout_ns, at::Tensor err) {
  TORCH_CHECK(slot.is_cuda() && slot.scalar_type() == at::kInt && slot.dim() == 2 && slot.is_contiguous(),
              "moe_combine: slot int32 [N, k]");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.dim() == 2 &&
                  out.size(0) == slot.size(0), "moe_combine: out [N, D] bf16");
  const c10::cuda::CUDAGuard guard(out.device());
  MoECombineParams p{};
  p.ybuf = reinterpret_cast<const __nv_bfloat16*>(ybuf);
  p.slot = slot.data_ptr<int>();
  p.w = f32_ptr_or_null(w);
  if (p.w != nullptr) TORCH_CHECK(w->sizes() == slot.sizes(), "moe_combine: w [N, k]");
  p.done = reinterpret_cast<const uint32_t*>(done);
  p.out = bfp(out);
  p.N = (int)slot.size(0);
  p.k = (int)slot.size(1);
  p.D = (int)out.size(1);
  p.world = (int)world;
  p.epoch = (uint32_t)epoch;
  p.timeout_ns = (unsigned long long)timeout_ns;
  p.err = err_ptr(err);
  TGO_CHECK_LAUNCH(moe_combine_launch(p, at::cuda::getCurrentCUDAStream()));
}

void moe_release(std::vector<int64_t> free_ptrs, int64_t rank, int64_t epoch) {
  TORCH_CHECK(!free_ptrs.empty() && (int)free_ptrs.size() <= kMaxPeers, "moe_release: one flag array per rank");
  uint32_t* f[kMaxPeers] = {};
  for (size_t r = 0; r < free_ptrs.size(); ++r) f[r] = reinterpret_cast<uint32_t*>(free_ptrs[r]);
  TGO_CHECK_LAUNCH(moe_release_launch(f, (int)rank, (int)free_ptrs.size(), (uint32_t)epoch,
                                      at::cuda::getCurrentCUDAStream()));
}

// ------------------------------------------------------------------------------------------------ adanorm
std::vector<at::Tensor> adanorm_fwd(at::Tensor x, c10::optional<at::Tensor> y, c10::optional<at::Tensor> gate,
                                    at::Tensor w, c10::optional<at::Tensor> shift, c10::optional<at::Tensor> scale,
                                    int64_t T, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "adanorm: x bf16 contiguous");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t D = x.size(-1), M = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && D <= 8192 && M % T == 0, "adanorm: bad shape");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.numel() == D, "adanorm: w fp32 [D]");
  if (y.has_value() && y->defined()) TORCH_CHECK(y->is_contiguous() && y->sizes() == x.sizes(), "adanorm: y shape");
  TORCH_CHECK(shift.has_value() == scale.has_value(), "adanorm: shift and scale together");
  AdaNormFwdParams p{};
  p.x = bfp(x);
  p.y = bf16_ptr_or_null(y);
  p.gate = bf16_ptr_or_null(gate);
  p.gate_bs = row_vec_stride(gate, D);
  p.w = w.data_ptr<float>();
  p.shift = bf16_ptr_or_null(shift);
  p.scale = bf16_ptr_or_null(scale);
  p.mod_bs = row_vec_stride(scale, D);
  TORCH_CHECK(row_vec_stride(shift, D) == p.mod_bs, "adanorm: shift and scale must share a batch stride");
  at::Tensor x_out;
  if (p.y != nullptr) {
    x_out = at::empty_like(x);
    p.x_out = bfp(x_out);
  }
  at::Tensor h = at::empty_like(x);
  at::Tensor rstd = at::empty({M}, x.options().dtype(at::kFloat));
  p.h = bfp(h);
  p.rstd = rstd.data_ptr<float>();
  p.M = (int)M;
  p.D = (int)D;
  p.T = (int)T;
  p.rows_per_cta = 16;
  p.eps = (float)eps;
  TGO_CHECK_LAUNCH(adanorm_fwd_launch(p, at::cuda::getCurrentCUDAStream()));
  return {x_out, h, rstd};
}

// Returns dx, dy (only with a gate), dshift, dscale (with modulation), dgate (with a gate); dw is accumulated (+=).
std::vector<at::Tensor> adanorm_bwd(at::Tensor dh, c10::optional<at::Tensor> dxe, at::Tensor xn, at::Tensor rstd,
                                    at::Tensor w, at::Tensor dw, c10::optional<at::Tensor> scale,
                                    c10::optional<at::Tensor> y, c10::optional<at::Tensor> gate, int64_t T) {
  TORCH_CHECK(dh.is_contiguous() && xn.is_contiguous() && dh.sizes() == xn.sizes(), "adanorm_bwd: shapes");
  const c10::cuda::CUDAGuard guard(dh.device());
  const int64_t D = dh.size(-1), M = dh.numel() / D;
  TORCH_CHECK(M % T == 0, "adanorm_bwd: M % T");
  const int64_t B = M / T;
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.is_contiguous() && dw.numel() == D, "adanorm_bwd: dw fp32 [D]");
  TORCH_CHECK(D <= 4096, "adanorm_bwd: D <= 4096 (one thread per 8 channels, at most 512 threads)");
  if (dxe.has_value() && dxe->defined()) TORCH_CHECK(dxe->is_contiguous() && dxe->sizes() == dh.sizes(), "dxe");
  AdaNormBwdParams p{};
  p.dh = bfp(dh);
  p.dxe = bf16_ptr_or_null(dxe);
  p.xn = bfp(xn);
  p.rstd = rstd.data_ptr<float>();
  p.w = w.data_ptr<float>();
  p.scale = bf16_ptr_or_null(scale);
  p.mod_bs = row_vec_stride(scale, D);
  p.y = bf16_ptr_or_null(y);
  p.gate = bf16_ptr_or_null(gate);
  p.gate_bs = row_vec_stride(gate, D);
  at::Tensor dx = at::empty_like(dh), dy;
  p.dx = bfp(dx);
  if (p.gate != nullptr && p.y != nullptr) {
    dy = at::empty_like(dh);
    p.dy = bfp(dy);
  }
  p.M = (int)M;
  p.D = (int)D;
  p.T = (int)T;
  p.rows_per_cta = 32;
  p.chunks = (int)((T + p.rows_per_cta - 1) / p.rows_per_cta);
  at::Tensor partial = at::empty({B, p.chunks, 4, D}, dh.options().dtype(at::kFloat));
  p.partial = partial.data_ptr<float>();
  auto fopt = dh.options().dtype(at::kFloat);
  at::Tensor dshift, dscale, dgate;
  if (p.scale != nullptr) {
    dshift = at::empty({B, D}, fopt);
    dscale = at::empty({B, D}, fopt);
  }
  if (p.dy != nullptr) dgate = at::empty({B, D}, fopt);
  TGO_CHECK_LAUNCH_N(adanorm_bwd_launch(p, dshift.defined() ? dshift.data_ptr<float>() : nullptr,
                                      dscale.defined() ? dscale.data_ptr<float>() : nullptr,
                                      dgate.defined() ? dgate.data_ptr<float>() : nullptr, dw.data_ptr<float>(),
                                      at::cuda::getCurrentCUDAStream()), 2);
  return {dx, dy, dshift, dscale, dgate};
}

// ------------------------------------------------------------------------------------------------ q/k norm + rope
static QKNormRopeParams qk_params(const at::Tensor& qkv, int64_t hq, int64_t hkv, int64_t hd,
                                  const c10::optional<at::Tensor>& q_w, const c10::optional<at::Tensor>& k_w,
                                  const c10::optional<at::Tensor>& cos, const c10::optional<at::Tensor>& sin, int64_t T,
                                  double eps) {
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.scalar_type() == at::kBFloat16, "qkv: [M, C] bf16");
  TORCH_CHECK(qkv.size(1) >= (hq + hkv) * hd && qkv.stride(0) % 8 == 0, "qkv: width");
  QKNormRopeParams p{};
  p.qkv = bfp(qkv);
  p.ld_qkv = qkv.stride(0);
  p.q_w = f32_ptr_or_null(q_w);
  p.k_w = f32_ptr_or_null(k_w);
  TORCH_CHECK((p.q_w == nullptr) == (p.k_w == nullptr), "qknorm_rope: q and k norm weights both or neither");
  p.cos = f32_ptr_or_null(cos);
  p.sin = f32_ptr_or_null(sin);
  if (p.cos != nullptr) {
    TORCH_CHECK(cos->size(-1) == hd && cos->size(-2) >= T && sin->sizes() == cos->sizes(), "rope table shape");
    p.rope_bs = cos->dim() == 3 && cos->size(0) > 1 ? cos->stride(0) : 0;
    TORCH_CHECK(cos->size(-2) == T, "rope table must have exactly T rows");
  }
  p.M = (int)qkv.size(0);
  p.T = (int)T;
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.hd = (int)hd;
  p.eps = (float)eps;
  TORCH_CHECK(hd == 64 || hd == 128, "head dim must be 64 or 128");
  TORCH_CHECK(p.M % T == 0, "rows must be a multiple of T");
  return p;
}

std::vector<at::Tensor> qknorm_rope_fwd(at::Tensor qkv, int64_t hq, int64_t hkv, int64_t hd,
                                        c10::optional<at::Tensor> q_w, c10::optional<at::Tensor> k_w,
                                        c10::optional<at::Tensor> cos, c10::optional<at::Tensor> sin, int64_t T,
                                        double eps) {
  const c10::cuda::CUDAGuard guard(qkv.device());
  QKNormRopeParams p = qk_params(qkv, hq, hkv, hd, q_w, k_w, cos, sin, T, eps);
  at::Tensor q = at::empty({qkv.size(0), hq * hd}, qkv.options());
  at::Tensor k = at::empty({qkv.size(0), hkv * hd}, qkv.options());
  at::Tensor rq, rk;
  if (p.q_w != nullptr) rq = at::empty({qkv.size(0), hq}, qkv.options().dtype(at::kFloat));
  if (p.k_w != nullptr) rk = at::empty({qkv.size(0), hkv}, qkv.options().dtype(at::kFloat));
  p.q_out = bfp(q);
  p.ld_q = q.stride(0);
  p.k_out = bfp(k);
  p.ld_k = k.stride(0);
  p.rstd_q = rq.defined() ? rq.data_ptr<float>() : nullptr;
  p.rstd_k = rk.defined() ? rk.data_ptr<float>() : nullptr;
  TGO_CHECK_LAUNCH(qknorm_rope_fwd_launch(p, at::cuda::getCurrentCUDAStream()));
  return {q, k, rq, rk};
}

// dq [M, hq*hd], dk [M, hkv*hd] -> written into dqkv[:, :(hq+hkv)*hd]; dwq / dwk accumulated (+=) when given.
void qknorm_rope_bwd(at::Tensor qkv, int64_t hq, int64_t hkv, int64_t hd, c10::optional<at::Tensor> q_w,
                     c10::optional<at::Tensor> k_w, c10::optional<at::Tensor> cos, c10::optional<at::Tensor> sin,
                     int64_t T, c10::optional<at::Tensor> rstd_q, c10::optional<at::Tensor> rstd_k, at::Tensor dq,
                     at::Tensor dk, at::Tensor dqkv, c10::optional<at::Tensor> dwq, c10::optional<at::Tensor> dwk) {
  const c10::cuda::CUDAGuard guard(qkv.device());
  QKNormRopeParams p = qk_params(qkv, hq, hkv, hd, q_w, k_w, cos, sin, T, 1e-6);
  p.rstd_q = rstd_q.has_value() && rstd_q->defined() ? rstd_q->data_ptr<float>() : nullptr;
  p.rstd_k = rstd_k.has_value() && rstd_k->defined() ? rstd_k->data_ptr<float>() : nullptr;
  // dq: bf16 [M, >= hq hd], or the attention backward's fp32 accumulator [M, hq hd] (read directly)
  TORCH_CHECK(dq.stride(-1) == 1 && dk.stride(-1) == 1 && dqkv.stride(-1) == 1 && dq.stride(0) % 8 == 0 &&
                  dk.stride(0) % 8 == 0 && dqkv.stride(0) % 8 == 0, "qknorm_rope_bwd: layouts (16-byte rows)");
  const bool dq_f32 = dq.scalar_type() == at::kFloat;
  TORCH_CHECK(dq_f32 || dq.scalar_type() == at::kBFloat16, "qknorm_rope_bwd: dq bf16 or fp32");
  TORCH_CHECK(dk.scalar_type() == at::kBFloat16 && dqkv.scalar_type() == at::kBFloat16, "qknorm_rope_bwd: dk / dqkv bf16");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(dq.data_ptr()) % 16 == 0, "qknorm_rope_bwd: dq alignment");
  TGO_CHECK_LAUNCH(qknorm_rope_bwd_launch(p, dq.data_ptr(), dq.stride(0), dq_f32, bfp(dk), dk.stride(0), bfp(dqkv), dqkv.stride(0),
                                          const_cast<float*>(f32_ptr_or_null(dwq)),
                                          const_cast<float*>(f32_ptr_or_null(dwk)), at::cuda::getCurrentCUDAStream()));
}

// ------------------------------------------------------------------------------------------------ swiglu
at::Tensor swiglu_fwd(at::Tensor ab) {
  TORCH_CHECK(ab.is_contiguous() && ab.scalar_type() == at::kBFloat16 && ab.size(-1) % 16 == 0, "swiglu: ab");
  const c10::cuda::CUDAGuard guard(ab.device());
  const int64_t H = ab.size(-1) / 2, M = ab.numel() / ab.size(-1);
  auto sizes = ab.sizes().vec();
  sizes.back() = H;
  at::Tensor g = at::empty(sizes, ab.options());
  TGO_CHECK_LAUNCH(swiglu_fwd_launch(bfp(ab), bfp(g), M, (int)H, at::cuda::getCurrentCUDAStream()));
  return g;
}
at::Tensor swiglu_bwd(at::Tensor ab, at::Tensor dg) {
  TORCH_CHECK(ab.is_contiguous() && dg.is_contiguous(), "swiglu_bwd: contiguous");
  const c10::cuda::CUDAGuard guard(ab.device());
  const int64_t H = ab.size(-1) / 2, M = ab.numel() / ab.size(-1);
  at::Tensor dab = at::empty_like(ab);
  TGO_CHECK_LAUNCH(swiglu_bwd_launch(bfp(ab), bfp(dg), bfp(dab), M, (int)H, at::cuda::getCurrentCUDAStream()));
  return dab;
}

// ------------------------------------------------------------------------------------------------ attention
static void attn_check4(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 4 && t.stride(3) == 1, name,
              ": [B, T, H, hd] bf16 with contiguous head dim");
  TORCH_CHECK(t.stride(0) % 8 == 0 && t.stride(1) % 8 == 0 && t.stride(2) % 8 == 0, name, ": strides % 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, ": 16-byte alignment");
}
static AttnParams attn_params(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                              const c10::optional<at::Tensor>& kv_len, double scale) {
  attn_check4(q, "q");
  attn_check4(k, "k");
  attn_check4(v, "v");
  AttnParams p{};
  p.B = (int)q.size(0);
  p.Tq = (int)q.size(1);
  p.Hq = (int)q.size(2);
  p.hd = (int)q.size(3);
  p.Tk = (int)k.size(1);
  p.Hkv = (int)k.size(2);
  TORCH_CHECK(k.size(0) == p.B && v.sizes() == k.sizes() && k.size(3) == p.hd, "attention: k/v shapes");
  TORCH_CHECK(p.Hq % p.Hkv == 0, "attention: Hq % Hkv");
  TORCH_CHECK(p.hd == 64 || p.hd == 128, "attention: head dim 64 or 128");
  p.rep = p.Hq / p.Hkv;
  p.q = bfp(q);
  p.q_bs = q.stride(0);
  p.q_ts = q.stride(1);
  p.q_hs = q.stride(2);
  p.k = bfp(k);
  p.k_bs = k.stride(0);
  p.k_ts = k.stride(1);
  p.k_hs = k.stride(2);
  p.v = bfp(v);
  p.v_bs = v.stride(0);
  p.v_ts = v.stride(1);
  p.v_hs = v.stride(2);
  p.kv_len = nullptr;
  if (kv_len.has_value() && kv_len->defined()) {
    TORCH_CHECK(kv_len->scalar_type() == at::kInt && kv_len->numel() == p.B && kv_len->is_cuda(), "kv_len: int32 [B]");
    p.kv_len = kv_len->data_ptr<int>();
  }
  p.scale = (float)scale;
  return p;
}

// o: optional preallocated [B, Tq, Hq, hd] output (may be a strided view)
std::vector<at::Tensor> attention_fwd(at::Tensor q, at::Tensor k, at::Tensor v, c10::optional<at::Tensor> kv_len,
                                      double scale, c10::optional<at::Tensor> out, at::Tensor err) {
  const c10::cuda::CUDAGuard guard(q.device());
  AttnParams p = attn_params(q, k, v, kv_len, scale);
  at::Tensor o = out.has_value() && out->defined() ? *out : at::empty({p.B, p.Tq, p.Hq, p.hd}, q.options());
  attn_check4(o, "o");
  at::Tensor lse = at::empty({p.B, p.Hq, p.Tq}, q.options().dtype(at::kFloat));
  p.o = bfp(o);
  p.o_bs = o.stride(0);
  p.o_ts = o.stride(1);
  p.o_hs = o.stride(2);
  p.lse = lse.data_ptr<float>();
  if (g_attention_tc) {
    CUtensorMap tq = make_tmap_bhtd(p.q, p.hd, p.Tq, p.Hq, p.B, p.q_ts, p.q_hs, p.q_bs, 128);
    CUtensorMap tk = make_tmap_bhtd(p.k, p.hd, p.Tk, p.Hkv, p.B, p.k_ts, p.k_hs, p.k_bs, 128);
    CUtensorMap tv = make_tmap_bhtd(p.v, p.hd, p.Tk, p.Hkv, p.B, p.v_ts, p.v_hs, p.v_bs, 128);
    TGO_CHECK_LAUNCH(attention_fwd_tc_launch(tq, tk, tv, p, err_ptr(err), at::cuda::getCurrentCUDAStream()));
  } else {
    TGO_CHECK_LAUNCH(attention_fwd_launch(p, at::cuda::getCurrentCUDAStream()));
  }
  return {o, lse};
}

// Packed variable-length causal / bidirectional attention (inference): q [total, Hq, hd], k / v [total, Hkv, hd],
// cu_seqlens int32 [n + 1] on the device (offsets of the n sequences), max_len = the longest sequence.
// Returns o [total, Hq, hd] and lse [Hq, total].
std::vector<at::Tensor> attention_varlen_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cu_seqlens,
                                             int64_t max_len, double scale, bool causal, at::Tensor err) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(g_attention_tc, "attention_varlen_fwd: needs the tcgen05 attention path");
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.sizes() == k.sizes(), "attention_varlen_fwd: q [T, Hq, hd], k / v [T, Hkv, hd]");
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16, "attention_varlen_fwd: bf16 CUDA tensors");
  TORCH_CHECK(q.stride(2) == 1 && k.stride(2) == 1 && v.stride(2) == 1, "attention_varlen_fwd: unit head-dim stride");
  TORCH_CHECK(k.size(0) == q.size(0) && k.size(2) == q.size(2), "attention_varlen_fwd: q / k token or head-dim mismatch");
  TORCH_CHECK(cu_seqlens.is_cuda() && cu_seqlens.scalar_type() == at::kInt && cu_seqlens.dim() == 1 &&
                  cu_seqlens.numel() >= 2 && cu_seqlens.is_contiguous(), "cu_seqlens: contiguous int32 [n + 1] on the device");
  TORCH_CHECK(max_len > 0 && max_len <= q.size(0), "attention_varlen_fwd: max_len");
  AttnParams p{};
  p.B = (int)cu_seqlens.numel() - 1;
  p.total = (int)q.size(0);
  p.Tq = p.Tk = (int)max_len;
  p.Hq = (int)q.size(1);
  p.Hkv = (int)k.size(1);
  p.hd = (int)q.size(2);
  TORCH_CHECK(p.Hq % p.Hkv == 0 && (p.hd == 64 || p.hd == 128), "attention_varlen_fwd: Hq % Hkv, head dim 64 / 128");
  p.rep = p.Hq / p.Hkv;
  p.q = bfp(q);
  p.q_ts = q.stride(0);
  p.q_hs = q.stride(1);
  p.k = bfp(k);
  p.k_ts = k.stride(0);
  p.k_hs = k.stride(1);
  p.v = bfp(v);
  p.v_ts = v.stride(0);
  p.v_hs = v.stride(1);
  p.scale = (float)scale;
  p.cu_seqlens = cu_seqlens.data_ptr<int>();
  p.causal = causal ? 1 : 0;
  at::Tensor o = at::empty({p.total, p.Hq, p.hd}, q.options());
  at::Tensor lse = at::empty({p.Hq, p.total}, q.options().dtype(at::kFloat));
  p.o = bfp(o);
  p.o_ts = o.stride(0);
  p.o_hs = o.stride(1);
  p.lse = lse.data_ptr<float>();
  CUtensorMap tq = make_tmap_bhtd(p.q, p.hd, p.total, p.Hq, 1, p.q_ts, p.q_hs, 0, 128);
  CUtensorMap tk = make_tmap_bhtd(p.k, p.hd, p.total, p.Hkv, 1, p.k_ts, p.k_hs, 0, 128);
  CUtensorMap tv = make_tmap_bhtd(p.v, p.hd, p.total, p.Hkv, 1, p.v_ts, p.v_hs, 0, 128);
  TGO_CHECK_LAUNCH(attention_fwd_tc_launch(tq, tk, tv, p, err_ptr(err), at::cuda::getCurrentCUDAStream()));
  return {o, lse};
}

// Writes dq, dk, dv (preallocated, possibly strided views). dO must have o's layout.
void attention_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, at::Tensor dO,
                   c10::optional<at::Tensor> kv_len, double scale, at::Tensor dq, at::Tensor dk, at::Tensor dv,
                   at::Tensor err) {
  const c10::cuda::CUDAGuard guard(q.device());
  if (g_attention_tc && q.size(3) == 64) {
    // head dim 64 (the text refiner): the tcgen05 backward on copies zero-padded to head dim 128. Zero columns add
    // nothing to Q K^T, P, delta = rowsum(dO O) or the log-sum-exp of the forward; the gradients' padded columns
    // are dropped. (The mma.sync path remains for set_attention_tc(false).)
    auto pad = [](const at::Tensor& t) { return at::constant_pad_nd(t, {0, 64}).contiguous(); };
    at::Tensor q2 = pad(q), k2 = pad(k), v2 = pad(v), o2 = pad(o), do2 = pad(dO);
    at::Tensor dq2 = at::empty(q2.sizes(), q2.options().dtype(dq.scalar_type()));
    at::Tensor dk2 = at::empty_like(k2), dv2 = at::empty_like(v2);
    attention_bwd(q2, k2, v2, o2, lse, do2, kv_len, scale, dq2, dk2, dv2, err);
    dq.copy_(dq2.narrow(3, 0, 64));
    dk.copy_(dk2.narrow(3, 0, 64));
    dv.copy_(dv2.narrow(3, 0, 64));
    return;
  }
  AttnParams p = attn_params(q, k, v, kv_len, scale);
  attn_check4(o, "o");
  attn_check4(dO, "dO");
  // dq: bf16 [B, T, Hq, hd], or (tcgen05 path) a contiguous fp32 [B, T, Hq, hd] that receives the accumulator
  // itself, so no conversion pass runs (the q/k-norm backward reads the fp32 values)
  const bool dq_f32 = dq.scalar_type() == at::kFloat;
  if (dq_f32) {
    TORCH_CHECK(dq.is_contiguous() && dq.dim() == 4 && dq.size(0) == q.size(0) && dq.size(1) == q.size(1) &&
                    dq.size(2) == q.size(2) && dq.size(3) == q.size(3), "attention_bwd: fp32 dq must be contiguous "
                "[B, T, Hq, hd]");
    if (!(g_attention_tc && q.size(3) == 128)) {  // the mma.sync path converts itself: through a bf16 temporary
      at::Tensor tmp = at::empty(dq.sizes(), dq.options().dtype(at::kBFloat16));
      attention_bwd(q, k, v, o, lse, dO, kv_len, scale, tmp, dk, dv, err);
      dq.copy_(tmp);
      return;
    }
  } else {
    attn_check4(dq, "dq");
  }
  attn_check4(dk, "dk");
  attn_check4(dv, "dv");
  TORCH_CHECK(dO.strides() == o.strides(), "attention_bwd: dO must have o's strides");
  p.o = bfp(o);
  p.o_bs = o.stride(0);
  p.o_ts = o.stride(1);
  p.o_hs = o.stride(2);
  p.lse = lse.data_ptr<float>();
  at::Tensor delta = at::empty({2, p.B, p.Hq, p.Tq}, q.options().dtype(at::kFloat));  // delta, lse * log2(e)
  float* lse2 = delta.data_ptr<float>() + (long long)p.B * p.Hq * p.Tq;
  if (g_attention_tc && p.hd == 128) {
    cudaStream_t st = at::cuda::getCurrentCUDAStream();
    // one key block covers every key (cross-attention against <= 128 text tokens): each dQ tile is final, so it is
    // stored straight into dq (no zeroed accumulator, no reduce-add, no conversion pass)
    const bool single = g_attention_dq_store && p.Tk <= 128;
    const int dq_mode = single ? (dq_f32 ? 1 : 2) : 0;
    at::Tensor dq_acc = dq_f32 || single ? dq : at::empty({p.B, p.Tq, p.Hq, p.hd}, q.options().dtype(at::kFloat));
    CUtensorMap tq = make_tmap_bhtd(p.q, p.hd, p.Tq, p.Hq, p.B, p.q_ts, p.q_hs, p.q_bs, 64);
    CUtensorMap tk = make_tmap_bhtd(p.k, p.hd, p.Tk, p.Hkv, p.B, p.k_ts, p.k_hs, p.k_bs, 128);
    CUtensorMap tv = make_tmap_bhtd(p.v, p.hd, p.Tk, p.Hkv, p.B, p.v_ts, p.v_hs, p.v_bs, 128);
    CUtensorMap tdo = make_tmap_bhtd(dO.data_ptr(), p.hd, p.Tq, p.Hq, p.B, dO.stride(1), dO.stride(2), dO.stride(0), 64);
    TGO_CHECK_LAUNCH(attention_bwd_prep_launch(p, bfp(dO), delta.data_ptr<float>(),
                                               dq_mode == 0 ? dq_acc.data_ptr<float>() : nullptr, st, lse2));
    CUtensorMap tdq = dq_mode == 2 ? make_tmap_dq_bf16(dq.data_ptr(), p.hd, p.Hq, p.Tq, p.B, dq.stride(2),
                                                       dq.stride(1), dq.stride(0))
                                   : make_tmap_dq(dq_acc.data_ptr<float>(), p.hd, p.Hq, p.Tq, p.B);
    TGO_CHECK_LAUNCH(attention_bwd_tc_launch(tq, tk, tv, tdo, tdq, p, delta.data_ptr<float>(), lse2, bfp(dk), dk.stride(0),
                                             dk.stride(1), dk.stride(2), bfp(dv), dv.stride(0), dv.stride(1),
                                             dv.stride(2), err_ptr(err), st, dq_mode));
    if (dq_mode == 0 && !dq_f32)
      TGO_CHECK_LAUNCH(attention_dq_convert_launch(p, dq_acc.data_ptr<float>(), bfp(dq), dq.stride(0), dq.stride(1),
                                                   dq.stride(2), st));
  } else {
    at::Tensor dq_acc = dq_f32 ? dq : at::empty({p.B, p.Tq, p.Hq, p.hd}, q.options().dtype(at::kFloat));
    TGO_CHECK_LAUNCH_N(attention_bwd_launch(p, bfp(dO), delta.data_ptr<float>(), dq_acc.data_ptr<float>(), bfp(dq),
                                          dq.stride(0), dq.stride(1), dq.stride(2), bfp(dk), dk.stride(0), dk.stride(1),
                                          dk.stride(2), bfp(dv), dv.stride(0), dv.stride(1), dv.stride(2),
                                          at::cuda::getCurrentCUDAStream()), 3);
  }
}

// ------------------------------------------------------------------------------------------------ sampler
// z [B, C, H, W] fp32 (in place) += dt * (v_u + w (v_c - v_u)), v from the token-major [2B, H*W, C] output
void euler_cfg(at::Tensor out, at::Tensor z, double dt, double w) {
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.dim() == 3, "euler_cfg: out bf16 [2B,T,C]");
  TORCH_CHECK(z.is_contiguous() && z.scalar_type() == at::kFloat && z.dim() == 4, "euler_cfg: z fp32 [B,C,H,W]");
  const int64_t B = z.size(0), C = z.size(1), T = z.size(2) * z.size(3);
  TORCH_CHECK(out.size(0) == 2 * B && out.size(1) == T && out.size(2) == C, "euler_cfg: shapes");
  const c10::cuda::CUDAGuard guard(z.device());
  TGO_CHECK_LAUNCH(euler_cfg_launch(bfp(out), z.data_ptr<float>(), (int)B, (int)T, (int)C, (float)dt, (float)w,
                                    at::cuda::getCurrentCUDAStream()));
}

std::vector<at::Tensor> fm_inputs(at::Tensor x0, at::Tensor eps, at::Tensor t) {
  TORCH_CHECK(x0.is_cuda() && x0.scalar_type() == at::kFloat && x0.is_contiguous() && x0.dim() == 4,
              "fm_inputs: x0 fp32 [B, C, H, W] contiguous");
  TORCH_CHECK(eps.sizes() == x0.sizes() && eps.scalar_type() == at::kFloat && eps.is_contiguous(), "fm_inputs: eps");
  TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == x0.size(0), "fm_inputs: t fp32 [B]");
  const int64_t B = x0.size(0), C = x0.size(1), T = x0.size(2) * x0.size(3);
  const c10::cuda::CUDAGuard guard(x0.device());
  auto z_tok = at::empty({B, T, C}, x0.options().dtype(at::kBFloat16));
  auto target = at::empty({B, T, C}, x0.options());
  TGO_CHECK_LAUNCH(fm_inputs_launch(x0.data_ptr<float>(), eps.data_ptr<float>(), t.data_ptr<float>(), bfp(z_tok),
                                    target.data_ptr<float>(), (int)B, (int)T, (int)C,
                                    at::cuda::getCurrentCUDAStream()));
  return {z_tok, target};
}

// ------------------------------------------------------------------------------------------------ peer memory
// Device buffers shared between the ranks of one node: allocated with cudaMalloc (zeroed), exported as a CUDA IPC
// handle, opened by the peers.  Pointers travel as integers.
static void cuda_ok(cudaError_t e, const char* what) { TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e)); }

std::tuple<int64_t, py::bytes> symm_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  cuda_ok(cudaMalloc(&p, (size_t)nbytes), "cudaMalloc (peer buffer)");
  cuda_ok(cudaMemset(p, 0, (size_t)nbytes), "cudaMemset (peer buffer)");
  cudaIpcMemHandle_t h;
  cuda_ok(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  return {reinterpret_cast<int64_t>(p), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}
void symm_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  cuda_ok(cudaFree(reinterpret_cast<void*>(ptr)), "cudaFree (peer buffer)");
}
int64_t ipc_open(py::bytes handle, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  std::string hs = handle;
  TORCH_CHECK(hs.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, hs.data(), sizeof(h));
  void* p = nullptr;
  cuda_ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}
void ipc_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  cuda_ok(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle");
}

// In-place bf16-transport average of fp32 grads [n] over `world` ranks through peer buffers.
void allreduce_bf16(at::Tensor grads, std::vector<int64_t> staging, std::vector<int64_t> result,
                    std::vector<int64_t> flags, int64_t rank, int64_t world, int64_t slice, int64_t epoch, double scale,
                    int64_t blocks, int64_t timeout_ns, at::Tensor err) {
  TORCH_CHECK(grads.is_cuda() && grads.scalar_type() == at::kFloat && grads.is_contiguous(), "grads: fp32 CUDA");
  TORCH_CHECK(world >= 1 && world <= kMaxPeers && (int64_t)staging.size() == world &&
              (int64_t)result.size() == world && (int64_t)flags.size() == world, "allreduce: peer lists");
  TORCH_CHECK(slice % 8 == 0 && slice * world >= grads.numel(), "allreduce: slice");
  const c10::cuda::CUDAGuard guard(grads.device());
  PeerAllReduceParams p{};
  p.grads = grads.data_ptr<float>();
  p.n = grads.numel();
  p.slice = slice;
  p.rank = (int)rank;
  p.world = (int)world;
  for (int i = 0; i < world; ++i) {
    p.staging[i] = reinterpret_cast<__nv_bfloat16*>(staging[i]);
    p.result[i] = reinterpret_cast<__nv_bfloat16*>(result[i]);
    p.flags[i] = reinterpret_cast<uint32_t*>(flags[i]);
  }
  p.epoch = (uint32_t)epoch;
  p.scale = (float)scale;
  p.timeout_ns = (unsigned long long)timeout_ns;
  p.err = err_ptr(err);
  TGO_CHECK_LAUNCH(allreduce_bf16_launch(p, (int)blocks, at::cuda::getCurrentCUDAStream()));
}

// Attention pipeline timeline of one CTA (clock64 per phase event and iteration, int64 [32 * 64]); None: off.
void attention_trace(c10::optional<at::Tensor> buf, int64_t cta) {
  long long* ptr = nullptr;
  if (buf.has_value() && buf->defined()) {
    TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == at::kLong && buf->numel() >= 32 * 64, "trace buffer");
    ptr = reinterpret_cast<long long*>(buf->data_ptr<int64_t>());
  }
  TORCH_CHECK(attention_set_trace(ptr, (int)cta) == cudaSuccess, "attention_set_trace failed");
}

// ---- sharded Muon over peer memory (muon_comm.cu) ----
// A bf16 tensor over device memory this process allocated elsewhere (a peer-visible buffer); no ownership.
at::Tensor tensor_from_ptr(int64_t ptr, int64_t n, int64_t device) {
  return at::from_blob(reinterpret_cast<void*>(ptr), {n},
                       at::TensorOptions().dtype(at::kBFloat16).device(at::kCUDA, (c10::DeviceIndex)device));
}

static void peer_list(const std::vector<int64_t>& v, int64_t world, const char* what) {
  TORCH_CHECK(world >= 1 && world <= kMaxPeers && (int64_t)v.size() == world, what, ": one pointer per rank");
}

void muon_rs(at::Tensor grads, std::vector<int64_t> staging, std::vector<int64_t> flags, at::Tensor segs,
             int64_t owned, at::Tensor g_owned, at::Tensor sumsq, int64_t rank, int64_t world, int64_t epoch,
             int64_t prev_epoch, int64_t blocks, int64_t timeout_ns, at::Tensor err) {
  TORCH_CHECK(grads.is_cuda() && grads.scalar_type() == at::kFloat && grads.is_contiguous(), "muon_rs: grads");
  TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == at::kLong && segs.dim() == 2 && segs.size(1) == 3 &&
              segs.is_contiguous(), "muon_rs: segs int64 [n, 3] on the device");
  TORCH_CHECK(g_owned.scalar_type() == at::kFloat && g_owned.is_contiguous() && g_owned.numel() >= owned,
              "muon_rs: g_owned");
  TORCH_CHECK(sumsq.scalar_type() == at::kFloat && sumsq.numel() >= 1, "muon_rs: sumsq");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(grads.data_ptr()) % 16 == 0, "muon_rs: grads must be 16-byte aligned");
  peer_list(staging, world, "muon_rs staging");
  peer_list(flags, world, "muon_rs flags");
  TORCH_CHECK(blocks >= 1 && blocks * world <= kMuonMaxFlags, "muon_rs: blocks");
  const c10::cuda::CUDAGuard guard(grads.device());
  MuonRSParams p{};
  p.grads = grads.data_ptr<float>();
  p.n = grads.numel();
  for (int i = 0; i < world; ++i) {
    p.staging[i] = reinterpret_cast<__nv_bfloat16*>(staging[i]);
    p.flags[i] = reinterpret_cast<uint32_t*>(flags[i]);
  }
  p.segs = reinterpret_cast<const long long*>(segs.data_ptr<int64_t>());
  p.nsegs = (int)segs.size(0);
  p.owned = owned;
  p.g_owned = g_owned.data_ptr<float>();
  p.scale = 1.f / (float)world;
  p.sumsq = sumsq.data_ptr<float>();
  p.rank = (int)rank;
  p.world = (int)world;
  p.epoch = (uint32_t)epoch;
  p.prev_epoch = (uint32_t)prev_epoch;
  p.timeout_ns = (unsigned long long)timeout_ns;
  p.err = err_ptr(err);
  TGO_CHECK_LAUNCH(muon_rs_launch(p, (int)blocks, at::cuda::getCurrentCUDAStream()));
}

void muon_momentum(at::Tensor g, at::Tensor buf, at::Tensor x_out, at::Tensor coef, double mu, bool nesterov,
                   int64_t seed) {
  TORCH_CHECK(coef.is_cuda() && coef.scalar_type() == at::kFloat && coef.numel() == 1, "muon_momentum: coef");
  TORCH_CHECK(g.is_cuda() && g.scalar_type() == at::kFloat && g.is_contiguous(), "muon_momentum: g");
  TORCH_CHECK(buf.is_contiguous() && buf.numel() == g.numel() &&
              (buf.scalar_type() == at::kFloat || buf.scalar_type() == at::kBFloat16), "muon_momentum: buf");
  TORCH_CHECK(x_out.is_contiguous() && x_out.scalar_type() == at::kBFloat16 && x_out.numel() == g.numel(),
              "muon_momentum: x_out");
  const c10::cuda::CUDAGuard guard(g.device());
  MuonMomentumParams p{};
  p.g = g.data_ptr<float>();
  p.n = g.numel();
  if (buf.scalar_type() == at::kFloat) p.buf_f32 = buf.data_ptr<float>();
  else p.buf_bf16 = bfp(buf);
  p.x_out = bfp(x_out);
  p.coef = coef.data_ptr<float>();
  p.mu = (float)mu;
  p.nesterov = nesterov ? 1 : 0;
  p.seed = (unsigned long long)seed;
  TGO_CHECK_LAUNCH(muon_momentum_launch(p, at::cuda::getCurrentCUDAStream()));
}

void muon_ag_apply(std::vector<int64_t> upd, std::vector<int64_t> flags, at::Tensor own, int64_t owned,
                   at::Tensor segs, at::Tensor coefs, double ema_rate, int64_t rank, int64_t world,
                   int64_t epoch, int64_t blocks, int64_t timeout_ns, at::Tensor err) {
  TORCH_CHECK(own.is_cuda() && own.scalar_type() == at::kLong && own.dim() == 2 && own.size(1) == 2 &&
              own.is_contiguous(), "muon_ag_apply: own int64 [n, 2] on the device");
  TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == at::kLong && segs.dim() == 2 && segs.size(1) == 5 &&
              segs.is_contiguous(), "muon_ag_apply: segs int64 [n, 5] on the device");
  TORCH_CHECK(coefs.is_cuda() && coefs.scalar_type() == at::kFloat && coefs.is_contiguous() &&
              coefs.numel() == 2 * segs.size(0), "muon_ag_apply: coefs fp32 [n, 2] on the device");
  peer_list(upd, world, "muon_ag_apply upd");
  peer_list(flags, world, "muon_ag_apply flags");
  TORCH_CHECK(blocks >= 1 && blocks * world <= kMuonMaxFlags, "muon_ag_apply: blocks");
  const c10::cuda::CUDAGuard guard(own.device());
  MuonAGParams p{};
  for (int i = 0; i < world; ++i) {
    p.upd[i] = reinterpret_cast<__nv_bfloat16*>(upd[i]);
    p.flags[i] = reinterpret_cast<uint32_t*>(flags[i]);
  }
  p.own = reinterpret_cast<const long long*>(own.data_ptr<int64_t>());
  p.nown = (int)own.size(0);
  p.owned = owned;
  p.segs = reinterpret_cast<const long long*>(segs.data_ptr<int64_t>());
  p.coefs = coefs.data_ptr<float>();
  p.nsegs = (int)segs.size(0);
  p.ema_rate = (float)ema_rate;
  p.rank = (int)rank;
  p.world = (int)world;
  p.epoch = (uint32_t)epoch;
  p.timeout_ns = (unsigned long long)timeout_ns;
  p.err = err_ptr(err);
  TGO_CHECK_LAUNCH(muon_ag_apply_launch(p, (int)blocks, at::cuda::getCurrentCUDAStream()));
}

// Single-owner Muon step: momentum + Nesterov direction read from the gradients in place (segment table
// (grad ptr, flat offset, length)), and the parameter update + bf16 shadow refresh from the flat updates.
void muon_seg_momentum(at::Tensor segs, at::Tensor buf, at::Tensor x_out, at::Tensor coef, double mu, bool nesterov,
                       int64_t seed, int64_t blocks) {
  TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == at::kLong && segs.dim() == 2 && segs.size(1) == 3 &&
              segs.is_contiguous(), "muon_seg_momentum: segs int64 [n, 3] on the device");
  TORCH_CHECK(coef.is_cuda() && coef.scalar_type() == at::kFloat && coef.numel() == 1, "muon_seg_momentum: coef");
  TORCH_CHECK(buf.is_cuda() && buf.is_contiguous() &&
              (buf.scalar_type() == at::kFloat || buf.scalar_type() == at::kBFloat16), "muon_seg_momentum: buf");
  TORCH_CHECK(x_out.is_cuda() && x_out.is_contiguous() && x_out.scalar_type() == at::kBFloat16 &&
              x_out.numel() == buf.numel(), "muon_seg_momentum: x_out");
  TORCH_CHECK(blocks >= 1 && blocks <= 65535, "muon_seg_momentum: blocks");
  const c10::cuda::CUDAGuard guard(buf.device());
  MuonSegMomentumParams p{};
  p.segs = reinterpret_cast<const long long*>(segs.data_ptr<int64_t>());
  p.nsegs = (int)segs.size(0);
  if (buf.scalar_type() == at::kFloat) p.buf_f32 = buf.data_ptr<float>();
  else p.buf_bf16 = bfp(buf);
  p.x_out = bfp(x_out);
  p.coef = coef.data_ptr<float>();
  p.mu = (float)mu;
  p.nesterov = nesterov ? 1 : 0;
  p.seed = (unsigned long long)seed;
  TGO_CHECK_LAUNCH(muon_seg_momentum_launch(p, (int)blocks, at::cuda::getCurrentCUDAStream()));
}

void muon_apply(at::Tensor upd, at::Tensor segs, at::Tensor coefs, double ema_rate, int64_t blocks) {
  TORCH_CHECK(upd.is_cuda() && upd.is_contiguous() && upd.scalar_type() == at::kBFloat16, "muon_apply: upd");
  TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == at::kLong && segs.dim() == 2 && segs.size(1) == 5 &&
              segs.is_contiguous(), "muon_apply: segs int64 [n, 5] on the device");
  TORCH_CHECK(coefs.is_cuda() && coefs.scalar_type() == at::kFloat && coefs.is_contiguous() &&
              coefs.numel() == 2 * segs.size(0), "muon_apply: coefs fp32 [n, 2] on the device");
  TORCH_CHECK(blocks >= 1 && blocks <= 65535, "muon_apply: blocks");
  const c10::cuda::CUDAGuard guard(upd.device());
  MuonApplyParams p{};
  p.upd = bfp(upd);
  p.segs = reinterpret_cast<const long long*>(segs.data_ptr<int64_t>());
  p.coefs = coefs.data_ptr<float>();
  p.nsegs = (int)segs.size(0);
  p.ema_rate = (float)ema_rate;
  TGO_CHECK_LAUNCH(muon_apply_launch(p, (int)blocks, at::cuda::getCurrentCUDAStream()));
}

// Global gradient norm and clip coefficient on the device (one launch; see optim.cu).
void grad_norm(at::Tensor segs, at::Tensor acc, at::Tensor counter, c10::optional<at::Tensor> extra, double clip,
               at::Tensor gnorm, at::Tensor coef, int64_t blocks) {
  TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == at::kLong && segs.dim() == 2 && segs.size(1) == 2 &&
              segs.is_contiguous(), "grad_norm: segs int64 [n, 2] on the device");
  for (const at::Tensor* t : {&acc, &gnorm, &coef})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->numel() >= 1, "grad_norm: fp32 scalars");
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == at::kInt && counter.numel() >= 1, "grad_norm: counter");
  TORCH_CHECK(blocks >= 1 && blocks <= 65535, "grad_norm: blocks");
  const c10::cuda::CUDAGuard guard(acc.device());
  GradNormParams p{};
  p.segs = reinterpret_cast<const long long*>(segs.data_ptr<int64_t>());
  p.nsegs = (int)segs.size(0);
  p.acc = acc.data_ptr<float>();
  p.counter = reinterpret_cast<unsigned int*>(counter.data_ptr<int>());
  if (extra.has_value() && extra->defined()) {
    TORCH_CHECK(extra->is_cuda() && extra->scalar_type() == at::kFloat, "grad_norm: extra");
    p.extra_sumsq = extra->data_ptr<float>();
  }
  p.clip = (float)clip;
  p.gnorm = gnorm.data_ptr<float>();
  p.coef = coef.data_ptr<float>();
  TGO_CHECK_LAUNCH(grad_norm_launch(p, (int)blocks, at::cuda::getCurrentCUDAStream()));
}

// Multi-tensor AdamW with the clip coefficient, bf16 shadow refresh and EMA fused in (see optim.cu).
void adamw(at::Tensor segs, at::Tensor hyper, c10::optional<at::Tensor> coef, double ema_rate, int64_t blocks) {
  TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == at::kLong && segs.dim() == 2 && segs.size(1) == 8 &&
              segs.is_contiguous(), "adamw: segs int64 [n, 8] on the device");
  TORCH_CHECK(hyper.is_cuda() && hyper.scalar_type() == at::kFloat && hyper.dim() == 2 && hyper.size(1) == 6 &&
              hyper.is_contiguous(), "adamw: hyper fp32 [groups, 6] on the device");
  TORCH_CHECK(blocks >= 1 && blocks <= 65535, "adamw: blocks");
  const c10::cuda::CUDAGuard guard(segs.device());
  AdamWParams p{};
  p.segs = reinterpret_cast<const long long*>(segs.data_ptr<int64_t>());
  p.nsegs = (int)segs.size(0);
  p.hyper = hyper.data_ptr<float>();
  if (coef.has_value() && coef->defined()) {
    TORCH_CHECK(coef->is_cuda() && coef->scalar_type() == at::kFloat, "adamw: coef");
    p.coef = coef->data_ptr<float>();
  }
  p.ema_rate = (float)ema_rate;
  TGO_CHECK_LAUNCH(adamw_launch(p, (int)blocks, at::cuda::getCurrentCUDAStream()));
}

// src (contiguous CUDA tensor) -> dst (a peer's mapped buffer), then dst_version := version (see comm.cu)
void peer_copy(int64_t dst, at::Tensor src, int64_t dst_version, int64_t counter, int64_t version, int64_t blocks) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "peer_copy: contiguous CUDA source");
  const c10::cuda::CUDAGuard guard(src.device());
  TGO_CHECK_LAUNCH(peer_copy_launch(reinterpret_cast<void*>(dst), src.data_ptr(), src.numel() * src.element_size(),
                                    reinterpret_cast<uint32_t*>(dst_version),
                                    reinterpret_cast<unsigned long long*>(counter), (uint32_t)version, (int)blocks,
                                    at::cuda::getCurrentCUDAStream()));
}

}  // namespace tgo

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels: tcgen05 GEMM, fused norms, attention, optimizer and comm kernels";
  m.def("gemm", &tgo::gemm, "tcgen05 bf16 GEMM: C = alpha * op(A) op(B)^T (+ beta D)", py::arg("A"), py::arg("B"),
        py::arg("C"), py::arg("a_mn"), py::arg("b_mn"), py::arg("D") = c10::nullopt, py::arg("alpha") = 1.0,
        py::arg("beta") = 0.0, py::arg("accumulate") = false, py::arg("err"));
  m.def("fm_inputs", &tgo::fm_inputs, "flow-matching input (bf16) and target (fp32), token-major, in one pass");
  m.def("euler_cfg", &tgo::euler_cfg, "fused classifier-free-guidance Euler step from token-major velocities");
  m.def("symm_alloc", &tgo::symm_alloc, "zeroed device buffer + its CUDA IPC handle");
  m.def("symm_free", &tgo::symm_free);
  m.def("ipc_open", &tgo::ipc_open, "map a peer's buffer from its IPC handle");
  m.def("ipc_close", &tgo::ipc_close);
  m.def("peer_copy", &tgo::peer_copy, "NVLink copy into a peer's buffer + version word (weight snapshots)");
  m.def("allreduce_bf16", &tgo::allreduce_bf16, "fused cast + reduce-scatter + all-gather over peer memory");
  m.def("attention_trace", &tgo::attention_trace, "install / remove the attention timeline buffer (profiling)");
  m.def("tensor_from_ptr", &tgo::tensor_from_ptr, "bf16 view of raw device memory (not owned)");
  m.def("muon_rs", &tgo::muon_rs, "sharded Muon: gradient bucket reduce-scatter to the matrix owners (NVLink)");
  m.def("muon_momentum", &tgo::muon_momentum, "sharded Muon: owner momentum + Nesterov -> bf16 NS input");
  m.def("muon_ag_apply", &tgo::muon_ag_apply, "sharded Muon: update all-gather fused with the parameter update");
  m.def("muon_seg_momentum", &tgo::muon_seg_momentum, "Muon: momentum + Nesterov from the gradients in place");
  m.def("muon_apply", &tgo::muon_apply, "Muon: parameter update + bf16 shadow refresh from the flat updates");
  m.def("grad_norm", &tgo::grad_norm, "global gradient norm and clip coefficient on the device (one launch)");
  m.def("adamw", &tgo::adamw, "multi-tensor AdamW with clip coefficient, bf16 shadow refresh and EMA fused in");
  m.def("set_attention_dq_store", &tgo::set_attention_dq_store,
        "attention backward with one key block: store the final dQ tiles (default) or reduce-add into a zeroed accumulator");
  m.def("set_attention_poll", &tgo::set_attention_poll,
        "attention barrier waits that poll instead of suspending, forward and backward masks (bit 0 MMA thread, "
        "1 softmax / dQ drain, 2 TMA producer; defaults 3 and 1)",
        py::arg("fwd_mask"), py::arg("bwd_mask") = -1);
  m.def("set_attention_fwd_pingpong", &tgo::set_attention_fwd_pingpong,
        "attention forward: the two softmax groups take turns for their exponential phases");
  m.def("set_attention_fwd_emu", &tgo::set_attention_fwd_emu,
        "eighths of the key pairs whose forward exponentials run as FMA-pipe polynomials (0 .. 4)");
  m.def("set_attention_fwd_split", &tgo::set_attention_fwd_split,
        "softmax warps per TMEM lane quarter in the tcgen05 attention forward (1 or 2)");
  m.def("set_attention_tc", &tgo::set_attention_tc, "use the tcgen05 attention forward (default) or mma.sync");
  m.def("set_gemm_tma_epilogue", &tgo::set_gemm_tma_epilogue,
        "GEMM epilogue through TMA stores / reduce-adds (default) or per-row global stores");
  m.def("set_qknorm_bwd_unroll", [](int64_t u) { TORCH_CHECK(tgo::qknorm_set_bwd_unroll((int)u) == cudaSuccess, "2 or 4"); },
        "q/k-norm + RoPE backward: heads in flight per lane group (A/B runs)");
  m.def("set_gemm_splitk", &tgo::set_gemm_splitk, "enable / disable split-K of the fp32-accumulating GEMMs (A/B runs)");
  m.def("set_adanorm_bwd_rows", &tgo::set_adanorm_bwd_rows, "adanorm backward: rows per block reduction (1 or 2)");
  m.def("set_gemm_tail_split", &tgo::set_gemm_tail_split,
        "2-CTA GEMM: run a last wave that fills at most half of the SM pairs as half-width tiles (off by default: measured slower)");
  m.def("set_gemm_poll", &tgo::set_gemm_poll,
        "GEMM barrier waits poll instead of suspending (bit 0 MMA thread, 1 epilogue, 2 TMA producer)");
  m.def("gemm_i8", &tgo::gemm_i8, "int8 W8A8 GEMM on tcgen05 kind::i8: C = (A B^T) * a_scale[m] * b_scale[n] (bf16)",
        py::arg("A"), py::arg("B"), py::arg("C"), py::arg("a_scale"), py::arg("b_scale"), py::arg("err"));
  m.def("quantize_rows_i8", &tgo::quantize_rows_i8, "per-row symmetric int8 quantisation of bf16 rows -> (q, scale)");
  m.def("set_gemm_syrk", &tgo::set_gemm_syrk, "enable / disable the symmetric (lower-triangle) GEMM mode (A/B runs)");
  m.def("gemm_syrk", &tgo::gemm_syrk, "symmetric C = alpha A A^T + beta D: lower-triangle tiles, mirrored stores");
  m.def("set_gemm_pair", &tgo::set_gemm_pair, "enable / disable the 2-CTA GEMM kernel (for A/B tests)");
  m.def("launch_count", &tgo::launch_count, "kernels launched by this extension so far");
  m.def("adanorm_fwd", &tgo::adanorm_fwd, "x_new = x + gate*y; h = rmsnorm(x_new)*w*(1+scale)+shift");
  m.def("adanorm_bwd", &tgo::adanorm_bwd, "backward of adanorm_fwd");
  m.def("qknorm_rope_fwd", &tgo::qknorm_rope_fwd, "per-head RMSNorm + RoPE of q and k from the qkv rows");
  m.def("qknorm_rope_bwd", &tgo::qknorm_rope_bwd, "backward of qknorm_rope_fwd into dqkv");
  m.def("swiglu_fwd", &tgo::swiglu_fwd, "silu(a) * b");
  m.def("swiglu_bwd", &tgo::swiglu_bwd, "backward of swiglu_fwd");
  m.def("attention_fwd", &tgo::attention_fwd, "flash attention forward (GQA, key-length mask)");
  m.def("attention_bwd", &tgo::attention_bwd, "flash attention backward");
  m.def("gemm_swiglu", &tgo::gemm_swiglu, "up projection + SwiGLU in one GEMM (gate / up rows interleaved)");
  m.def("gemm_grouped", &tgo::gemm_grouped, "grouped GEMM with a device-side tile schedule (MoE experts)");
  m.def("gemm_peer", &tgo::gemm_peer, "MoE expert GEMM: wait for peer-dispatched A rows, or scatter C to peers");
  m.def("moe_dispatch", &tgo::moe_dispatch, "MoE dispatch: token gather + stores into the owners' receive buffers");
  m.def("moe_combine", &tgo::moe_combine, "MoE combine: weighted gather-sum of the rows the owners returned");
  m.def("moe_release", &tgo::moe_release, "MoE: release this rank's receive rows to every source");
  m.def("attention_varlen_fwd", &tgo::attention_varlen_fwd,
        "packed variable-length (optionally causal) attention forward on tcgen05");
}
