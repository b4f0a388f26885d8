// Torch-facing wrappers of the sm_100a kernels: argument checks, TMA descriptor encoding, launches on the current
// stream.  Exposed as the extension module trenowanie_generatora_obrazkow_b200._C.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "kernels.h"

namespace tgo {

#define TGO_CHECK_LAUNCH(expr)                                                             \
  do {                                                                                     \
    cudaError_t _e = (expr);                                                               \
    TORCH_CHECK(_e == cudaSuccess, "kernel launch failed: ", cudaGetErrorString(_e));      \
  } while (0)

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
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
  const int bn = N <= 128 ? 128 : 256;
  const uint64_t bsA = batched ? A.stride(0) : 0, bsB = batched ? B.stride(0) : 0;
  CUtensorMap ta = make_tmap_bf16_sw128(A.data_ptr(), A.size(-1), A.size(-2), batch, A.stride(-2), bsA,
                                        a_mn ? 64 : 128);
  CUtensorMap tb = make_tmap_bf16_sw128(B.data_ptr(), B.size(-1), B.size(-2), batch, B.stride(-2), bsB,
                                        b_mn ? 64 : bn);
  GemmParams p;
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
  if (D.has_value() && D->defined()) {
    TORCH_CHECK(!out_f32 && D->scalar_type() == at::kBFloat16 && D->stride(-1) == 1, "gemm: D must be bf16");
    TORCH_CHECK(D->dim() == C.dim() && D->size(-2) == M && D->size(-1) == N, "gemm: D shape mismatch");
    TORCH_CHECK(D->stride(-2) % 8 == 0 && reinterpret_cast<uintptr_t>(D->data_ptr()) % 16 == 0, "gemm: D align");
    p.D = reinterpret_cast<const __nv_bfloat16*>(D->data_ptr());
    p.ldd = D->stride(-2);
    p.bsd = batched ? D->stride(0) : 0;
  }
  TORCH_CHECK(p.ldc % 8 == 0 && reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0, "gemm: C alignment");
  p.alpha = (float)alpha;
  p.beta = (float)beta;
  p.err = err_ptr(err);
  const int epi = out_f32 ? (accumulate ? 2 : 1) : 0;
  TGO_CHECK_LAUNCH(gemm_launch(ta, tb, p, bn, a_mn, b_mn, epi, at::cuda::getCurrentCUDAStream()));
}

}  // namespace tgo

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels: tcgen05 GEMM, fused norms, attention, optimizer and comm kernels";
  m.def("gemm", &tgo::gemm, "tcgen05 bf16 GEMM: C = alpha * op(A) op(B)^T (+ beta D)", py::arg("A"), py::arg("B"),
        py::arg("C"), py::arg("a_mn"), py::arg("b_mn"), py::arg("D") = c10::nullopt, py::arg("alpha") = 1.0,
        py::arg("beta") = 0.0, py::arg("accumulate") = false, py::arg("err"));
}
