// Launch interfaces of the sm_100a kernels.  Plain CUDA types only: the torch-facing argument checks live in
// ops.cpp, so the .cu files compile without the torch headers.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tgo {

int num_sms();

// ---------------------------------------------------------------- GEMM (gemm.cu)
struct GemmParams {
  int M, N, K, batch;
  void* C;
  long long ldc, bsc;  // elements
  const __nv_bfloat16* D;
  long long ldd, bsd;
  float alpha, beta;
  int* err;
};
// epi: 0 = bf16 store, 1 = fp32 store, 2 = fp32 accumulate (C += alpha * A B^T)
cudaError_t gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int bn, bool a_mn,
                        bool b_mn, int epi, cudaStream_t s);

}  // namespace tgo
