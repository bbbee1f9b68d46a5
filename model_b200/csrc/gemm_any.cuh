// Strided float32 GEMMs of the layer backward on the tensor cores (gemm_any.cu).
#pragma once

#include "common.cuh"

namespace ml {

struct GemmScratch {
  float* p;       // 256-byte aligned
  size_t floats;
};

// Scratch floats launch_gemm_any needs for these shapes (0: it runs on the SIMT path).
size_t gemm_any_scratch_floats(int64_t M, int64_t N, int64_t K);

// C[i ldc + j] (+)= sum_k A(i, k) B(k, j), A(i, k) = A[i sai + k sak],
// B(k, j) = B[k sbk + j sbj]; any strides.
cudaError_t launch_gemm_any(const float* A, int64_t sai, int64_t sak, const float* B, int64_t sbk, int64_t sbj,
                            float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, bool accumulate,
                            const GemmScratch& sc, int* err, cudaStream_t s);

// out[j] = sum over rows of X[r ld + j], deterministic (part: colsum_scratch_floats(cols)).
size_t colsum_scratch_floats(int64_t cols);
cudaError_t launch_colsum_det(const float* X, int64_t rows, int64_t cols, int64_t ld, float* part, float* out,
                              cudaStream_t s);

}  // namespace ml
