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

// C[i ldc + j] (+)= sum_k A(i, k) B(k, j) (+ bias[j]), A(i, k) = A[i sai + k sak],
// B(k, j) = B[k sbk + j sbj]; any strides.
cudaError_t launch_gemm_any(const float* A, int64_t sai, int64_t sak, const float* B, int64_t sbk, int64_t sbj,
                            float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, bool accumulate,
                            const GemmScratch& sc, int* err, cudaStream_t s, const float* bias = nullptr);

// dst[s][r][kk] (rows_pad rows per slice) = tf32 hi / lo of src[r s_row + k s_col],
// k = s Ks + kk (zero for k >= cols); `batch` such copies, src + z src_b -> dst + z dst_b.
cudaError_t launch_gather_split(const float* src, int64_t rows, int64_t cols, int64_t s_row, int64_t s_col,
                                int64_t Ks, int S, int64_t rows_pad, float* hi, float* lo, int batch, int64_t src_b,
                                int64_t dst_b, cudaStream_t s);

// C[i ldc + j] (+)= sum over s < S of P[s][i][j] (P: S blocks of M x N), slices in order (+ bias[j]).
cudaError_t launch_sum_slices(const float* P, int S, int64_t M, int64_t N, float* C, int64_t ldc, bool accumulate,
                              cudaStream_t s, const float* bias = nullptr);

// The GEMM that splits its operands itself (gemm_raw_tc.cu): A(i, k) =
// A[i sai + k sak], B(k, j) = B[k sbk + j sbj], each with one unit stride.
// Slice s of S (kq_slice 32-element K stages each) writes
// out + s out_stride (row pitch ld), + bias and accumulated when asked.
// batch > 1: `batch` products, product b on A rows [b M, +M) and B rows
// [b N, +N) (the "row" index i of A, j of B), writing C + b c_boff; M a
// multiple of 128 and N of the column tile.  a_rows / b_rows: the operands'
// total rows (0: batch M / batch N).
int gemm_raw_bn(int64_t N);
// K slices (S) and 32-element stages per slice (per) for `tiles` output tiles
// over kq stages, partials of out_elems floats each within cap floats.
void raw_slices(int64_t tiles, int64_t kq, int64_t out_elems, int sms, size_t cap, int64_t* S, int64_t* per);
bool gemm_raw_supported(const float* A, int64_t sai, int64_t sak, const float* B, int64_t sbk, int64_t sbj,
                        int64_t M, int64_t N, int64_t K);
cudaError_t launch_gemm_raw(const float* A, int64_t sai, int64_t sak, const float* B, int64_t sbk, int64_t sbj,
                            int64_t M, int64_t N, int64_t K, int S, int kq_slice, float* out, int64_t out_stride,
                            int64_t ld, const float* bias, bool accumulate, int* err, cudaStream_t s, int batch = 1,
                            int64_t a_rows = 0, int64_t b_rows = 0, int64_t c_boff = 0);

// out[j] = sum over rows of X[r ld + j], deterministic (part: colsum_scratch_floats(cols)).
size_t colsum_scratch_floats(int64_t cols);
cudaError_t launch_colsum_det(const float* X, int64_t rows, int64_t cols, int64_t ld, float* part, float* out,
                              cudaStream_t s);

}  // namespace ml
