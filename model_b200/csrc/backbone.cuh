// Kernels of the language model around the memory layer (backbone.cu) and
// the general Dense layer they use (gemm_tc.cu / prep.cu).
#pragma once

#include "common.cuh"

namespace ml {

bool attn_supported(int head_dim);
bool ln_supported(int d_model);   // 32, 64, 128, 256, 512 or 1024
cudaError_t launch_embed(const int* tokens, int64_t M, int T, const int* pos, const float* E, const float* Pe, int V,
                         int dm, int max_len, float* x, int* err, cudaStream_t s);
cudaError_t launch_add_ln(float* x, const float* y, const float* scale, const float* bias, float* h, int64_t M, int dm,
                          cudaStream_t s);
cudaError_t launch_attn_prefill(const float* qkv, float* out, int64_t B, int T, int H, int DH, cudaStream_t s);
cudaError_t launch_attn_decode(const float* qkv, float* cache_k, float* cache_v, const int* pos, int max_len,
                               int64_t B, int H, int DH, float* out, int* err, cudaStream_t s);
cudaError_t launch_merge_status(const int* from, int* to, cudaStream_t s);
cudaError_t launch_add(float* y, const float* z, int64_t n, cudaStream_t s);
// C [M, N] = h [M, K] . E [N, K]^T (K <= 1536), SIMT.
cudaError_t launch_logits_gemv(const float* h, const float* E, float* C, int64_t M, int N, int K, cudaStream_t s);

// Dense activations: none, SiLU, GELU (tanh approximation, flax's nn.gelu).
enum { ACT_NONE = 0, ACT_SILU = 1, ACT_GELU = 2 };
// C [M, N] = act(A [M, K] . B [K, N] + bias), SIMT float32 (any shape; GEMV for few rows).
cudaError_t launch_gemm_act(const float* A, const float* B, const float* bias, float* C, int64_t M, int N, int K,
                            int act, cudaStream_t s);
// The tensor-core (3xTF32) form: A as tf32 halves [M, K], the weight as
// tf32 halves of its transpose [N, K].  bias may be NULL; act NONE or GELU.
bool dense_tc_supported(int64_t M, int K, int N);
// Column tile of the tensor-core GEMM for N output columns.
int dense_tc_bn(int N);
// `slices` independent products in one launch (a split inner dimension):
// slice s multiplies A rows [s m_pad, +M) by B rows [s n_pad, +N) (K each)
// into C + s M N, no bias.  m_pad a multiple of 128, n_pad of the column tile.
cudaError_t launch_dense_tc_sliced(const float* a_hi, const float* a_lo, int64_t M, int64_t m_pad, int K,
                                   const float* bt_hi, const float* bt_lo, int N, int64_t n_pad, int slices,
                                   float* C, int* err, cudaStream_t s);
// accumulate: C += A B^T + bias (no activation)
cudaError_t launch_dense_tc(const float* a_hi, const float* a_lo, int64_t M, int K, const float* bt_hi,
                            const float* bt_lo, int N, const float* bias, float* C, int act, int* err,
                            cudaStream_t s, bool accumulate = false);

}  // namespace ml
