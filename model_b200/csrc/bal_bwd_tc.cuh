// Balance-term backward on the tensor cores (bal_bwd_tc.cu).
#pragma once

#include "common.cuh"

namespace ml {

// Token slices of the transposed d cos and the scratch sizes (floats).
struct BalBwdPlan {
  int S;          // token slices
  int Ks;         // tokens per slice (a multiple of 128)
  int m_tiles;    // 128-token tiles per codebook, S * Ks / 128
  int64_t q_floats, k_floats, qt_floats, dct_floats, part_floats;
};

struct BalBwdBufs {
  const float* qn;       // [M][H*2][half] unit queries
  const float* q_hi;     // [H*2][M][half] their tf32 halves, codebook-major
  const float* q_lo;
  const float* keys_n;   // [H*2][n][half] unit sub-keys
  const float* k_hi;     // tf32 halves of keys_n
  const float* k_lo;
  float* kt_hi;          // [H*2][half][n] scratch
  float* kt_lo;
  float* qt_hi;          // [S][H*2*half][Ks] scratch
  float* qt_lo;
  float* dct_hi;         // [S][H*2][n][Ks] scratch
  float* dct_lo;
  float* part;           // [S][H*2][n][half] scratch
  const float* cnt;      // [H*2][n] the forward's clean top-k counts
  const float* qlen;     // [M][H*2]
  const float* scal;     // [1] temperature
  float* dqbal;          // [M][H*2][half] (= d cos K_hat)
  float* dkhat;          // [H*2][n][half] (= d cos^T Q_hat)
  float* dT_row;         // [H*2][M]
  float* dql_row;        // [M][H*2] or nullptr
  int* err;              // status word (bounded waits: 17-19)
};

bool bal_bwd_tc_supported(const Dims& D);
BalBwdPlan bal_bwd_plan(const Dims& D, int sms);
cudaError_t launch_bal_bwd_tc(const Dims& D, const BalBwdPlan& P, const BalBwdBufs& B, float coef, cudaStream_t s);

}  // namespace ml
