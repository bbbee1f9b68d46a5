// Balance-term backward on the tensor cores (bal_bwd_tc.cu).
#pragma once

#include "common.cuh"

namespace ml {

// Layout of the transposed d cos, the d k_hat GEMM's slices and the scratch sizes (floats).
struct BalBwdPlan {
  int m_tiles;    // 128-token tiles
  int64_t Mp;     // row pitch of the transposed d cos (m_tiles * 128)
  int S;          // K slices of the d k_hat GEMM
  int kq_slice;   // 32-token K stages per slice
  int64_t q_floats, k_floats, dct_floats, part_floats;
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
  float* dct;            // [H*2][n][Mp] scratch: d cos, transposed
  float* part;           // [S][H*2][n][half] scratch (S > 1)
  const float* cnt;      // [H*2][n] the forward's clean top-k counts
  const float* qlen;     // [M][H*2]
  const float* scal;     // [1] temperature
  float* dqbal;          // [M][H*2][half] (= d cos K_hat)
  float* dkhat;          // [H*2][n][half] (= d cos^T Q_hat)
  float* dT_row;         // [H*2][M]
  float* dql_row;        // [M][H*2] or nullptr
  int* err;              // status word (bounded waits: 17-19)
  const int* ent_slot;   // [M][H*2][k] the routing backward's (codebook * n + sub-key) entries ...
  const float* ent_w;    // ... and their d cos (0: padding), added into the d cos matrix
};

bool bal_bwd_tc_supported(const Dims& D);
BalBwdPlan bal_bwd_plan(const Dims& D, int sms);
cudaError_t launch_bal_bwd_tc(const Dims& D, const BalBwdPlan& P, const BalBwdBufs& B, float coef, cudaStream_t s);

}  // namespace ml
