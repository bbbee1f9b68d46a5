// The float32 GEMMs of the layer backward (model.py:110-119 and the balance
// term of memory.py:205-214 differentiated): C (+)= op(A) op(B) with any
// row / column strides, on the 5th-generation tensor cores through the
// 3xTF32 GEMM of gemm_tc.cu.
//
//   0. operands whose rows or whose k run contiguously (16-byte aligned,
//      at least one tile) go to gemm_raw_tc.cu, which loads them as stored
//      and splits them inside the GEMM -- unless its tiles would convert the
//      operands over six times over (short K, many tiles both ways: the
//      recomputed router projection); otherwise:
//   1. both operands are gathered into K-major tf32 hi / lo halves in the
//      caller's scratch (32 x 32 tiles through shared memory, so either
//      stride order reads coalesced), zero-padded to a multiple of the K
//      stage;
//   2. a long inner dimension with few output tiles (the weight and sub-key
//      gradients sum over every token) is cut into S slices that run as
//      separate GEMM tiles, filling the SMs;
//   3. the S partial products are added in slice order (deterministic) into
//      C, on top of C's contents when accumulating.
// Shapes the tensor-core GEMM does not take (fewer than 128 rows, a column
// count that is not a multiple of 16) run on a float32 SIMT GEMM with the
// same strides.
#include <algorithm>

#include "backbone.cuh"
#include "gemm_any.cuh"
#include "tc_common.cuh"

namespace ml {

namespace {

constexpr int KQ = 32;   // K stage of the tensor-core GEMM

// dst[s][r][kk] (rows_pad rows per slice) = tf32 halves of
// src[r * s_row + k * s_col], k = s * Ks + kk, zero for k >= cols.
// blockIdx.z: batch (src + z src_b, hi / lo + z dst_b).
__global__ void __launch_bounds__(256) gather_split_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                                                           int64_t s_row, int64_t s_col, int64_t Ks, int S,
                                                           int64_t rows_pad, float* __restrict__ hi,
                                                           float* __restrict__ lo, int64_t src_b, int64_t dst_b) {
  __shared__ float t[32][33];
  src += blockIdx.z * src_b;
  hi += blockIdx.z * dst_b;
  lo += blockIdx.z * dst_b;
  const int64_t r0 = (int64_t)blockIdx.y * 32, k0 = (int64_t)blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8
  if (s_col == 1) {          // rows contiguous along k: lanes over k
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + i, k = k0 + tx;
      t[i][tx] = (r < rows && k < cols) ? src[r * s_row + k] : 0.f;
    }
  } else {                   // columns contiguous along r: lanes over r
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + tx, k = k0 + i;
      t[tx][i] = (r < rows && k < cols) ? src[r * s_row + k * s_col] : 0.f;
    }
  }
  __syncthreads();
  const int64_t kp = (int64_t)S * Ks;
  for (int i = ty; i < 32; i += 8) {
    const int64_t r = r0 + i, k = k0 + tx;
    if (r >= rows || k >= kp) continue;
    const int64_t sl = k / Ks, kk = k - sl * Ks;
    const float v = t[i][tx];
    const float h = tc::to_tf32(v);
    const int64_t at = (sl * rows_pad + r) * Ks + kk;
    hi[at] = h;
    lo[at] = tc::to_tf32(v - h);
  }
}

// C[i ldc + j] = (acc ? C : 0) + (bias ? bias[j] : 0) + sum_s P[s][i][j], slices in order.
__global__ void __launch_bounds__(256) sum_slices_kernel(const float* __restrict__ P, int S, int64_t M, int64_t N,
                                                         float* __restrict__ C, int64_t ldc, int acc,
                                                         const float* __restrict__ bias) {
  const int64_t n = M * N;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / N, j = e - i * N;
    float x = 0.f;
    for (int s0 = 0; s0 < S; s0 += 8) {   // up to eight loads in flight, added in slice order
      float a[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) a[q] = s0 + q < S ? P[(int64_t)(s0 + q) * n + e] : 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (s0 + q < S) x += a[q];
    }
    if (bias) x += bias[j];
    float* c = C + i * ldc + j;
    *c = acc ? *c + x : x;
  }
}

// SIMT float32 GEMM with strides: 64 x 64 tile, 4 x 4 outputs per thread.
constexpr int SB = 64, SK = 16;
__global__ void __launch_bounds__(256) gemm_strided_simt_kernel(const float* __restrict__ A, int64_t sai, int64_t sak,
                                                                const float* __restrict__ B, int64_t sbk,
                                                                int64_t sbj, float* __restrict__ C, int64_t ldc,
                                                                int64_t M, int64_t N, int64_t K, int acc,
                                                                const float* __restrict__ bias) {
  __shared__ float As[SK][SB + 4];
  __shared__ float Bs[SK][SB + 4];
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const int64_t m0 = (int64_t)blockIdx.y * SB, n0 = (int64_t)blockIdx.x * SB;
  float c[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += SK) {
    for (int e = tid; e < SB * SK; e += 256) {
      const int mi = sak == 1 ? e / SK : e % SB, ki = sak == 1 ? e % SK : e / SB;
      const int64_t gm = m0 + mi, gk = k0 + ki;
      As[ki][mi] = (gm < M && gk < K) ? A[gm * sai + gk * sak] : 0.f;
    }
    for (int e = tid; e < SB * SK; e += 256) {
      const int nj = sbj == 1 ? e % SB : e / SK, ki = sbj == 1 ? e / SB : e % SK;
      const int64_t gn = n0 + nj, gk = k0 + ki;
      Bs[ki][nj] = (gn < N && gk < K) ? B[gk * sbk + gn * sbj] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) c[i][j] = fmaf(a[i], b[j], c[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      float* cp = C + gm * ldc + gn;
      const float v = c[i][j] + (bias ? bias[gn] : 0.f);
      *cp = acc ? *cp + v : v;
    }
  }
}

// Column sums out[j] = sum_r X[r ld + j]: partial sums of CS_CHUNKS row
// chunks (enough blocks to cover the SMs several times), then the chunks in
// order (deterministic).
constexpr int CS_CHUNKS = 256;
__global__ void __launch_bounds__(256) colsum_part_kernel(const float* __restrict__ X, int64_t rows, int64_t cols,
                                                          int64_t ld, float* __restrict__ part) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= cols) return;
  const int64_t per = (rows + CS_CHUNKS - 1) / CS_CHUNKS;
  const int64_t r0 = blockIdx.y * per, r1 = min(rows, r0 + per);
  float x = 0.f;
  for (int64_t r = r0; r < r1; ++r) x += X[r * ld + j];
  part[(int64_t)blockIdx.y * cols + j] = x;
}

// 32 columns per block; thread (column c, group g) adds chunks g, g + 8, ...
// in order, then the 8 groups are added in order (deterministic).
__global__ void __launch_bounds__(256) colsum_final_kernel(const float* __restrict__ part, int64_t cols,
                                                           float* __restrict__ out) {
  __shared__ float red[8][33];
  const int c = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int64_t j = (int64_t)blockIdx.x * 32 + c;
  float x = 0.f;
  if (j < cols)
    for (int q = g; q < CS_CHUNKS; q += 8) x += part[(int64_t)q * cols + j];
  red[g][c] = x;
  __syncthreads();
  if (g == 0 && j < cols) {
    float t = red[0][c];
#pragma unroll
    for (int i = 1; i < 8; ++i) t += red[i][c];
    out[j] = t;
  }
}

struct GemmPlan {
  bool tc;
  int S;
  int64_t Ks, Kp, m_pad, n_pad;
  size_t a_floats, b_floats, p_floats;
};

GemmPlan gemm_plan(int64_t M, int64_t N, int64_t K, int sms) {
  GemmPlan g{};
  g.tc = M >= 128 && N >= 16 && N % 16 == 0 && K >= 1 && M < (1ll << 31);
  if (!g.tc) return g;
  const int64_t cap = N > 256 ? 256 : 128;               // the tensor-core GEMM's column tile
  const int64_t bn = N >= cap ? cap : (N + 15) / 16 * 16;
  const int64_t tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  const int64_t kq = (K + KQ - 1) / KQ;                   // K stages
  int64_t S = 1;
  while (tiles * S < sms && kq / (S * 2) >= 8) S *= 2;    // slices of at least 8 stages
  g.S = (int)S;
  g.Ks = ((kq + S - 1) / S) * KQ;
  g.Kp = g.Ks * S;
  g.m_pad = S > 1 ? (M + 127) / 128 * 128 : M;          // slices start on whole tiles
  g.n_pad = S > 1 ? (N + bn - 1) / bn * bn : N;
  g.a_floats = 2 * (size_t)g.m_pad * g.Kp;
  g.b_floats = 2 * (size_t)g.n_pad * g.Kp;
  g.p_floats = (size_t)S * M * N;
  return g;
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

// K slices of the operand-splitting GEMM: the count that minimises
// (rounds of units over the SMs) x (K stages per unit), plus the slice sum's
// traffic (a stage of ~1.7 us against ~5000 bytes per ns); at least 8 stages a
// slice, the partials within `cap` floats.
void raw_slices(int64_t tiles, int64_t kq, int64_t out_elems, int sms, size_t cap, int64_t* S_out, int64_t* per_out) {
  double best = 1e30;
  int64_t bS = 1, bper = kq;
  for (int64_t S = 1; S <= 64 && S <= kq; ++S) {
    const int64_t per = (kq + S - 1) / S, s2 = (kq + per - 1) / per;   // every slice non-empty
    if (s2 > 1 && (per < 8 || (size_t)s2 * out_elems > cap)) continue;
    const int64_t rounds = (tiles * s2 + sms - 1) / sms;
    const double cost = rounds * per * 1.7e3 + (s2 > 1 ? (double)(s2 + 2) * out_elems * 4 / 5000.0 : 0.0);   // ns
    if (cost < best - 1e-9) {
      best = cost;
      bS = s2;
      bper = per;
    }
  }
  *S_out = bS;
  *per_out = bper;
}

size_t gemm_any_scratch_floats(int64_t M, int64_t N, int64_t K) {
  const GemmPlan g = gemm_plan(M, N, K, sm_count());
  if (!g.tc) return 0;
  return g.a_floats + g.b_floats + g.p_floats + 3 * 64;   // + alignment slack
}

cudaError_t launch_gemm_any(const float* A, int64_t sai, int64_t sak, const float* B, int64_t sbk, int64_t sbj,
                            float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, bool accumulate,
                            const GemmScratch& sc, int* err, cudaStream_t s, const float* bias) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (K == 0) {
    if (accumulate && !bias) return cudaSuccess;
    return cudaErrorInvalidValue;   // the backward never asks for an empty product
  }
  // The operand-splitting GEMM converts A once per column tile and B once per
  // row tile; when that repeats the operands many times over (a short K with
  // many tiles both ways) one splitting pass plus the pre-split GEMM is cheaper.
  const int64_t mt = (M + 127) / 128, nt = (N + gemm_raw_bn(N) - 1) / gemm_raw_bn(N);
  const double redundancy = ((double)M * K * nt + (double)N * K * mt) / ((double)M * K + (double)N * K);
  const GemmPlan g0 = gemm_plan(M, N, K, sm_count());
  const bool presplit = redundancy > 6.0 && g0.tc && sc.floats >= gemm_any_scratch_floats(M, N, K);
  if (!presplit && gemm_raw_supported(A, sai, sak, B, sbk, sbj, M, N, K)) {
    // operands split inside the GEMM (gemm_raw_tc.cu); K slices when few tiles
    int64_t S, per;
    raw_slices(mt * nt, (K + KQ - 1) / KQ, M * N, sm_count(), sc.floats, &S, &per);
    if (S == 1)
      return launch_gemm_raw(A, sai, sak, B, sbk, sbj, M, N, K, 1, (int)per, C, 0, ldc, bias, accumulate, err, s);
    cudaError_t e = launch_gemm_raw(A, sai, sak, B, sbk, sbj, M, N, K, (int)S, (int)per, sc.p, M * N, N, nullptr,
                                    false, err, s);
    if (e != cudaSuccess) return e;
    return launch_sum_slices(sc.p, (int)S, M, N, C, ldc, accumulate, s, bias);
  }
  const GemmPlan g = gemm_plan(M, N, K, sm_count());
  if (!g.tc || sc.floats < gemm_any_scratch_floats(M, N, K)) {
    const dim3 grid((unsigned)((N + SB - 1) / SB), (unsigned)((M + SB - 1) / SB));
    gemm_strided_simt_kernel<<<grid, 256, 0, s>>>(A, sai, sak, B, sbk, sbj, C, ldc, M, N, K, accumulate ? 1 : 0,
                                                   bias);
    count_launch();
    return cudaGetLastError();
  }
  auto align64 = [](size_t x) { return (x + 63) / 64 * 64; };   // 256-byte aligned regions
  float* a_hi = sc.p;
  float* a_lo = a_hi + align64(g.a_floats / 2);
  float* b_hi = a_lo + align64(g.a_floats / 2);
  float* b_lo = b_hi + align64(g.b_floats / 2);
  float* part = b_lo + align64(g.b_floats / 2);
  // A'(i, k) = A[i sai + k sak];  B'(j, k) = B(k, j) = B[k sbk + j sbj]
  gather_split_kernel<<<dim3((unsigned)((g.Kp + 31) / 32), (unsigned)((M + 31) / 32)), 256, 0, s>>>(
      A, M, K, sai, sak, g.Ks, g.S, g.m_pad, a_hi, a_lo, 0, 0);
  count_launch();
  gather_split_kernel<<<dim3((unsigned)((g.Kp + 31) / 32), (unsigned)((N + 31) / 32)), 256, 0, s>>>(
      B, N, K, sbj, sbk, g.Ks, g.S, g.n_pad, b_hi, b_lo, 0, 0);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // one slice over a dense C: the epilogue adds the bias and accumulates
  const bool direct = g.S == 1 && ldc == N;
  if (g.S == 1)
    e = launch_dense_tc(a_hi, a_lo, M, (int)g.Ks, b_hi, b_lo, (int)N, direct ? bias : nullptr, direct ? C : part,
                        ACT_NONE, err, s, direct && accumulate);
  else   // every slice's tiles in one launch, one partial product per slice
    e = launch_dense_tc_sliced(a_hi, a_lo, M, g.m_pad, (int)g.Ks, b_hi, b_lo, (int)N, g.n_pad, g.S, part, err, s);
  if (e != cudaSuccess) return e;
  if (direct) return cudaSuccess;
  const int64_t n = M * N;
  const int64_t blocks = (n + 255) / 256;
  sum_slices_kernel<<<(unsigned)std::min<int64_t>(blocks, 148 * 16), 256, 0, s>>>(part, g.S, M, N, C, ldc,
                                                                                  accumulate ? 1 : 0, bias);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_gather_split(const float* src, int64_t rows, int64_t cols, int64_t s_row, int64_t s_col,
                                int64_t Ks, int S, int64_t rows_pad, float* hi, float* lo, int batch, int64_t src_b,
                                int64_t dst_b, cudaStream_t s) {
  if (rows == 0 || batch == 0) return cudaSuccess;
  const int64_t kp = (int64_t)S * Ks;
  gather_split_kernel<<<dim3((unsigned)((kp + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)batch), 256, 0,
                        s>>>(src, rows, cols, s_row, s_col, Ks, S, rows_pad, hi, lo, src_b, dst_b);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_sum_slices(const float* P, int S, int64_t M, int64_t N, float* C, int64_t ldc, bool accumulate,
                              cudaStream_t s, const float* bias) {
  const int64_t n = M * N;
  if (n == 0) return cudaSuccess;
  const int64_t blocks = (n + 255) / 256;
  sum_slices_kernel<<<(unsigned)std::min<int64_t>(blocks, 148 * 16), 256, 0, s>>>(P, S, M, N, C, ldc,
                                                                                  accumulate ? 1 : 0, bias);
  count_launch();
  return cudaGetLastError();
}

size_t colsum_scratch_floats(int64_t cols) { return (size_t)CS_CHUNKS * cols; }

cudaError_t launch_colsum_det(const float* X, int64_t rows, int64_t cols, int64_t ld, float* part, float* out,
                              cudaStream_t s) {
  if (cols == 0) return cudaSuccess;
  if (rows == 0) return cudaMemsetAsync(out, 0, sizeof(float) * cols, s);
  colsum_part_kernel<<<dim3((unsigned)((cols + 255) / 256), CS_CHUNKS), 256, 0, s>>>(X, rows, cols, ld, part);
  count_launch();
  colsum_final_kernel<<<(unsigned)((cols + 31) / 32), 256, 0, s>>>(part, cols, out);
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
