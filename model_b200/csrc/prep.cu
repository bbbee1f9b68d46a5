// Normalisation, temperature, float32 GEMM (router / gate / output
// projections) and the final aux reductions of the memory layer.
#include "backbone.cuh"
#include "tc_common.cuh"

namespace ml {

// One warp per sub-key row: keys_n = x * rsqrt(sum(x*x) + 1e-6)
// (memory.py:30-31,139).  Block 0 also writes the clamped temperature.
__global__ void prep_keys_kernel(const float* __restrict__ keys, float* __restrict__ keys_n,
                                 float* __restrict__ k_hi, float* __restrict__ k_lo, int64_t rows, int half,
                                 const float* __restrict__ log_t, float min_t, float max_t,
                                 float* __restrict__ scal, int* __restrict__ err, int* __restrict__ fin_ctr) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    scal[0] = clamped_temperature(log_t[0], min_t, max_t);
    *err = 0;      // device error code of this call's bounded waits
    *fin_ctr = 0;  // block ticket of the aux reduction
  }
  int lane = threadIdx.x & 31;
  int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* x = keys + row * half;
  float ss = 0.f;
  for (int i = lane; i < half; i += 32) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  float r = 1.0f / sqrtf(ss + 1e-6f);
  float* y = keys_n + row * half;
  for (int i = lane; i < half; i += 32) {
    const float v = x[i] * r;
    y[i] = v;
    if (k_hi) {
      const float hi = tc::to_tf32(v);
      k_hi[row * half + i] = hi;
      k_lo[row * half + i] = tc::to_tf32(v - hi);
    }
  }
}

// One warp per (token, head, half): q_len (memory.py:137) and unit q (:138).
__global__ void normalize_q_kernel(const float* __restrict__ q, float* __restrict__ qn, float* __restrict__ qlen,
                                   float* __restrict__ q_hi, float* __restrict__ q_lo, int64_t rows, int half,
                                   int hc_count, int64_t M) {
  int lane = threadIdx.x & 31;
  int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* x = q + row * half;
  float ss = 0.f;
  for (int i = lane; i < half; i += 32) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  float t = ss + 1e-6f;
  if (lane == 0) qlen[row] = sqrtf(t) / sqrtf((float)half);
  float r = 1.0f / sqrtf(t);
  float* y = qn + row * half;
  // codebook-major copy for the tensor-core path: [hc][m][half]
  const int64_t tr = (row % hc_count) * M + row / hc_count;
  for (int i = lane; i < half; i += 32) {
    const float v = x[i] * r;
    y[i] = v;
    if (q_hi) {
      const float hi = tc::to_tf32(v);
      q_hi[tr * half + i] = hi;
      q_lo[tr * half + i] = tc::to_tf32(v - hi);
    }
  }
}

cudaError_t launch_prep_keys(const Dims& D, const float* sub_keys, const float* log_t, float min_t, float max_t,
                             float* keys_n, float* k_hi, float* k_lo, float* scal, int* err, int* fin_ctr,
                             cudaStream_t s) {
  int64_t rows = (int64_t)D.H * 2 * D.n;
  int wpb = 8;
  prep_keys_kernel<<<(unsigned)((rows + wpb - 1) / wpb), wpb * 32, 0, s>>>(sub_keys, keys_n, k_hi, k_lo, rows,
                                                                            D.half, log_t, min_t, max_t, scal, err, fin_ctr);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_normalize_queries(const Dims& D, const float* q, float* qn, float* qlen, float* q_hi,
                                     float* q_lo, cudaStream_t s) {
  int64_t rows = D.M * D.H * 2;
  if (rows == 0) return cudaSuccess;
  int wpb = 8;
  normalize_q_kernel<<<(unsigned)((rows + wpb - 1) / wpb), wpb * 32, 0, s>>>(q, qn, qlen, q_hi, q_lo, rows, D.half,
                                                                              D.H * 2, D.M);
  count_launch();
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// float32 SIMT GEMM: C[M,N] = act(A[M,K] @ B[K,N] + bias), all row-major.
// 64x64 tile, 16-deep k-slices, 256 threads, 4x4 outputs per thread.
// ---------------------------------------------------------------------------
constexpr int GB_M = 64, GB_N = 64, GB_K = 16;

// act: 0 none, 1 SiLU (model.py:118), 2 GELU with the tanh approximation
// (flax's nn.gelu, model.py:104): 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == 1) return v / (1.0f + expf(-v));
  if (act == 2) return v * (0.5f * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * (v * v * v)))));
  return v;
}

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                       const float* __restrict__ bias, float* __restrict__ C,
                                                       int64_t M, int N, int K, int act) {
  __shared__ float As[GB_K][GB_M + 4];
  __shared__ float Bs[GB_K][GB_N + 4];
  int tid = threadIdx.x;
  int ty = tid / 16, tx = tid % 16;
  int64_t m0 = (int64_t)blockIdx.y * GB_M;
  int n0 = blockIdx.x * GB_N;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += GB_K) {
    // A tile: 64 rows x 16 k (1024 elements, 4 per thread)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      int e = tid + r * 256;
      int mi = e / GB_K, ki = e % GB_K;
      int64_t gm = m0 + mi;
      int gk = k0 + ki;
      As[ki][mi] = (gm < M && gk < K) ? A[gm * K + gk] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      int e = tid + r * 256;
      int ki = e / GB_N, ni = e % GB_N;
      int gk = k0 + ki, gn = n0 + ni;
      Bs[ki][ni] = (gk < K && gn < N) ? B[(int64_t)gk * N + gn] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < GB_K; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      C[gm * N + gn] = apply_act(acc[i][j] + (bias ? bias[gn] : 0.f), act);
    }
  }
}

// Few rows (decode): C[m, n] = act(sum_k A[m, k] B[k, n] + bias).  Lane =
// output column (coalesced rows of B), the 8 warps of a CTA split K into
// contiguous ranges and their partial sums are added in warp order through
// shared memory (deterministic); up to GV_M rows per CTA.
constexpr int GV_M = 8;

struct GemvOut {
  const float* B;      // [K, N]
  const float* bias;   // [N] or nullptr
  float* C;            // [M, N]
  int N, act;
};

// Up to two products of the same A in one launch: column blocks
// [0, nb0) compute out0, the rest out1 (the router and gate Dense layers of
// a decode step share the hidden state).
__global__ void __launch_bounds__(256) gemv_f32_kernel(const float* __restrict__ A, GemvOut out0, GemvOut out1,
                                                       int nb0, int64_t M, int K) {
  __shared__ float part[8][GV_M][32];
  const bool second = (int)blockIdx.x >= nb0;
  const float* __restrict__ B = second ? out1.B : out0.B;
  const float* __restrict__ bias = second ? out1.bias : out0.bias;
  float* __restrict__ C = second ? out1.C : out0.C;
  const int N = second ? out1.N : out0.N, act = second ? out1.act : out0.act;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int n = ((int)blockIdx.x - (second ? nb0 : 0)) * 32 + lane;
  const int64_t m0 = (int64_t)blockIdx.y * GV_M;
  const int kper = (K + 7) / 8, k0 = w * kper, k1 = min(K, k0 + kper);
  float acc[GV_M];
#pragma unroll
  for (int i = 0; i < GV_M; ++i) acc[i] = 0.f;
  if (n < N) {
#pragma unroll 4
    for (int k = k0; k < k1; ++k) {
      const float b = __ldg(B + (int64_t)k * N + n);
#pragma unroll
      for (int i = 0; i < GV_M; ++i)
        if (m0 + i < M) acc[i] = fmaf(__ldg(A + (m0 + i) * K + k), b, acc[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < GV_M; ++i) part[w][i][lane] = acc[i];
  __syncthreads();
  if (w == 0 && n < N) {
#pragma unroll
    for (int i = 0; i < GV_M; ++i) {
      if (m0 + i >= M) break;
      float x = 0.f;
#pragma unroll
      for (int ww = 0; ww < 8; ++ww) x += part[ww][i][lane];
      if (bias) x += bias[n];
      C[(m0 + i) * N + n] = apply_act(x, act);
    }
  }
}

cudaError_t launch_gemm(const float* A, const float* B, const float* bias, float* C, int64_t M, int N, int K,
                        bool silu, cudaStream_t s) {
  return launch_gemm_act(A, B, bias, C, M, N, K, silu ? 1 : 0, s);
}

cudaError_t launch_gemm_act(const float* A, const float* B, const float* bias, float* C, int64_t M, int N, int K,
                            int act, cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  if (M <= 4 * GV_M) {
    const GemvOut o{B, bias, C, N, act};
    const int nb = (N + 31) / 32;
    gemv_f32_kernel<<<dim3(nb, (unsigned)((M + GV_M - 1) / GV_M)), 256, 0, s>>>(A, o, o, nb, M, K);
    count_launch();
    return cudaGetLastError();
  }
  dim3 grid((N + GB_N - 1) / GB_N, (unsigned)((M + GB_M - 1) / GB_M));
  gemm_f32_kernel<<<grid, 256, 0, s>>>(A, B, bias, C, M, N, K, act);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_gemm2(const float* A, const float* B0, const float* bias0, float* C0, int N0, bool silu0,
                         const float* B1, const float* bias1, float* C1, int N1, bool silu1, int64_t M, int K,
                         cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  if (M > 4 * GV_M) {
    cudaError_t e = launch_gemm(A, B0, bias0, C0, M, N0, K, silu0, s);
    return e != cudaSuccess ? e : launch_gemm(A, B1, bias1, C1, M, N1, K, silu1, s);
  }
  const GemvOut o0{B0, bias0, C0, N0, silu0 ? 1 : 0}, o1{B1, bias1, C1, N1, silu1 ? 1 : 0};
  const int nb0 = (N0 + 31) / 32, nb1 = (N1 + 31) / 32;
  gemv_f32_kernel<<<dim3(nb0 + nb1, (unsigned)((M + GV_M - 1) / GV_M)), 256, 0, s>>>(A, o0, o1, nb0, M, K);
  count_launch();
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// aux finalisation: top1_weight = mean over (token, head) of the max weight
// (memory.py:225) and the temperature.  FIN_BLOCKS blocks sum fixed
// contiguous ranges in double; the last block to finish (ticket counter)
// adds the partials in block order, so the result is deterministic.
// ---------------------------------------------------------------------------
constexpr int FIN_BLOCKS = 64;

__global__ void __launch_bounds__(256) finalize_kernel(const float* __restrict__ top1_part, int64_t count,
                                                       float* __restrict__ top1, const float* __restrict__ scal,
                                                       float* __restrict__ temperature, double* __restrict__ part,
                                                       int* __restrict__ ctr) {
  __shared__ double red[8];
  __shared__ bool last;
  const int64_t chunk = (count + FIN_BLOCKS - 1) / FIN_BLOCKS;
  const int64_t lo = blockIdx.x * chunk, hi = lo + chunk < count ? lo + chunk : count;
  double acc = 0.0;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) acc += (double)top1_part[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += red[w];
    part[blockIdx.x] = t;
    __threadfence();
    last = atomicAdd(ctr, 1) == FIN_BLOCKS - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    double t = 0.0;
    for (int b = 0; b < FIN_BLOCKS; ++b) t += ((volatile double*)part)[b];
    if (top1) top1[0] = count > 0 ? (float)(t / (double)count) : __int_as_float(0x7fc00000);
    if (temperature) temperature[0] = scal[0];
    *ctr = 0;
  }
}

cudaError_t launch_finalize(const Dims& D, const Work& W, float* top1, float* temperature, cudaStream_t s) {
  if (!top1 && !temperature) return cudaSuccess;
  finalize_kernel<<<FIN_BLOCKS, 256, 0, s>>>(W.top1_part, D.M * D.H, top1, W.scal, temperature, W.fin_part,
                                             W.fin_ctr);
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
