// Sub-key maintenance of the training step (memory_pool_model/memory.py):
//   key_diversity_loss (:230-240)  mean squared off-diagonal cosine inside
//                                  each codebook, and its gradient;
//   revive_dead_keys (:243-281)    re-initialise rarely used sub-keys onto
//                                  observed queries (random draws passed in).
//
// Diversity: with K the codebook's n unit keys (rows) and M = K^T K
// (half x half), sum over i != j of (k_i . k_j)^2 = ||M||_F^2 - sum_i
// ||k_i||^4, and d/dk_i = 4 / D (M k_i - ||k_i||^2 k_i), D = H * 2 * n *
// (n - 1): the half x half Gram replaces the n x n one.  Three launches:
// chunked partial Grams (keys normalised in shared memory), their sum with
// the loss partials, and the gradient (K M per 32-key block, M staged in
// shared memory) with the loss.  Every reduction runs in a fixed order
// (float64 for the loss): the results are deterministic.
#include "common.cuh"
#include "keys.cuh"

namespace ml {

namespace {

constexpr int KD_R = 64;   // keys per Gram row chunk
constexpr int KD_T = 64;   // Gram output tile (rows and columns of M)
constexpr int KD_G = 32;   // keys per gradient block

// d = d_key / 2 <= 128 (the config check caps d_key at 256): a key row is
// at most 4 values per lane of a warp.
__host__ __device__ inline int kd_ld(int d) { return (d + 3) & ~3; }   // float4-aligned row stride

// Partial Gram of one codebook's row chunk: Mpart[s][hc] (tile) =
// sum over the chunk's keys (in key order) of k k^T, with the chunk's keys
// normalised in shared memory first (memory.py:31).  Blocks of tile 0 also
// write the chunk's sum of |k|^4 to sqpart[hc][s].
__global__ void __launch_bounds__(256) kd_gram_kernel(const float* __restrict__ x, int n, int d, int S,
                                                      float* __restrict__ Mpart, float* __restrict__ sqpart) {
  extern __shared__ float4 kd_smem4[];
  float* ks = reinterpret_cast<float*>(kd_smem4);          // [KD_R][ld]
  __shared__ float sq2[KD_R];
  const int ld = kd_ld(d);
  const int s = blockIdx.x, tile = blockIdx.y, hc = blockIdx.z, HC = gridDim.z;
  const int tiles_d = (d + KD_T - 1) / KD_T;
  const int ta = tile / tiles_d, tb = tile - ta * tiles_d;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = s * KD_R, rn = min(KD_R, n - r0);
  for (int i = warp; i < KD_R; i += 8) {
    float* kr = ks + i * ld;
    if (i >= rn) {
      for (int e = lane; e < ld; e += 32) kr[e] = 0.f;
      if (lane == 0) sq2[i] = 0.f;
      continue;
    }
    const float* xr = x + ((int64_t)hc * n + r0 + i) * d;
    float xv[4], ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = lane + 32 * j;
      xv[j] = e < d ? xr[e] : 0.f;
      ss = fmaf(xv[j], xv[j], ss);
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + 1e-6f);
    float s2 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = lane + 32 * j;
      const float v = xv[j] * r;
      if (e < ld) kr[e] = v;
      s2 = fmaf(v, v, s2);
    }
    s2 = warp_sum(s2);
    if (lane == 0) sq2[i] = s2 * s2;
  }
  __syncthreads();
  if (tile == 0 && threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < rn; ++i) t += sq2[i];
    sqpart[(int64_t)hc * S + s] = t;
  }
  // 16 x 16 threads, 4 x 4 outputs each
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int a0 = ta * KD_T + ty * 4, b0 = tb * KD_T + tx * 4;
  if (a0 >= ld || b0 >= ld) return;
  float acc[4][4] = {};
  for (int i = 0; i < rn; ++i) {
    const float4 va = *reinterpret_cast<const float4*>(ks + i * ld + a0);
    const float4 vb = *reinterpret_cast<const float4*>(ks + i * ld + b0);
    const float av[4] = {va.x, va.y, va.z, va.w}, bv[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[p][q] = fmaf(av[p], bv[q], acc[p][q]);
  }
  float* out = Mpart + ((int64_t)s * HC + hc) * d * d;
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (a0 + p < d && b0 + q < d) out[(int64_t)(a0 + p) * d + b0 + q] = acc[p][q];
}

// M = sum over the S chunk partials (chunk order); lpart[block] = the
// block's sum of M^2 in float64 (fixed thread -> element map, fixed tree).
__global__ void __launch_bounds__(256) kd_reduce_kernel(const float* __restrict__ Mpart, int S, int64_t count,
                                                        float* __restrict__ M, double* __restrict__ lpart) {
  __shared__ double red[8];
  double acc = 0.0;
  for (int64_t e = (int64_t)blockIdx.x * 256 + threadIdx.x; e < count; e += (int64_t)gridDim.x * 256) {
    float v = 0.f;
    for (int s = 0; s < S; ++s) v += Mpart[(int64_t)s * count + e];
    M[e] = v;
    acc += (double)v * (double)v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += red[w];
    lpart[blockIdx.x] = t;
  }
}

// Gradient of KD_G keys of one codebook: with Y = K M (M staged in shared
// memory), dk_i = coef (Y_i - |k_i|^2 k_i) and grad x_i = r_i dk_i - r_i^3
// (x_i . dk_i) x_i.  Block (0, 0) also writes the loss
// (sum lpart - sum sqpart) / denom.  grad == nullptr: loss only.
__global__ void __launch_bounds__(256) kd_grad_kernel(const float* __restrict__ x, const float* __restrict__ M,
                                                      const double* __restrict__ lpart, int nlp,
                                                      const float* __restrict__ sqpart, int nsq, double denom,
                                                      int n, int d, float coef, float* __restrict__ loss,
                                                      float* __restrict__ grad) {
  extern __shared__ float4 kd_smem4[];
  const int ld = kd_ld(d);
  float* Ms = reinterpret_cast<float*>(kd_smem4);          // [d][ld]
  float* ks = Ms + d * ld;                                  // [KD_G][ld]
  float* xs = ks + KD_G * ld;                               // [KD_G][ld]
  __shared__ float rr[KD_G], sqs[KD_G];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (loss && blockIdx.x == 0 && blockIdx.y == 0 && warp == 0) {
    double t = 0.0;
    for (int i = lane; i < nlp; i += 32) t += lpart[i];
    for (int i = lane; i < nsq; i += 32) t -= (double)sqpart[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(FULL, t, o);
    // n = 1: the reference's off-diagonal is exactly zero and its loss 0 / 0
    if (lane == 0) *loss = denom > 0.0 ? (float)(t / denom) : __int_as_float(0x7fc00000);
  }
  if (!grad) return;
  const int hc = blockIdx.y, r0 = blockIdx.x * KD_G, rn = min(KD_G, n - r0);
  const float* Mc = M + (int64_t)hc * d * d;
  if (ld == d) {
    const float4* src = reinterpret_cast<const float4*>(Mc);   // 16-byte aligned: d % 4 == 0, 256-byte base
    float4* dst = reinterpret_cast<float4*>(Ms);
    for (int e = threadIdx.x; e < d * d / 4; e += 256) dst[e] = src[e];
  } else {
    for (int a = warp; a < d; a += 8)
      for (int b = lane; b < ld; b += 32) Ms[a * ld + b] = b < d ? Mc[(int64_t)a * d + b] : 0.f;
  }
  for (int i = warp; i < KD_G; i += 8) {
    float* kr = ks + i * ld;
    float* xr_s = xs + i * ld;
    if (i >= rn) {
      for (int e = lane; e < ld; e += 32) kr[e] = xr_s[e] = 0.f;
      if (lane == 0) rr[i] = sqs[i] = 0.f;
      continue;
    }
    const float* xr = x + ((int64_t)hc * n + r0 + i) * d;
    float xv[4], ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = lane + 32 * j;
      xv[j] = e < d ? xr[e] : 0.f;
      ss = fmaf(xv[j], xv[j], ss);
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + 1e-6f);
    float s2 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = lane + 32 * j;
      const float v = xv[j] * r;
      if (e < ld) {
        xr_s[e] = xv[j];
        kr[e] = v;
      }
      s2 = fmaf(v, v, s2);
    }
    s2 = warp_sum(s2);
    if (lane == 0) {
      rr[i] = r;
      sqs[i] = s2;
    }
  }
  __syncthreads();
  // warp w: keys 4w..4w+3; lane: columns 4 lane..4 lane+3 (d <= 128)
  const int i0 = warp * 4, c0 = lane * 4;
  const bool active = c0 < ld;
  float acc[4][4] = {};
  if (active) {
    for (int b = 0; b < d; ++b) {
      const float4 m = *reinterpret_cast<const float4*>(Ms + b * ld + c0);   // M symmetric: row b = column b
      const float mv[4] = {m.x, m.y, m.z, m.w};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float kv = ks[(i0 + p) * ld + b];
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[p][q] = fmaf(kv, mv[q], acc[p][q]);
      }
    }
  }
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int i = i0 + p;
    float dk[4], dot = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = c0 + q;
      dk[q] = (active && c < d) ? coef * (acc[p][q] - sqs[i] * ks[i * ld + c]) : 0.f;
      if (active && c < d) dot = fmaf(xs[i * ld + c], dk[q], dot);
    }
    dot = warp_sum(dot);
    if (i < rn && active) {
      const float r = rr[i];
      float* g = grad + ((int64_t)hc * n + r0 + i) * d;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (c0 + q < d) g[c0 + q] = r * dk[q] - r * r * r * dot * xs[i * ld + c0 + q];
    }
  }
}

// ---- revive_dead_keys ----
// Keys: one warp per key (dead = usage < threshold / n); a dead key becomes
// the unit vector of queries[pick] + noise_scale * noise and its optimiser
// moments are zeroed.
__global__ void __launch_bounds__(256) revive_keys_kernel(float* __restrict__ keys, const float* __restrict__ usage,
                                                          const float* __restrict__ queries, int64_t tokens,
                                                          const int* __restrict__ pick,
                                                          const float* __restrict__ noise, int64_t nkeys, int HC,
                                                          int n, int d, float thr, float noise_scale,
                                                          int* __restrict__ dead_out, float* __restrict__ m0,
                                                          float* __restrict__ m1) {
  const int lane = threadIdx.x & 31;
  const int64_t key = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (key >= nkeys) return;
  const bool dead = usage[key] < thr;
  if (dead_out && lane == 0) dead_out[key] = dead;
  if (!dead) return;
  const int hc = (int)(key / n);
  // an index outside [0, tokens) is normalised and clamped as an XLA
  // gather does (negative counts from the end)
  int64_t p = pick[key];
  if (p < 0) p += tokens;
  p = p < 0 ? 0 : (p >= tokens ? tokens - 1 : p);
  const float* q = queries + ((int64_t)p * HC + hc) * d;
  const float* z = noise + key * d;
  float ss = 0.f;
  for (int e = lane; e < d; e += 32) {
    const float v = q[e] + noise_scale * z[e];
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss + 1e-6f);
  const int64_t o = key * d;
  for (int e = lane; e < d; e += 32) {
    keys[o + e] = (q[e] + noise_scale * z[e]) * r;
    if (m0) m0[o + e] = 0.f;
    if (m1) m1[o + e] = 0.f;
  }
}

// Usage: one block per codebook; dead entries become 1 / n and the row is
// divided by its sum (fixed-order tree).  Runs after revive_keys_kernel,
// which reads the old usage.
__global__ void __launch_bounds__(256) revive_usage_kernel(float* __restrict__ usage, int n, float thr) {
  __shared__ float red[256];
  float* u = usage + (int64_t)blockIdx.x * n;
  float part = 0.f;
  for (int i = threadIdx.x; i < n; i += 256) part += u[i] < thr ? 1.0f / (float)n : u[i];
  red[threadIdx.x] = part;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  const float total = red[0];
  for (int i = threadIdx.x; i < n; i += 256) u[i] = (u[i] < thr ? 1.0f / (float)n : u[i]) / total;
}

constexpr int KD_REDUCE_BLOCKS = 296;   // 2 x 148 SMs

int kd_chunks(int n) { return (n + KD_R - 1) / KD_R; }

}  // namespace

KeyDivLayout key_div_layout(int HC, int n, int d) {
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  KeyDivLayout L{};
  const int64_t dd = (int64_t)HC * d * d;
  const int S = kd_chunks(n);
  L.o_Mpart = 0;
  L.o_M = L.o_Mpart + up(4 * dd * S);
  L.o_lpart = L.o_M + up(4 * dd);
  L.o_sqpart = L.o_lpart + up(8 * KD_REDUCE_BLOCKS);
  L.bytes = L.o_sqpart + up(4 * (int64_t)HC * S);
  return L;
}

cudaError_t launch_key_diversity(const float* sub_keys, int HC, int n, int d, char* ws, float* loss, float* grad,
                                 float scale, cudaStream_t s) {
  const KeyDivLayout L = key_div_layout(HC, n, d);
  float* Mpart = reinterpret_cast<float*>(ws + L.o_Mpart);
  float* M = reinterpret_cast<float*>(ws + L.o_M);
  double* lpart = reinterpret_cast<double*>(ws + L.o_lpart);
  float* sqpart = reinterpret_cast<float*>(ws + L.o_sqpart);
  const int S = kd_chunks(n), ld = kd_ld(d), td = (d + KD_T - 1) / KD_T;
  const size_t gram_smem = (size_t)KD_R * ld * 4;
  const size_t grad_smem = (size_t)(d + 2 * KD_G) * ld * 4;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(kd_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)grad_smem)) !=
      cudaSuccess)
    return e;
  kd_gram_kernel<<<dim3(S, td * td, HC), 256, gram_smem, s>>>(sub_keys, n, d, S, Mpart, sqpart);
  const int64_t count = (int64_t)HC * d * d;
  int nb = (int)((count + 255) / 256);
  nb = nb < KD_REDUCE_BLOCKS ? nb : KD_REDUCE_BLOCKS;
  kd_reduce_kernel<<<nb, 256, 0, s>>>(Mpart, S, count, M, lpart);
  const double denom = (double)HC * n * (double)(n - 1);
  const float coef = denom > 0.0 ? (float)(4.0 * scale / denom) : NAN;   // n = 1: NaN, as the loss
  const dim3 grid = grad ? dim3((n + KD_G - 1) / KD_G, HC) : dim3(1, 1);
  kd_grad_kernel<<<grid, 256, grad ? grad_smem : 0, s>>>(sub_keys, M, lpart, nb, sqpart, HC * S, denom, n, d, coef,
                                                         loss, grad);
  count_launch(3);
  return cudaGetLastError();
}

cudaError_t launch_revive(float* keys, float* usage, const float* queries, int64_t tokens, const int* pick,
                          const float* noise, int HC, int n, int d, float threshold, float noise_scale, int* dead,
                          float* m0, float* m1, cudaStream_t s) {
  const float thr = threshold / (float)n;
  const int64_t nkeys = (int64_t)HC * n;
  revive_keys_kernel<<<(unsigned)((nkeys + 7) / 8), 256, 0, s>>>(keys, usage, queries, tokens, pick, noise, nkeys,
                                                                  HC, n, d, thr, noise_scale, dead, m0, m1);
  revive_usage_kernel<<<HC, 256, 0, s>>>(usage, n, thr);
  count_launch(2);
  return cudaGetLastError();
}

}  // namespace ml
