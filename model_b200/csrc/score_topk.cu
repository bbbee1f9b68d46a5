// Stage 1 of the product-key search (memory.py:149-164): cosine scores of
// every unit query half against every unit sub-key of its codebook, the
// temperature / query-length scaling, optional Gumbel selection noise, and a
// per-(token, head, half) running top-k kept in registers, so the
// [M, H, 2, n] score tensor never reaches global memory.
//
// SIMT float32 path: a CTA owns SCORE_TM tokens of one (head, half)
// codebook and streams the codebook through shared memory in SCORE_TN-key
// chunks; each chunk's score tile is staged in shared memory and scanned by
// one thread per token.
#include <float.h>

#include "common.cuh"

namespace ml {

namespace {

constexpr int TM = SCORE_TM, TN = SCORE_TN, NT = 256;

// Cosine tile [TM x TN] for the current key chunk into ss (row stride TN+1).
__device__ __forceinline__ void cos_tile(const float* qs, const float* ks, float* ss, int half) {
  int tid = threadIdx.x;
  int ty = tid / 16, tx = tid % 16;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int d = 0; d < half; ++d) {
    float4 a0 = *reinterpret_cast<const float4*>(&qs[d * TM + ty * 8]);
    float4 a1 = *reinterpret_cast<const float4*>(&qs[d * TM + ty * 8 + 4]);
    float4 b = *reinterpret_cast<const float4*>(&ks[d * TN + tx * 4]);
    float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) ss[(ty * 8 + i) * (TN + 1) + tx * 4 + j] = acc[i][j];
}

__device__ __forceinline__ void load_q_tile(const Dims& D, const float* qn, float* qs, int64_t m0, int h, int c) {
  const int half = D.half;
  for (int e = threadIdx.x; e < TM * half; e += NT) {
    int mi = e / half, di = e % half;
    int64_t m = m0 + mi;
    qs[di * TM + mi] = (m < D.M) ? qn[((m * D.H + h) * 2 + c) * half + di] : 0.f;
  }
}

__device__ __forceinline__ void load_k_chunk(const Dims& D, const float* keys_n, float* ks, int hc, int k0) {
  const int half = D.half;
  for (int e = threadIdx.x; e < TN * half; e += NT) {
    int kj = e / half, di = e % half;
    int key = k0 + kj;
    ks[di * TN + kj] = key < D.n ? keys_n[((int64_t)hc * D.n + key) * half + di] : 0.f;
  }
}

template <int KM, bool NOISY, bool BAL>
__global__ void __launch_bounds__(NT) score_topk_kernel(Dims D, const float* __restrict__ qn,
                                                        const float* __restrict__ qlen,
                                                        const float* __restrict__ keys_n,
                                                        const float* __restrict__ gumbel,
                                                        const float* __restrict__ scal, int* __restrict__ sub_idx,
                                                        float* __restrict__ sub_score, float* __restrict__ sub_sel,
                                                        int* __restrict__ clean_idx, float* __restrict__ row_max,
                                                        float* __restrict__ row_sum) {
  extern __shared__ float smem[];
  const int half = D.half;
  float* qs = smem;
  float* ks = qs + half * TM;
  float* ss = ks + half * TN;
  const int hc = blockIdx.y, h = hc >> 1, c = hc & 1;
  const int64_t m0 = (int64_t)blockIdx.x * TM;
  const int tid = threadIdx.x;
  load_q_tile(D, qn, qs, m0, h, c);

  const float T = scal[0];
  const int64_t m = m0 + tid;
  const bool owner = tid < TM && m < D.M;
  const int64_t row = (m * D.H + h) * 2 + c;
  const float ql = (owner && D.qscale) ? qlen[row] : 1.f;
  const float* grow = (NOISY && owner) ? gumbel + row * D.n : nullptr;

  float v[KM], sc[KM], cv[NOISY && BAL ? KM : 1];
  int ix[KM], cix[NOISY && BAL ? KM : 1];
#pragma unroll
  for (int j = 0; j < KM; ++j) {
    v[j] = -INFINITY;
    sc[j] = -INFINITY;
    ix[j] = 0;
  }
  if constexpr (NOISY && BAL) {
#pragma unroll
    for (int j = 0; j < KM; ++j) {
      cv[j] = -INFINITY;
      cix[j] = 0;
    }
  }
  float rmax = -INFINITY, rsum = 0.f;

  for (int k0 = 0; k0 < D.n; k0 += TN) {
    load_k_chunk(D, keys_n, ks, hc, k0);
    __syncthreads();
    cos_tile(qs, ks, ss, half);
    __syncthreads();
    if (owner) {
      const int lim = min(TN, D.n - k0);
      for (int j = 0; j < lim; ++j) {
        const float cosv = ss[tid * (TN + 1) + j];
        float score = __fmul_rn(cosv, T);                       // memory.py:150
        if (D.qscale) score = __fmul_rn(score, ql);             // memory.py:151-152
        float sel = score;
        if constexpr (NOISY) sel = __fadd_rn(score, __fmul_rn(D.noise_coef, grow[k0 + j]));  // :158
        if (sel > v[KM - 1]) list_insert3<KM>(v, ix, sc, sel, k0 + j, score);
        if constexpr (NOISY && BAL) {
          if (score > cv[KM - 1]) list_insert<KM>(cv, cix, score, k0 + j);
        }
        if constexpr (BAL) {
          const float p = D.btgrad ? score : __fmul_rn(cosv, T);   // memory.py:211
          if (p > rmax) {
            rsum = rsum * expf(rmax - p) + 1.f;
            rmax = p;
          } else {
            rsum += expf(p - rmax);
          }
        }
      }
    }
    __syncthreads();
  }
  if (!owner) return;
  const int64_t o = row * D.k;
#pragma unroll
  for (int j = 0; j < KM; ++j) {
    if (j < D.k) {
      sub_idx[o + j] = ix[j];
      sub_sel[o + j] = v[j];
      sub_score[o + j] = sc[j];
      if constexpr (NOISY && BAL) clean_idx[o + j] = cix[j];
    }
  }
  if constexpr (BAL) {
    row_max[row] = rmax;
    row_sum[row] = rsum;
  }
}

// Balance-loss column sums (memory.py:211-212): for each sub-key i,
// sum over the tile's tokens of softmax(p)[m, i], written per tile.
__global__ void __launch_bounds__(NT) balance_cols_kernel(Dims D, const float* __restrict__ qn,
                                                          const float* __restrict__ qlen,
                                                          const float* __restrict__ keys_n,
                                                          const float* __restrict__ scal,
                                                          const float* __restrict__ row_max,
                                                          const float* __restrict__ row_sum,
                                                          float* __restrict__ p_part) {
  extern __shared__ float smem[];
  const int half = D.half;
  float* qs = smem;
  float* ks = qs + half * TM;
  float* ss = ks + half * TN;
  __shared__ float rm[TM], rs[TM], rq[TM];
  const int hc = blockIdx.y, h = hc >> 1, c = hc & 1;
  const int64_t m0 = (int64_t)blockIdx.x * TM;
  const int tid = threadIdx.x;
  load_q_tile(D, qn, qs, m0, h, c);
  const float T = scal[0];
  if (tid < TM) {
    int64_t m = m0 + tid;
    bool ok = m < D.M;
    int64_t row = (m * D.H + h) * 2 + c;
    rm[tid] = ok ? row_max[row] : 0.f;
    rs[tid] = ok ? row_sum[row] : 1.f;
    rq[tid] = (ok && D.qscale) ? qlen[row] : 1.f;
  }
  const int valid = (int)(D.M - m0 < TM ? D.M - m0 : TM);
  float* dst = p_part + ((int64_t)blockIdx.x * D.H * 2 + hc) * D.n;
  for (int k0 = 0; k0 < D.n; k0 += TN) {
    load_k_chunk(D, keys_n, ks, hc, k0);
    __syncthreads();
    cos_tile(qs, ks, ss, half);
    __syncthreads();
    if (tid < TN && k0 + tid < D.n) {
      float acc = 0.f;
      for (int mi = 0; mi < valid; ++mi) {
        const float cosv = ss[mi * (TN + 1) + tid];
        float p = __fmul_rn(cosv, T);
        if (D.btgrad && D.qscale) p = __fmul_rn(p, rq[mi]);
        acc += expf(p - rm[mi]) / rs[mi];
      }
      dst[k0 + tid] = acc;
    }
    __syncthreads();
  }
}

// Clean top-k counts per sub-key, through a shared-memory histogram per
// block (skewed routing makes global atomics on a few sub-keys serialise);
// integer-valued float adds are exact, so the order does not matter.
__global__ void count_clean_smem_kernel(Dims D, const int* __restrict__ idx, float* __restrict__ cnt) {
  extern __shared__ float hist[];
  const int bins = D.H * 2 * D.n;
  for (int i = threadIdx.x; i < bins; i += blockDim.x) hist[i] = 0.f;
  __syncthreads();
  const int64_t total = D.M * D.H * 2 * D.k;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / D.k;
    const int hc = (int)(row % (D.H * 2));
    atomicAdd(&hist[hc * D.n + idx[e]], 1.f);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < bins; i += blockDim.x)
    if (hist[i] != 0.f) atomicAdd(&cnt[i], hist[i]);
}

// Clean top-k counts per sub-key (the f of memory.py:208-209).
__global__ void count_clean_kernel(Dims D, const int* __restrict__ idx, float* __restrict__ cnt) {
  int64_t total = D.M * D.H * 2 * D.k;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t row = e / D.k;
    int hc = (int)(row % (D.H * 2));
    atomicAdd(&cnt[(int64_t)hc * D.n + idx[e]], 1.f);
  }
}

// balance_loss = n * mean_{h,c} sum_i f[h,c,i] * P[h,c,i]   (memory.py:214)
// balance_loss = n * mean_{h,c} sum_i f[h,c,i] * P[h,c,i]   (memory.py:214).
// One block per 32 sub-keys: the 8 warps add disjoint sets of the `planes`
// partial column sums (lane = sub-key), the sets are added in warp order,
// then f * P is summed per block; the last block (ticket) adds the block sums
// in block order.  Every sum has a fixed order: the result is deterministic.
__global__ void __launch_bounds__(256) balance_finalize_kernel(Dims D, const float* __restrict__ p_part, int planes,
                                                               const float* __restrict__ cnt,
                                                               double* __restrict__ part, int* __restrict__ ticket,
                                                               float* __restrict__ out) {
  __shared__ double red[8][32];
  __shared__ bool last;
  const int64_t total = (int64_t)D.H * 2 * D.n;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t e = (int64_t)blockIdx.x * 32 + lane;
  double P = 0.0;
  if (e < total)
    for (int t = w; t < planes; t += 8) P += (double)p_part[(int64_t)t * total + e];
  red[w][lane] = P;
  __syncthreads();
  if (w == 0) {
    double Pe = 0.0;
    for (int ww = 0; ww < 8; ++ww) Pe += red[ww][lane];
    const double inv_mk = 1.0 / ((double)D.M * D.k);
    double c = e < total ? ((double)cnt[e] * inv_mk) * (Pe / (double)D.M) : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(FULL, c, o);
    if (lane == 0) {
      part[blockIdx.x] = c;
      __threadfence();
      last = atomicAdd(ticket, 1) == (int)gridDim.x - 1;
    }
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    double t = 0.0;
    for (unsigned b = 0; b < gridDim.x; ++b) t += ((volatile double*)part)[b];
    out[0] = D.M > 0 ? (float)((double)D.n * t / (double)(D.H * 2)) : __int_as_float(0x7fc00000);
    *ticket = 0;
  }
}

template <int KM, bool NOISY, bool BAL>
cudaError_t launch_score_t(const Dims& D, const Work& W, const float* gumbel, cudaStream_t s) {
  size_t smem = (size_t)(D.half * TM + D.half * TN + TM * (TN + 1)) * sizeof(float);
  auto kern = score_topk_kernel<KM, NOISY, BAL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((D.M + TM - 1) / TM), D.H * 2);
  kern<<<grid, NT, smem, s>>>(D, W.qn, W.qlen, W.keys_n, gumbel, W.scal, W.sub_idx, W.sub_score, W.sub_sel,
                              W.clean_idx, W.row_max, W.row_sum);
  count_launch();
  return cudaGetLastError();
}

template <int KM>
cudaError_t launch_score_k(const Dims& D, const Work& W, const float* gumbel, bool bal, cudaStream_t s) {
  if (D.noisy) return bal ? launch_score_t<KM, true, true>(D, W, gumbel, s) : launch_score_t<KM, true, false>(D, W, gumbel, s);
  return bal ? launch_score_t<KM, false, true>(D, W, gumbel, s) : launch_score_t<KM, false, false>(D, W, gumbel, s);
}

}  // namespace

cudaError_t launch_score_topk(const Dims& D, const Work& W, const float* gumbel, bool want_balance,
                              cudaStream_t s) {
  if (D.M == 0) return cudaSuccess;
  switch (D.kmax) {
    case 4: return launch_score_k<4>(D, W, gumbel, want_balance, s);
    case 8: return launch_score_k<8>(D, W, gumbel, want_balance, s);
    case 16: return launch_score_k<16>(D, W, gumbel, want_balance, s);
    case 32: return launch_score_k<32>(D, W, gumbel, want_balance, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_balance(const Dims& D, const Work& W, float* balance_loss, cudaStream_t s) {
  int planes = (int)((D.M + TM - 1) / TM);
  cudaError_t e = cudaMemsetAsync(W.clean_cnt, 0, sizeof(float) * D.H * 2 * D.n, s);
  if (e != cudaSuccess) return e;
  if (D.M > 0) {
    if (W.q_hi) {
      // tensor-core pass over the same query / key halves as the score kernel
      if ((e = launch_balance_tc(D, W, &planes, s)) != cudaSuccess) return e;
    } else {
      size_t smem = (size_t)(D.half * TM + D.half * TN + TM * (TN + 1)) * sizeof(float);
      e = cudaFuncSetAttribute(balance_cols_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      balance_cols_kernel<<<dim3(planes, D.H * 2), NT, smem, s>>>(D, W.qn, W.qlen, W.keys_n, W.scal, W.row_max,
                                                                  W.row_sum, W.p_part);
      count_launch();
    }
    const int* idx = D.noisy ? W.clean_idx : W.sub_idx;
    int64_t total = D.M * D.H * 2 * D.k;
    unsigned blocks = (unsigned)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
    const size_t hbytes = sizeof(float) * D.H * 2 * D.n;
    if (hbytes <= 48 * 1024)
      count_clean_smem_kernel<<<blocks < 296 ? blocks : 296, 256, hbytes, s>>>(D, idx, W.clean_cnt);
    else
      count_clean_kernel<<<blocks, 256, 0, s>>>(D, idx, W.clean_cnt);
    count_launch();
  }
  if ((e = cudaMemsetAsync(W.bal_ctr, 0, sizeof(int), s)) != cudaSuccess) return e;   // workspace starts undefined
  const unsigned fb = (unsigned)((D.H * 2 * D.n + 31) / 32);
  balance_finalize_kernel<<<fb, 256, 0, s>>>(D, W.p_part, planes, W.clean_cnt, W.bal_part, W.bal_ctr, balance_loss);
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
