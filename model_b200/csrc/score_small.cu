// Stage 1 of the product-key search (memory.py:149-164) for few tokens
// (decode batches): the sub-keys of each codebook are split into slices of
// 256 keys over many CTAs, so a call with one token still spreads over the
// GPU.  Each CTA scores its slice against up to 8 tokens of the call (float32
// dot products, the same operation order as the 128-token SIMT path), keeps
// each token's top-k of the slice (per-lane sorts of 8 keys, then a warp
// tournament on (value desc, key asc)), and a merge kernel selects the top-k
// of all slices per (token, head, half): a tournament over the slice lists
// (one list per lane) for up to 32 slices, a warp bitonic sort of all slice
// candidates beyond.  Ties resolve lowest key first, as lax.top_k does (in
// the bitonic merge, equal values keep slice-list order, which is key
// order).
#include "combine.cuh"

namespace ml {

namespace {

constexpr int SLICE = 256;      // keys per CTA
constexpr int SMALL_M = 64;     // most tokens per call on this path
constexpr int MB = 8;           // tokens per CTA (grid z covers the call's tokens)
constexpr int KS_LD = 36;       // padded row of the staged key chunk (conflict-free float4 reads)

template <int KM, bool NOISY>
__global__ void __launch_bounds__(SLICE) score_slice_kernel(Dims D, int S, const float* __restrict__ qn,
                                                            const float* __restrict__ qlen,
                                                            const float* __restrict__ keys_n,
                                                            const float* __restrict__ gumbel,
                                                            const float* __restrict__ scal,
                                                            float* __restrict__ part_sel,
                                                            float* __restrict__ part_clean,
                                                            int* __restrict__ part_key) {
  extern __shared__ float sm[];
  const int half = D.half, HC = D.H * 2;
  const int mz = blockIdx.z * MB;                       // first token of this CTA
  const int M = min(MB, (int)D.M - mz);                 // tokens of this CTA
  float* qs = sm;                          // [MB][half]
  float* ssel = qs + MB * half;            // [MB][SLICE] selection scores
  float* scln = ssel + MB * SLICE;         // [MB][SLICE] clean scores
  float* ks = scln + MB * SLICE;           // [SLICE][KS_LD] one 32-dimension chunk of the slice's keys
  const int s = blockIdx.x, hc = blockIdx.y, h = hc >> 1, c = hc & 1;
  for (int e = threadIdx.x; e < M * half; e += SLICE) {
    const int m = e / half, i = e - m * half;
    qs[e] = qn[((int64_t)((mz + m) * D.H + h) * 2 + c) * half + i];
  }
  __syncthreads();
  const int key = s * SLICE + threadIdx.x;
  const bool kv = key < D.n;
  float acc[MB];
#pragma unroll
  for (int m = 0; m < MB; ++m) acc[m] = 0.f;
  const float* kbase = keys_n + ((int64_t)hc * D.n + (int64_t)s * SLICE) * half;
  const int nkeys = min(SLICE, D.n - s * SLICE);
  for (int dc = 0; dc < half; dc += 32) {
    // coalesced copy of the slice's keys, dimensions [dc, dc + 32)
    const int dw = min(32, half - dc) / 4;        // float4 per key in this chunk
    __syncthreads();
    for (int e = threadIdx.x; e < nkeys * dw; e += SLICE) {
      const int kj = e / dw, d4 = e - kj * dw;
      *reinterpret_cast<float4*>(ks + kj * KS_LD + d4 * 4) =
          __ldg(reinterpret_cast<const float4*>(kbase + (int64_t)kj * half + dc) + d4);
    }
    __syncthreads();
    if (kv) {
      for (int d4 = 0; d4 < dw; ++d4) {
        const float4 kk = *reinterpret_cast<const float4*>(ks + threadIdx.x * KS_LD + d4 * 4);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          if (m < M) {   // dot product in dimension order (memory.py:149)
            const float4 q = *reinterpret_cast<const float4*>(qs + m * half + dc + d4 * 4);
            acc[m] = fmaf(q.x, kk.x, acc[m]);
            acc[m] = fmaf(q.y, kk.y, acc[m]);
            acc[m] = fmaf(q.z, kk.z, acc[m]);
            acc[m] = fmaf(q.w, kk.w, acc[m]);
          }
        }
      }
    }
  }
  const float T = scal[0];
#pragma unroll
  for (int m = 0; m < MB; ++m) {
    if (m < M) {
      const int64_t row = (int64_t)((mz + m) * D.H + h) * 2 + c;
      float score = __fmul_rn(acc[m], T);                                       // memory.py:150
      if (D.qscale) score = __fmul_rn(score, qlen[row]);                        // memory.py:151-152
      float sel = score;
      if (NOISY && kv) sel = __fadd_rn(score, __fmul_rn(D.noise_coef, gumbel[row * D.n + key]));   // :158
      ssel[m * SLICE + threadIdx.x] = kv ? sel : -INFINITY;
      scln[m * SLICE + threadIdx.x] = score;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int C = SLICE / 32;
  for (int m = warp; m < M; m += SLICE / 32) {
    // each lane sorts its 8 keys (value desc, key asc), then KM rounds of a
    // warp tournament pop the best remaining head
    float v[C];
    int f[C];
#pragma unroll
    for (int r = 0; r < C; ++r) {
      const int pos = lane * C + r;
      v[r] = ssel[m * SLICE + pos];
      f[r] = s * SLICE + pos;      // key id (keys past n carry -inf and lose every tie-free comparison)
    }
#pragma unroll
    for (int a = 0; a < C; ++a)
#pragma unroll
      for (int b = C - 1; b > a; --b)
        if (ranks_before(v[b], f[b], v[b - 1], f[b - 1])) {
          const float tv = v[b]; v[b] = v[b - 1]; v[b - 1] = tv;
          const int tf = f[b]; f[b] = f[b - 1]; f[b - 1] = tf;
        }
    const int64_t base = ((int64_t)((mz + m) * HC + hc) * S + s) * KM;
    for (int j = 0; j < KM; ++j) {
      float bv = v[0];
      int bf = f[0];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, bv, o);
        const int of = __shfl_xor_sync(FULL, bf, o);
        if (ranks_before(ov, of, bv, bf)) {
          bv = ov;
          bf = of;
        }
      }
      if (f[0] == bf) {            // the winning lane pops its head
#pragma unroll
        for (int r = 0; r < C - 1; ++r) {
          v[r] = v[r + 1];
          f[r] = f[r + 1];
        }
        v[C - 1] = -INFINITY;
        f[C - 1] = 0x7fffffff;
      }
      if (lane == 0) {
        part_sel[base + j] = bv;
        part_key[base + j] = bf;
        part_clean[base + j] = bf < D.n ? scln[m * SLICE + (bf - s * SLICE)] : -INFINITY;
      }
    }
  }
}

// One warp per (token, codebook): top-k of the S * KM slice candidates.
template <int KM, int C>
__global__ void __launch_bounds__(256) score_merge_kernel(Dims D, int S, const float* __restrict__ part_sel,
                                                          const float* __restrict__ part_clean,
                                                          const int* __restrict__ part_key,
                                                          int* __restrict__ sub_idx, float* __restrict__ sub_score,
                                                          float* __restrict__ sub_sel) {
  const int lane = threadIdx.x & 31;
  const int64_t rowi = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);   // m * H*2 + hc = output row
  if (rowi >= D.M * D.H * 2) return;
  const int total = S * KM;
  const int64_t base = rowi * total;
  float v[C];
  int f[C];
#pragma unroll
  for (int r = 0; r < C; ++r) {
    const int pos = lane * C + r;
    const bool ok = pos < total;
    v[r] = ok ? part_sel[base + pos] : -INFINITY;
    f[r] = ok ? pos : (1 << 30) + pos;   // equal values: lower position = lower key
  }
  warp_sort_desc<C>(v, f, lane);
  const int k = D.k;
#pragma unroll
  for (int r = 0; r < C; ++r) {
    const int pos = lane * C + r;
    if (pos < k) {
      const int src = f[r];
      sub_idx[rowi * k + pos] = part_key[base + src];
      sub_sel[rowi * k + pos] = v[r];
      sub_score[rowi * k + pos] = part_clean[base + src];
    }
  }
}

// With at most 32 slices: lane s holds slice s's sorted list in registers and
// k rounds of a warp tournament pop the best head (value desc, key asc).
template <int KM>
__global__ void __launch_bounds__(256) score_merge32_kernel(Dims D, int S, const float* __restrict__ part_sel,
                                                            const float* __restrict__ part_clean,
                                                            const int* __restrict__ part_key,
                                                            int* __restrict__ sub_idx, float* __restrict__ sub_score,
                                                            float* __restrict__ sub_sel) {
  const int lane = threadIdx.x & 31;
  const int64_t rowi = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);   // m * H*2 + hc = output row
  if (rowi >= D.M * D.H * 2) return;
  const int64_t base = (rowi * S + lane) * KM;
  float v[KM], cl[KM];
  int f[KM];
#pragma unroll
  for (int j = 0; j < KM; ++j) {
    v[j] = lane < S ? part_sel[base + j] : -INFINITY;
    f[j] = lane < S ? part_key[base + j] : 0x7fffffff;
    cl[j] = lane < S ? part_clean[base + j] : 0.f;
  }
  const int k = D.k;
  for (int j = 0; j < k; ++j) {
    float bv = v[0];
    int bf = f[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(FULL, bv, o);
      const int of = __shfl_xor_sync(FULL, bf, o);
      if (ranks_before(ov, of, bv, bf)) {
        bv = ov;
        bf = of;
      }
    }
    if (f[0] == bf && lane < S) {      // keys are distinct across slices: one winner
      sub_idx[rowi * k + j] = bf;
      sub_sel[rowi * k + j] = bv;
      sub_score[rowi * k + j] = cl[0];
#pragma unroll
      for (int r = 0; r < KM - 1; ++r) {
        v[r] = v[r + 1];
        f[r] = f[r + 1];
        cl[r] = cl[r + 1];
      }
      v[KM - 1] = -INFINITY;
      f[KM - 1] = 0x7fffffff;
    }
  }
}

inline int slices(const Dims& D) { return (D.n + SLICE - 1) / SLICE; }

template <int KM>
cudaError_t launch_small_k(const Dims& D, const Work& W, const float* gumbel, float* scratch, cudaStream_t s) {
  const int S = slices(D), HC = D.H * 2;
  float* part_sel = scratch;
  float* part_clean = part_sel + (int64_t)D.M * HC * S * KM;
  int* part_key = reinterpret_cast<int*>(part_clean + (int64_t)D.M * HC * S * KM);
  const size_t smem = sizeof(float) * ((size_t)MB * D.half + 2 * (size_t)MB * SLICE + SLICE * KS_LD);
  auto k1 = D.noisy ? score_slice_kernel<KM, true> : score_slice_kernel<KM, false>;
  cudaError_t e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k1<<<dim3(S, HC, (unsigned)((D.M + MB - 1) / MB)), SLICE, smem, s>>>(D, S, W.qn, W.qlen, W.keys_n, gumbel, W.scal,
                                                                       part_sel, part_clean, part_key);
  const unsigned blocks = (unsigned)((D.M * HC + 7) / 8);
  const int total = S * KM;
  const int C = total <= 32 ? 1 : total <= 64 ? 2 : total <= 128 ? 4 : total <= 256 ? 8 : total <= 512 ? 16 : 32;
#define ML_MG(CV) \
  score_merge_kernel<KM, CV><<<blocks, 256, 0, s>>>(D, S, part_sel, part_clean, part_key, W.sub_idx, W.sub_score, W.sub_sel)
  if (S <= 32) {
    score_merge32_kernel<KM><<<blocks, 256, 0, s>>>(D, S, part_sel, part_clean, part_key, W.sub_idx, W.sub_score,
                                                    W.sub_sel);
    count_launch(2);
    return cudaGetLastError();
  }
  switch (C) {
    case 1: ML_MG(1); break;
    case 2: ML_MG(2); break;
    case 4: ML_MG(4); break;
    case 8: ML_MG(8); break;
    case 16: ML_MG(16); break;
    default: ML_MG(32); break;
  }
#undef ML_MG
  count_launch(2);
  return cudaGetLastError();
}

}  // namespace

bool score_small_supported(const Dims& D) {
  return D.M >= 1 && D.M <= SMALL_M && D.half % 4 == 0 && (int64_t)slices(D) * D.kmax <= 1024 &&
         sizeof(float) * ((size_t)MB * D.half + 2 * (size_t)MB * SLICE + SLICE * KS_LD) <= 200 * 1024;
}

size_t score_small_scratch_bytes(const Dims& D) {
  return (size_t)D.M * D.H * 2 * slices(D) * D.kmax * 12;
}

cudaError_t launch_score_small(const Dims& D, const Work& W, const float* gumbel, float* scratch, cudaStream_t s) {
  switch (D.kmax) {
    case 4: return launch_small_k<4>(D, W, gumbel, scratch, s);
    case 8: return launch_small_k<8>(D, W, gumbel, scratch, s);
    case 16: return launch_small_k<16>(D, W, gumbel, scratch, s);
    case 32: return launch_small_k<32>(D, W, gumbel, scratch, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ml
