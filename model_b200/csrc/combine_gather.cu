// Stage 2 of the product-key search, softmax, value gather and mix
// (memory.py:166-192), the routing counters (memory.py:196-216) and the
// SiLU gate of the layer block (model.py:118), fused in one kernel.
//
// One CTA per token, one warp per head.  Each warp
//   1. forms the k x k cartesian candidates a_i + b_j of its two stage-1
//      lists.  Both lists are sorted (value desc, index asc), so candidate
//      (i, j) is dominated by every (i', j') with i' <= i, j' <= j, which
//      rank ahead of it under (value desc, flat index asc); with
//      (i+1)(j+1) > k at least k candidates rank ahead, so only the
//      candidates with (i+1)(j+1) <= k can be selected.  The top-k of those
//      is taken by k rounds of warp arg-max with lowest-flat-index ties,
//      which is lax.top_k's order on the full k*k list (memory.py:171);
//   2. turns the k winners into slot ids idx_a * n + idx_b (memory.py:172-175)
//      and softmax weights (memory.py:178);
//   3. streams its k value rows (16-byte loads, float32 accumulation in
//      registers) into a per-head partial sum.
// The CTA then sums the heads in a fixed order (deterministic) and applies
// the gate.  Counters use integer-valued float atomics (exact, order-free).
#include <float.h>

#include "common.cuh"

namespace ml {

namespace {

__device__ __forceinline__ float tc_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

template <typename VT, int VEC>
__device__ __forceinline__ void load_group(const VT* p, float (&o)[VEC]) {
  if constexpr (VEC == 1) {
    o[0] = VecLoad<VT>::scalar(p);
  } else {
    VecLoad<VT>::load(p, o);
  }
}

template <int KM, typename VT, int VEC, int CH>
__global__ void __launch_bounds__(1024) combine_gather_kernel(
    Dims D, const int* __restrict__ sub_idx, const float* __restrict__ sub_score, const float* __restrict__ sub_sel,
    const VT* __restrict__ values, int* __restrict__ slots, float* __restrict__ weights, float* __restrict__ out,
    float* __restrict__ memg, float* __restrict__ memg_hi, float* __restrict__ memg_lo,
    const float* __restrict__ gate, float* __restrict__ slot_counts, float* __restrict__ subkey_counts,
    float* __restrict__ top1_part) {
  extern __shared__ float red[];  // [H][d]
  constexpr int CPL = (KM * KM + 31) / 32;
  const int64_t m = blockIdx.x;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k = D.k, d = D.d;
  const int64_t ra = ((m * D.H + h) * 2) * k, rb = ra + k;

  const bool lk = lane < k;
  const float as = lk ? sub_sel[ra + lane] : -INFINITY;
  const float bs = lk ? sub_sel[rb + lane] : -INFINITY;
  const float ac = lk ? sub_score[ra + lane] : 0.f;
  const float bc = lk ? sub_score[rb + lane] : 0.f;
  const int ai = lk ? sub_idx[ra + lane] : 0;
  const int bi = lk ? sub_idx[rb + lane] : 0;

  // candidate f = lane + 32 t  (i = f / k, j = f % k)
  float cv[CPL];
  uint32_t used = 0;
#pragma unroll
  for (int t = 0; t < CPL; ++t) {
    const int f = lane + 32 * t;
    const int i = f / k, j = f - (f / k) * k;
    const float x = __shfl_sync(FULL, as, i & 31);
    const float y = __shfl_sync(FULL, bs, j & 31);
    const bool ok = f < k * k && (i + 1) * (j + 1) <= k;
    cv[t] = x + y;
    if (!ok) used |= 1u << t;
  }
  int my_flat = 0;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bf = INT_MAX;
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const int f = lane + 32 * t;
      if (!((used >> t) & 1u) && ranks_before(cv[t], f, bv, bf)) {
        bv = cv[t];
        bf = f;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(FULL, bv, o);
      const int of = __shfl_xor_sync(FULL, bf, o);
      if (ranks_before(ov, of, bv, bf)) {
        bv = ov;
        bf = of;
      }
    }
    if (lane == (bf & 31)) used |= 1u << (bf >> 5);
    if (lane == r) my_flat = bf;
  }
  const int fi = lk ? my_flat / k : 0, fj = lk ? my_flat - (my_flat / k) * k : 0;
  const float s = __shfl_sync(FULL, ac, fi) + __shfl_sync(FULL, bc, fj);     // memory.py:172
  const int ia = __shfl_sync(FULL, ai, fi), ib = __shfl_sync(FULL, bi, fj);  // memory.py:173-174
  const int slot = ia * D.n + ib;                                            // memory.py:175
  const float mx = warp_max(lk ? s : -INFINITY);
  const float e = lk ? expf(s - mx) : 0.f;
  const float w = e / warp_sum(e);                                           // memory.py:178
  const float top1 = warp_max(lk ? w : -INFINITY);
  const int64_t ow = (m * D.H + h) * k;
  if (lk) {
    slots[ow + lane] = slot;
    weights[ow + lane] = w;
    if (slot_counts) atomicAdd(&slot_counts[slot], 1.f);                      // memory.py:216
    if (subkey_counts) {                                                     // memory.py:205
      atomicAdd(&subkey_counts[(int64_t)(h * 2) * D.n + ia], 1.f);
      atomicAdd(&subkey_counts[(int64_t)(h * 2 + 1) * D.n + ib], 1.f);
    }
  }
  if (lane == 0 && top1_part) top1_part[m * D.H + h] = top1;

  // read (slot + N/2 + 1) % N under shuffle_reads (memory.py:179)
  const int64_t rs = D.shuffle ? ((int64_t)slot + D.N / 2 + 1) % D.N : (int64_t)slot;
  float acc[CH][VEC];
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[c][v] = 0.f;
  const int groups = d / VEC;
#pragma unroll 4
  for (int r = 0; r < k; ++r) {
    const int64_t row = __shfl_sync(FULL, rs, r);
    const float wr = __shfl_sync(FULL, w, r);
    const VT* base = values + row * d;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int g = c * 32 + lane;
      if (g < groups) {
        float x[VEC];
        load_group<VT, VEC>(base + g * VEC, x);
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[c][v] = fmaf(wr, x[v], acc[c][v]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int g = c * 32 + lane;
    if (g < groups) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) red[h * d + g * VEC + v] = acc[c][v];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float o = 0.f;
    for (int hh = 0; hh < D.H; ++hh) o += red[hh * d + i];   // heads summed (memory.py:192)
    if (out) out[m * d + i] = o;
    if (memg || memg_hi) {
      const float g = o * gate[m * d + i];                   // model.py:119 mem * gate
      if (memg) memg[m * d + i] = g;
      if (memg_hi) {                                         // tf32 halves for the tensor-core out GEMM
        const float hi = tc_round(g);
        memg_hi[m * d + i] = hi;
        memg_lo[m * d + i] = tc_round(g - hi);
      }
    }
  }
}

template <int KM, typename VT, int VEC>
cudaError_t launch_ch(const Dims& D, int ch, dim3 grid, dim3 block, size_t smem, cudaStream_t s, const Work& W,
                      const VT* values, int* slots, float* weights, float* out, float* memg, float* mhi, float* mlo,
                      const float* gate, float* slot_counts, float* subkey_counts) {
#define ML_CG(CHV)                                                                                             \
  combine_gather_kernel<KM, VT, VEC, CHV><<<grid, block, smem, s>>>(D, W.sub_idx, W.sub_score, W.sub_sel,    \
                                                                    values, slots, weights, out, memg, mhi, \
                                                                    mlo, gate, slot_counts, subkey_counts,  \
                                                                    W.top1_part)
  switch (ch) {
    case 1: ML_CG(1); break;
    case 2: ML_CG(2); break;
    case 4: ML_CG(4); break;
    case 8: ML_CG(8); break;
    default: return cudaErrorInvalidValue;
  }
#undef ML_CG
  count_launch();
  return cudaGetLastError();
}

inline int ch_for(int groups) {
  int ch = (groups + 31) / 32;
  return ch <= 1 ? 1 : ch <= 2 ? 2 : ch <= 4 ? 4 : ch <= 8 ? 8 : -1;
}

template <int KM>
cudaError_t launch_k(const Dims& D, const Work& W, const void* values, int* slots, float* weights, float* out,
                     float* memg, float* mhi, float* mlo, const float* gate, float* slot_counts,
                     float* subkey_counts, cudaStream_t s) {
  dim3 grid((unsigned)D.M), block(32 * D.H);
  size_t smem = sizeof(float) * D.H * D.d;
  const bool aligned = (reinterpret_cast<uintptr_t>(values) & 15) == 0;
  if (D.vdtype == MEMLAYER_F16)
    return launch_ch<KM, __half, 8>(D, ch_for(D.d / 8), grid, block, smem, s, W, (const __half*)values, slots,
                                    weights, out, memg, mhi, mlo, gate, slot_counts, subkey_counts);
  if (D.vdtype == MEMLAYER_BF16)
    return launch_ch<KM, __nv_bfloat16, 8>(D, ch_for(D.d / 8), grid, block, smem, s, W,
                                           (const __nv_bfloat16*)values, slots, weights, out, memg, mhi, mlo,
                                           gate, slot_counts, subkey_counts);
  if (D.d % 4 == 0 && aligned)
    return launch_ch<KM, float, 4>(D, ch_for(D.d / 4), grid, block, smem, s, W, (const float*)values, slots,
                                   weights, out, memg, mhi, mlo, gate, slot_counts, subkey_counts);
  return launch_ch<KM, float, 1>(D, ch_for(D.d), grid, block, smem, s, W, (const float*)values, slots, weights,
                                 out, memg, mhi, mlo, gate, slot_counts, subkey_counts);
}

}  // namespace

cudaError_t launch_combine_gather(const Dims& D, const Work& W, const void* values, int* slots, float* weights,
                                  float* out, float* mem_gated, float* memg_hi, float* memg_lo, const float* gate,
                                  float* slot_counts, float* subkey_counts, cudaStream_t s) {
  if (D.M == 0) return cudaSuccess;
#define ML_K(KV) \
  launch_k<KV>(D, W, values, slots, weights, out, mem_gated, memg_hi, memg_lo, gate, slot_counts, subkey_counts, s)
  switch (D.kmax) {
    case 4: return ML_K(4);
    case 8: return ML_K(8);
    case 16: return ML_K(16);
    case 32: return ML_K(32);
    default: return cudaErrorInvalidValue;
  }
#undef ML_K
}

}  // namespace ml
