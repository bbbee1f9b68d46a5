// Stage 2 of the product-key search, softmax, value gather and mix
// (memory.py:166-192), the routing counters (memory.py:196-216) and the
// SiLU gate of the layer block (model.py:118), fused in one kernel.
//
// One CTA per token, one warp per head.  Each warp
//   1. runs stage 2 (combine.cuh: k x k re-top-k over the eligible
//      candidates, slot ids, softmax weights);
//   2. streams its k value rows (16-byte loads, float32 accumulation in
//      registers) into a per-head partial sum.
// The CTA then sums the heads in a fixed order (deterministic) and applies
// the gate.  Counters use integer-valued float atomics (exact, order-free).
#include <float.h>

#include "combine.cuh"

namespace ml {

namespace {

template <int KM, typename VT, int VEC, int CH>
__global__ void __launch_bounds__(1024) combine_gather_kernel(
    Dims D, const __grid_constant__ PairTable pairs, const int* __restrict__ sub_idx,
    const float* __restrict__ sub_score, const float* __restrict__ sub_sel,
    const VT* __restrict__ values, int* __restrict__ slots, float* __restrict__ weights, float* __restrict__ out,
    float* __restrict__ memg, float* __restrict__ memg_hi, float* __restrict__ memg_lo,
    const float* __restrict__ gate, float* __restrict__ slot_counts, float* __restrict__ subkey_counts,
    float* __restrict__ top1_part, int* __restrict__ err, int64_t m0) {
  extern __shared__ float red[];  // [H][d]
  __shared__ uint16_t tab[128];   // pair table, staged for divergent per-lane reads
  __shared__ uint16_t lbtab[32];
  for (int i = threadIdx.x; i < pairs.count; i += blockDim.x) tab[i] = pairs.ij[i];
  for (int i = threadIdx.x; i < 32; i += blockDim.x) lbtab[i] = pairs.lb[i];
  __syncthreads();
  const int64_t m = m0 + blockIdx.x;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k = D.k, d = D.d;
  const int64_t ra = ((m * D.H + h) * 2) * k;

  const bool lk = lane < k;
  const HeadPick p = combine_head<KM>(D, tab, lbtab, pairs.count, sub_idx, sub_score, sub_sel, ra, lane, err);
  const int slot = p.slot, ia = p.ia, ib = p.ib;
  const float w = p.w, top1 = p.top1;
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
  if (values == nullptr) return;   // routing only (the host-table read gathers afterwards)

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
                      const float* gate, float* slot_counts, float* subkey_counts, int64_t m0) {
  const PairTable pairs = make_pairs(D.k);
#define ML_CG(CHV)                                                                                             \
  combine_gather_kernel<KM, VT, VEC, CHV><<<grid, block, smem, s>>>(D, pairs, W.sub_idx, W.sub_score, W.sub_sel, \
                                                                    values, slots, weights, out, memg, mhi, \
                                                                    mlo, gate, slot_counts, subkey_counts,  \
                                                                    W.top1_part, W.err, m0)
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
                     float* subkey_counts, cudaStream_t s, int64_t m0, int64_t count) {
  dim3 grid((unsigned)count), block(32 * D.H);
  size_t smem = sizeof(float) * D.H * D.d;
  const bool aligned = (reinterpret_cast<uintptr_t>(values) & 15) == 0;
  if (D.vdtype == MEMLAYER_F16)
    return launch_ch<KM, __half, 8>(D, ch_for(D.d / 8), grid, block, smem, s, W, (const __half*)values, slots,
                                    weights, out, memg, mhi, mlo, gate, slot_counts, subkey_counts, m0);
  if (D.vdtype == MEMLAYER_BF16)
    return launch_ch<KM, __nv_bfloat16, 8>(D, ch_for(D.d / 8), grid, block, smem, s, W,
                                           (const __nv_bfloat16*)values, slots, weights, out, memg, mhi, mlo,
                                           gate, slot_counts, subkey_counts, m0);
  if (D.d % 4 == 0 && aligned)
    return launch_ch<KM, float, 4>(D, ch_for(D.d / 4), grid, block, smem, s, W, (const float*)values, slots,
                                   weights, out, memg, mhi, mlo, gate, slot_counts, subkey_counts, m0);
  return launch_ch<KM, float, 1>(D, ch_for(D.d), grid, block, smem, s, W, (const float*)values, slots, weights,
                                 out, memg, mhi, mlo, gate, slot_counts, subkey_counts, m0);
}

}  // namespace

cudaError_t launch_combine_gather(const Dims& D, const Work& W, const void* values, int* slots, float* weights,
                                  float* out, float* mem_gated, float* memg_hi, float* memg_lo, const float* gate,
                                  float* slot_counts, float* subkey_counts, cudaStream_t s, int64_t m0,
                                  int64_t count) {
  if (count <= 0) count = D.M - m0;
  if (count <= 0) return cudaSuccess;
#define ML_K(KV)                                                                                              \
  launch_k<KV>(D, W, values, slots, weights, out, mem_gated, memg_hi, memg_lo, gate, slot_counts, subkey_counts, s, \
               m0, count)
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
