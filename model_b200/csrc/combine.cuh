// Stage 2 of the product-key search for one (token, head) on one warp:
// k x k cartesian re-top-k, slot ids and softmax weights (memory.py:166-178).
// Shared by the single-GPU gather kernel and the row-sharded push kernel.
//
// Both stage-1 lists are sorted (value desc, index asc), so candidate (i, j)
// is dominated by every (i', j') with i' <= i, j' <= j, which rank ahead of
// it under (value desc, flat index asc); with (i+1)(j+1) > k at least k
// candidates rank ahead, so only the candidates with (i+1)(j+1) <= k can be
// selected (8 / 20 / 50 / 119 of them for k = 4 / 8 / 16 / 32).  Those are
// sorted across the warp by a bitonic network on (value desc, flat index
// asc), which is lax.top_k's order on the full k*k list (memory.py:171);
// candidates under a lower bound of the k-th best sum are dropped first, so
// the sort is usually 32 wide.
#pragma once

#include "common.cuh"

namespace ml {

// rna_tf32(x): the high half of the 3xTF32 split used by the tensor-core GEMMs.
__device__ __forceinline__ float tc_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// VEC consecutive value-row elements as float32.
template <typename VT, int VEC>
__device__ __forceinline__ void load_group(const VT* p, float (&o)[VEC]) {
  if constexpr (VEC == 1) {
    o[0] = VecLoad<VT>::scalar(p);
  } else {
    VecLoad<VT>::load(p, o);
  }
}

// Eligible stage-2 candidates (i, j) with (i+1)(j+1) <= k, row-major, and
// the k candidates with the smallest (i+1)(j+1): the minimum of their sums is
// a lower bound of the k-th best sum (at least k candidates reach it).
struct PairTable {
  uint16_t ij[128];  // i | j << 8
  uint16_t lb[32];   // the k most dominant pairs
  int count;
};

inline PairTable make_pairs(int k) {
  PairTable t{};
  int c = 0;
  for (int i = 0; i < k; ++i)
    for (int j = 0; j < k && (i + 1) * (j + 1) <= k; ++j) t.ij[c++] = (uint16_t)(i | (j << 8));
  t.count = c;
  int n = 0;
  for (int prod = 1; n < k; ++prod)          // products in increasing order, row-major within one
    for (int i = 0; i < k && n < k; ++i)
      if (prod % (i + 1) == 0 && prod / (i + 1) - 1 < k) t.lb[n++] = (uint16_t)(i | ((prod / (i + 1) - 1) << 8));
  return t;
}

// Position of the n-th (0-based) set bit of m; requires n < popc(m).
__device__ __forceinline__ int nth_set_bit(unsigned m, int n) {
  int pos = 0;
#pragma unroll
  for (int w = 16; w > 0; w >>= 1) {
    const int c = __popc((unsigned)(((uint64_t)m >> pos) & ((1ull << w) - 1)));
    if (c <= n) {
      n -= c;
      pos += w;
    }
  }
  return pos;
}

// Bitonic sort of 32*C (value, flat) pairs held C per lane (position
// lane*C + r) into (value desc, flat asc) order.  Flats must be distinct.
template <int C>
__device__ __forceinline__ void warp_sort_desc(float (&v)[C], int (&f)[C], int lane) {
  constexpr int N = 32 * C;
#pragma unroll
  for (int size = 2; size <= N; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride < C) {
#pragma unroll
        for (int r = 0; r < C; ++r) {
          const int rp = r ^ stride;
          if (rp > r) {
            const bool desc = ((lane * C + r) & size) == 0;
            const bool swap = desc ? ranks_before(v[rp], f[rp], v[r], f[r]) : ranks_before(v[r], f[r], v[rp], f[rp]);
            if (swap) {
              const float tv = v[r];
              v[r] = v[rp];
              v[rp] = tv;
              const int tf = f[r];
              f[r] = f[rp];
              f[rp] = tf;
            }
          }
        }
      } else {
        const int ls = stride / C;
#pragma unroll
        for (int r = 0; r < C; ++r) {
          const float ov = __shfl_xor_sync(FULL, v[r], ls);
          const int of = __shfl_xor_sync(FULL, f[r], ls);
          const bool lower = (lane & ls) == 0;
          const bool desc = ((lane * C + r) & size) == 0;
          const bool mine_better = ranks_before(v[r], f[r], ov, of);
          if (mine_better != (lower == desc)) {
            v[r] = ov;
            f[r] = of;
          }
        }
      }
    }
  }
}

// Result of stage 2 on one warp: lane r < k holds the r-th winner.
struct HeadPick {
  int slot;    // ia * n + ib (memory.py:175)
  int ia, ib;  // sub-key ids of the two halves
  float w;     // softmax weight (memory.py:178)
  float top1;  // max weight over the k winners (every lane)
};

// One (token m, head h) on one warp.  `tab` is the pair table staged in
// shared memory; ra indexes the head's first-half stage-1 list.
template <int KM>
__device__ __forceinline__ HeadPick combine_head(const Dims& D, const uint16_t* tab, const uint16_t* lbtab,
                                                 int pair_count, const int* __restrict__ sub_idx,
                                                 const float* __restrict__ sub_score,
                                                 const float* __restrict__ sub_sel, int64_t ra, int lane,
                                                 int* __restrict__ err) {
  constexpr int C = KM <= 8 ? 1 : KM <= 16 ? 2 : 4;   // candidate slots per lane (32*C >= eligible count)
  const int k = D.k;
  const int64_t rb = ra + k;
  const bool lk = lane < k;
  const float as = lk ? sub_sel[ra + lane] : -INFINITY;
  const float bs = lk ? sub_sel[rb + lane] : -INFINITY;
  // without selection noise the clean scores are the selection scores
  const float* scs = D.noisy ? sub_score : sub_sel;
  const float ac = lk ? scs[ra + lane] : 0.f;
  const float bc = lk ? scs[rb + lane] : 0.f;
  const int ai = lk ? sub_idx[ra + lane] : 0;
  const int bi = lk ? sub_idx[rb + lane] : 0;

  // eligible candidates into slots lane*C + r; padding ranks last
  float cv[C];
  int cf[C];
#pragma unroll
  for (int r = 0; r < C; ++r) {
    const int slot = lane * C + r;
    const bool ok = slot < pair_count;
    const int ij = ok ? tab[slot] : 0;
    const int i = ij & 0xFF, j = ij >> 8;
    const float x = __shfl_sync(FULL, as, i);
    const float y = __shfl_sync(FULL, bs, j);
    cv[r] = ok ? x + y : -INFINITY;                  // memory.py:168 cand_select
    cf[r] = ok ? i * k + j : (1 << 30) + slot;       // flat index in the k*k grid
  }
  // candidates below the k-th best's lower bound cannot be selected: when at
  // most 32 remain, one per lane, a 32-wide sort replaces the 32*C-wide one
  unsigned msk[C];
  int basep[C], tot = 64;
  if constexpr (C > 1) {
    const int lij = lane < k ? lbtab[lane] : 0;
    const float lbs = __shfl_sync(FULL, as, lij & 0xFF) + __shfl_sync(FULL, bs, lij >> 8);
    float bound = lane < k ? lbs : INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bound = fminf(bound, __shfl_xor_sync(FULL, bound, o));
    tot = 0;
#pragma unroll
    for (int r = 0; r < C; ++r) {
      msk[r] = __ballot_sync(FULL, cv[r] >= bound);
      basep[r] = tot;
      tot += __popc(msk[r]);
    }
  }
  int my_flat = 0;
  if (C > 1 && tot <= 32) {
    int rr = -1, nn = 0;
#pragma unroll
    for (int r = 0; r < C; ++r)
      if (rr < 0 && lane < basep[r] + __popc(msk[r])) {
        rr = r;
        nn = lane - basep[r];
      }
    const int src = rr >= 0 ? nth_set_bit(msk[rr], nn) : 0;
    float v1[1] = {-INFINITY};
    int f1[1] = {(1 << 30) + 128 + lane};      // padding: distinct, ranks last
#pragma unroll
    for (int r = 0; r < C; ++r) {
      const float tv = __shfl_sync(FULL, cv[r], src);
      const int tf = __shfl_sync(FULL, cf[r], src);
      if (rr == r) {
        v1[0] = tv;
        f1[0] = tf;
      }
    }
    warp_sort_desc<1>(v1, f1, lane);
    my_flat = f1[0];
  } else {
    warp_sort_desc<C>(cv, cf, lane);
    // lane r < k takes sorted position r
#pragma unroll
    for (int r = 0; r < C; ++r) {
      const int f = __shfl_sync(FULL, cf[r], lane / C);
      if ((lane % C) == r) my_flat = f;
    }
  }
  const int fi = lk ? my_flat / k : 0, fj = lk ? my_flat - (my_flat / k) * k : 0;
  const float s = __shfl_sync(FULL, ac, fi) + __shfl_sync(FULL, bc, fj);     // memory.py:172
  int ia = __shfl_sync(FULL, ai, fi), ib = __shfl_sync(FULL, bi, fj);        // memory.py:173-174
  if (lk && ((unsigned)ia >= (unsigned)D.n || (unsigned)ib >= (unsigned)D.n)) {
    // a sub-key id out of range can only come from a bug upstream: record
    // it (status read by the host) and read row 0 instead of faulting
    atomicCAS(err, 0, 21);
    ia = 0;
    ib = 0;
  }
  HeadPick p;
  p.ia = ia;
  p.ib = ib;
  p.slot = ia * D.n + ib;                                                    // memory.py:175
  const float mx = warp_max(lk ? s : -INFINITY);
  const float e = lk ? expf(s - mx) : 0.f;
  p.w = e / warp_sum(e);                                                     // memory.py:178
  p.top1 = warp_max(lk ? p.w : -INFINITY);
  return p;
}

}  // namespace ml
