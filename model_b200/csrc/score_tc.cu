// Stage 1 of the product-key search on the 5th-generation tensor cores
// (memory.py:149-164): cos = q_hat . k_hat for every (token, head, half,
// sub-key), scaled by the temperature (and |q| under query_scale), with the
// per-(token, head, half) top-k taken in the TMEM epilogue, so the
// [M, H, 2, n] score tensor never reaches global memory.
//
// Precision: routing must reproduce float32 slot selection, which a single
// tf32 product (10-bit mantissa) does not.  Each operand is split into
// x = hi + lo with hi = rna_tf32(x), lo = rna_tf32(x - hi) (|x - hi - lo| <=
// 2^-22 |x|), and the score is accumulated in float32 TMEM as
// hi.hi + hi.lo + lo.hi (three kind::tf32 MMAs per K step), which keeps the
// cosine within a few float32 ulps of a float32 dot product.
//
// CTA = 10 warps, persistent over work units (128-token tile, head, half):
//   warp 0     TMA producer: A = q_hi / q_lo [128 x 32] and B = k_hi / k_lo
//              [BN x 32] tiles (128-byte swizzle) into a multi-stage ring;
//   warp 1     TMEM allocator and MMA issuer (one thread): 128 x BN float32
//              accumulators, double-buffered in TMEM (2 x 256 columns);
//   warps 2-9  epilogue.  TMEM lane = token row; the two warps that share a
//              lane quarter split each chunk's columns in halves.  Each
//              thread keeps a sorted register top-k (value desc, index asc)
//              of its row's half.  Per chunk a group-max pass gives a lower
//              bound of the chunk's k-th best score; values beating both it
//              and the list's k-th are collected 16 at a time as a bit mask
//              and inserted in lockstep across the warp (no per-value
//              divergence).  At the end of a unit the two halves of every
//              row are merged through shared memory.
// Every mbarrier wait is bounded; a timeout sets an error code and unwinds.
#include <cudaTypedefs.h>

#include <mutex>

#include "tc_pipeline.cuh"

namespace ml {

namespace {

constexpr int TC_M = tc::PIPE_M;   // tokens per tile (UMMA M)
constexpr int TC_K = tc::PIPE_K;   // float32 elements per 128-byte swizzled row
constexpr int EPI_WARPS = 8;
constexpr int TC_THREADS = 64 + 32 * EPI_WARPS;
constexpr int ACC_STRIDE = tc::PIPE_ACC_STRIDE;

struct TcShape {
  tc::PipeShape P;
  int m_tiles;     // 128-token tiles of this launch
  int mt0;         // first tile of this launch
  int n_chunks;
  uint32_t merge_off;
};

// Smallest float32 strictly greater than v (v not NaN, v < +inf).
__device__ __forceinline__ float succ_f32(float v) {
  if (v == 0.f) return __int_as_float(1);
  const int b = __float_as_int(v);
  return __int_as_float(v > 0.f ? b + 1 : b - 1);
}

// Index of the single set bit of a one-hot 16-bit word, on the ALU pipe.
__device__ __forceinline__ int low_bit_index16(uint32_t low) {
  return ((low & 0xFF00u) ? 8 : 0) | ((low & 0xF0F0u) ? 4 : 0) | ((low & 0xCCCCu) ? 2 : 0) |
         ((low & 0xAAAAu) ? 1 : 0);
}

// a[t] for a runtime t in [0, 16): select tree, no local memory.
__device__ __forceinline__ float pick16(const float (&a)[16], int t) {
  float l8[8], l4[4], l2[2];
#pragma unroll
  for (int i = 0; i < 8; ++i) l8[i] = (t & 8) ? a[i + 8] : a[i];
#pragma unroll
  for (int i = 0; i < 4; ++i) l4[i] = (t & 4) ? l8[i + 4] : l8[i];
#pragma unroll
  for (int i = 0; i < 2; ++i) l2[i] = (t & 2) ? l4[i + 2] : l4[i];
  return (t & 1) ? l2[1] : l2[0];
}

// ---- sorting networks (all indices compile-time; registers only) ----------
// Bitonic sort of N values into descending order.
template <int N>
__device__ __forceinline__ void sort_desc_v(float (&v)[N]) {
#pragma unroll
  for (int size = 2; size <= N; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1)
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int l = i ^ stride;
        if (l > i) {
          const float a = v[i], b = v[l];
          if ((i & size) == 0) {
            v[i] = fmaxf(a, b);
            v[l] = fminf(a, b);
          } else {
            v[i] = fminf(a, b);
            v[l] = fmaxf(a, b);
          }
        }
      }
}

// (value desc, index asc) order without short-circuit branches.
__device__ __forceinline__ bool before_nb(float va, int ia, float vb, int ib) {
  return (va > vb) | ((va == vb) & (ia < ib));
}

// Compare-exchange of pairs i, l: the better one goes to i when `desc`.
__device__ __forceinline__ void ce_pairs(float& vi, int& xi, float& vl, int& xl, bool desc) {
  const bool lb = before_nb(vl, xl, vi, xi);
  const bool sw = desc ? lb : !lb;
  const float a = vi, b = vl;
  const int ia = xi, ib = xl;
  vi = sw ? b : a;
  vl = sw ? a : b;
  xi = sw ? ib : ia;
  xl = sw ? ia : ib;
}

// Bitonic sort of N (value, index) pairs into (value desc, index asc) order.
template <int N>
__device__ __forceinline__ void sort_desc_pairs(float (&v)[N], int (&ix)[N]) {
#pragma unroll
  for (int size = 2; size <= N; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1)
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int l = i ^ stride;
        if (l > i) ce_pairs(v[i], ix[i], v[l], ix[l], (i & size) == 0);
      }
}

// a := top N of (a, b), both sorted (value desc, index asc); result sorted.
template <int N>
__device__ __forceinline__ void merge_top_pairs(float (&a)[N], int (&ia)[N], const float (&b)[N],
                                                const int (&ib)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const bool take = before_nb(b[N - 1 - i], ib[N - 1 - i], a[i], ia[i]);
    a[i] = take ? b[N - 1 - i] : a[i];
    ia[i] = take ? ib[N - 1 - i] : ia[i];
  }
  // a is now bitonic: clean it into descending order
#pragma unroll
  for (int stride = N >> 1; stride > 0; stride >>= 1)
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const int l = i ^ stride;
      if (l > i) ce_pairs(a[i], ia[i], a[l], ia[l], true);
    }
}

// Exact top-16 of one 128-column half-chunk merged into the running list
// (clean selection, no query noise).  Returns false (warp-uniform) when a
// lane's candidates overflow the buffer or the 16th score is tied; the
// caller then takes the general path for this half-chunk.
//   A. 32 group maxima (groups of 4); their 16th largest g16 bounds the
//      half-chunk's 16th largest cosine from below (16 distinct values are
//      >= g16).  Two 16-sorts give g16 = min_i max(lo[i], hi[15 - i]).
//   B. scores >= score(g16) go to a per-thread shared-memory buffer (<= 32).
//   C. value-only top-16 of the buffer: t* = the 16th largest score.
//   D. second TMEM scan: (score, key) of the values >= t*, in key order;
//      exactly 16 unless t* is tied.  Sort them and merge into the list.
// buf: this thread's slot 0; slots are 256 floats apart (bank-conflict free).
// Predicated shared store (no branch).
__device__ __forceinline__ void st_shared_if(float* p, float v, bool pred) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.shared.f32 [%0], %1;\n\t}" ::"r"(
                   tc::smem_u32(p)),
               "f"(v), "r"((int)pred)
               : "memory");
}

template <bool QS>
__device__ __forceinline__ float score_of(uint32_t bits, float T, float ql) {
  float sc = __fmul_rn(__uint_as_float(bits), T);   // memory.py:150
  if (QS) sc = __fmul_rn(sc, ql);                   // memory.py:151-152
  return sc;
}

// 64 consecutive TMEM columns of this warp's lanes: two loads, one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&x)[64]) {
  tc::tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&x[0]));
  tc::tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&x[32]));
  tc::tmem_wait_ld();
}

template <bool QS>
__device__ __forceinline__ bool fast_top16(uint32_t taddr, int key0, float T, float ql, bool owner, bool first,
                                           float (&rv)[16], int (&ri)[16], float* buf) {
  // A. 16th largest of the 32 group maxima (groups of 4 cosines)
  float lo[16], hi[16];
#pragma unroll
  for (int part = 0; part < 2; ++part) {
    uint32_t x[64];
    tmem_ld64(taddr + part * 64, x);
#pragma unroll
    for (int g = 0; g < 16; ++g) {
      const float m4 = fmaxf(fmaxf(__uint_as_float(x[4 * g]), __uint_as_float(x[4 * g + 1])),
                             fmaxf(__uint_as_float(x[4 * g + 2]), __uint_as_float(x[4 * g + 3])));
      if (part == 0)
        lo[g] = m4;
      else
        hi[g] = m4;
    }
  }
  sort_desc_v<16>(lo);
  sort_desc_v<16>(hi);
  float g16 = INFINITY;
#pragma unroll
  for (int i = 0; i < 16; ++i) g16 = fminf(g16, fmaxf(lo[i], hi[15 - i]));
  float tau = score_of<QS>(__float_as_uint(g16), T, ql);
  if (!owner) tau = INFINITY;

  // B. candidate (score, key) pairs (score >= tau) into this thread's slots,
  // in key order.  Slot offsets come from per-8-value prefix counts, so the
  // running count is a chain of 16 additions, not 128.
  int cnt = 0;
#pragma unroll
  for (int part = 0; part < 2; ++part) {
    uint32_t x[64];
    tmem_ld64(taddr + part * 64, x);
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      float sc[8];
      int off[8], run = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sc[i] = score_of<QS>(x[8 * g + i], T, ql);
        off[i] = run;
        run += sc[i] >= tau;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int slot = (cnt + off[i]) & 31;
        st_shared_if(buf + slot * 256, sc[i], sc[i] >= tau);
        st_shared_if(buf + (32 + slot) * 256, __int_as_float(key0 + part * 64 + 8 * g + i), sc[i] >= tau);
      }
      cnt += run;
    }
  }
  if (__any_sync(FULL, cnt > 32)) return false;

  // C. value-only top-16 of the candidates: t* = their 16th largest
  float va[16], vb[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    va[i] = i < cnt ? buf[i * 256] : -INFINITY;
    vb[i] = 16 + i < cnt ? buf[(16 + i) * 256] : -INFINITY;
  }
  sort_desc_v<16>(va);
  sort_desc_v<16>(vb);
  float tstar = INFINITY;
#pragma unroll
  for (int i = 0; i < 16; ++i) tstar = fminf(tstar, fmaxf(va[i], vb[15 - i]));

  // D. the candidates >= t*, compacted in place (still in key order; 16
  // unless t* is tied)
  int cnt2 = 0;
  const float tst = owner ? tstar : INFINITY;
#pragma unroll 8
  for (int j = 0; j < 32; ++j) {
    const float v = buf[j * 256], kf = buf[(32 + j) * 256];
    const bool c = (j < cnt) && (v >= tst);
    st_shared_if(buf + (cnt2 & 15) * 256, v, c);
    st_shared_if(buf + (32 + (cnt2 & 15)) * 256, kf, c);
    cnt2 += c;
  }
  if (__any_sync(FULL, owner && cnt2 != 16)) return false;
  float pv[16];
  int pc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    pv[i] = owner ? buf[i * 256] : -INFINITY;
    pc[i] = owner ? __float_as_int(buf[(32 + i) * 256]) : (1 << 30) + i;
  }
  sort_desc_pairs<16>(pv, pc);
  if (first) {   // the row's list is still empty
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      rv[i] = pv[i];
      ri[i] = pc[i];
    }
  } else {
    merge_top_pairs<16>(rv, ri, pv, pc);
  }
  return true;
}

// Insertion of (s, i) at its (value desc, index asc) rank, for any index.
// Precondition: (s, i) ranks before the list's last element.
template <int KM>
__device__ __forceinline__ void list_insert_any(float (&v)[KM], int (&ix)[KM], float s, int i) {
#pragma unroll
  for (int j = KM - 1; j >= 0; --j) {
    const bool before_j = ranks_before(v[j], ix[j], s, i);
    const bool before_prev = j == 0 || ranks_before(v[j - 1], ix[j - 1], s, i);
    if (!before_prev) {
      v[j] = v[j - 1];
      ix[j] = ix[j - 1];
    } else if (!before_j) {
      v[j] = s;
      ix[j] = i;
    }
  }
}

template <int KM>
__device__ __forceinline__ void list_insert_any3(float (&v)[KM], int (&ix)[KM], float (&a)[KM], float s, int i,
                                                 float x) {
#pragma unroll
  for (int j = KM - 1; j >= 0; --j) {
    const bool before_j = ranks_before(v[j], ix[j], s, i);
    const bool before_prev = j == 0 || ranks_before(v[j - 1], ix[j - 1], s, i);
    if (!before_prev) {
      v[j] = v[j - 1];
      ix[j] = ix[j - 1];
      a[j] = a[j - 1];
    } else if (!before_j) {
      v[j] = s;
      ix[j] = i;
      a[j] = x;
    }
  }
}

// Per-thread state of one (token, head, half) row, over this warp's columns.
template <int KM, bool NOISY, bool BAL>
struct RowState {
  static constexpr bool CLEAN = NOISY && BAL;   // separate clean top-k for the balance counts
  float v[KM], sc[NOISY ? KM : 1], cv[CLEAN ? KM : 1];
  int ix[KM], cix[CLEAN ? KM : 1];
  float rmax, rsum;

  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int j = 0; j < KM; ++j) {
      v[j] = -INFINITY;
      ix[j] = 0;
      if constexpr (NOISY) sc[j] = -INFINITY;
      if constexpr (CLEAN) {
        cv[j] = -INFINITY;
        cix[j] = 0;
      }
    }
    rmax = -INFINITY;
    rsum = 0.f;
  }
};

template <int KM, bool NOISY, bool BAL, bool QS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    score_topk_tc_kernel(const __grid_constant__ CUtensorMap tA_hi, const __grid_constant__ CUtensorMap tA_lo,
                         const __grid_constant__ CUtensorMap tB_hi, const __grid_constant__ CUtensorMap tB_lo,
                         Dims D, TcShape S, const float* __restrict__ qlen, const float* __restrict__ gumbel,
                         const float* __restrict__ scal, int* __restrict__ sub_idx, float* __restrict__ sub_score,
                         float* __restrict__ sub_sel, int* __restrict__ clean_idx, float* __restrict__ row_max,
                         float* __restrict__ row_sum, int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  tc::PipeCtl* ctl = reinterpret_cast<tc::PipeCtl*>(smem);
  uint8_t* tiles = smem + 1024;
  volatile int* abort = &ctl->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = S.m_tiles * D.H * 2;
  const tc::PipeShape& P = S.P;
  // unit u = (codebook hc, 128-token tile mt): A rows of q in [hc][M][half],
  // B rows of the codebook's keys in [hc][n][half]
  auto coords = [&](int u, int& arow, int& brow0, int& nch) {
    const int hc = u / S.m_tiles, mt = S.mt0 + u - hc * S.m_tiles;
    arow = (int)(hc * D.M + (int64_t)mt * TC_M);
    brow0 = hc * D.n;
    nch = S.n_chunks;
  };
  const uint32_t tmem_base = tc::pipe_init(ctl, P, EPI_WARPS);

  if (warp == 0) {
    if (lane == 0) tc::pipe_produce(ctl, P, tiles, units, &tA_hi, &tA_lo, &tB_hi, &tB_lo, coords, err);
  } else if (warp == 1) {
    if (lane == 0) tc::pipe_mma(ctl, P, tiles, units, tmem_base, coords, err);
  } else {
    // ---------------- epilogue: per-row top-k ----------------
    using RS = RowState<KM, NOISY, BAL>;
    constexpr bool FAST16 = KM == 16 && !NOISY && !BAL;
    float* fbuf = reinterpret_cast<float*>(smem + S.merge_off) + (threadIdx.x - 64);
    // full half-chunk width and the prefilter's group size (>= k groups)
    constexpr int HALF_BN_FULL = (KM >= 32 ? 128 : 256) / 2;
    constexpr int GS = HALF_BN_FULL / KM;
    const int quarter = warp & 3;            // TMEM lane quarter this warp may read
    const int hf = (warp - 2) >> 2;          // column half of every chunk
    const int r_in_tile = quarter * 32 + lane;
    const int half_bn = P.BN >> 1;
    const float T = scal[0];
    // merge buffer: [128 rows][KM] values, indices (+ clean-score copies)
    float* mv = reinterpret_cast<float*>(smem + S.merge_off);
    int* mi = reinterpret_cast<int*>(mv + TC_M * KM);
    float* mx = reinterpret_cast<float*>(mi + TC_M * KM);   // NOISY: sc; later the clean list
    float* mrow = mx + (NOISY ? TC_M * KM : 0);             // BAL: rmax, rsum per row
    RS R;
    int acc = 0;
    uint32_t aph = 0, pph = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      const int hc = u / S.m_tiles, mt = S.mt0 + u - hc * S.m_tiles;
      const int h = hc >> 1, c = hc & 1;
      const int64_t m = (int64_t)mt * TC_M + r_in_tile;
      const bool owner = m < D.M;
      const int64_t row = (m * D.H + h) * 2 + c;
      const float ql = (QS && owner) ? qlen[row] : 1.f;
      const float* grow = (NOISY && owner) ? gumbel + row * D.n : nullptr;
      R.reset();
      for (int j = 0; j < S.n_chunks; ++j) {
        // warp-uniform outcome, so every lane leaves together on a timeout
        if (!__all_sync(FULL, tc::mbar_wait(&ctl->tfull[acc], aph, abort, err, 14))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const int key0 = j * P.BN;
        const int valid = min(P.BN, D.n - key0);
        const int cb = hf * half_bn, ce = min(cb + half_bn, valid);
        const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * ACC_STRIDE);

        // exact per-half-chunk top-16 (clean selection), else the general path
        bool fast_done = false;
        if constexpr (FAST16) {
          if (ce - cb == HALF_BN_FULL)
            fast_done = fast_top16<QS>(taddr + cb, key0 + cb, T, ql, owner, j == 0, R.v, R.ix, fbuf);
        }
        if (!fast_done) {
        // pass A: a lower bound of this half-chunk's k-th best selection
        // score: min over the maxima of HALF_BN_FULL / KM disjoint groups
        // (at least k groups).  Computed on raw cosines: the scaling
        // s = (cos * T) [* q_len] is monotone, so it commutes with max / min.
        float thr_base = -INFINITY;
        if constexpr (!NOISY) {
          if (ce - cb == HALF_BN_FULL) {
            float gmin = INFINITY, carry = -INFINITY;
            for (int cc = cb; cc < ce; cc += 16) {
              uint32_t r[16];
              tc::tmem_ld16(taddr + cc, r);
              tc::tmem_wait_ld();
              if constexpr (GS >= 16) {
#pragma unroll
                for (int t = 0; t < 16; ++t) carry = fmaxf(carry, __uint_as_float(r[t]));
                if (((cc - cb + 16) % GS) == 0) {
                  gmin = fminf(gmin, carry);
                  carry = -INFINITY;
                }
              } else {
#pragma unroll
                for (int g = 0; g < 16 / GS; ++g) {
                  float gm = __uint_as_float(r[g * GS]);
#pragma unroll
                  for (int t = 1; t < GS; ++t) gm = fmaxf(gm, __uint_as_float(r[g * GS + t]));
                  gmin = fminf(gmin, gm);
                }
              }
            }
            float tau = __fmul_rn(gmin, T);
            if constexpr (QS) tau = __fmul_rn(tau, ql);
            thr_base = tau;
          }
        }
        if (!owner) thr_base = INFINITY;

        // pass B: candidates beating max(tau, list k-th), inserted in lockstep
        for (int cc = cb; cc < ce; cc += 16) {
          uint32_t r[16];
          tc::tmem_ld16(taddr + cc, r);
          tc::tmem_wait_ld();
          const int nv = min(16, ce - cc);
          float sel[16], scr[NOISY ? 16 : 1];
          uint32_t mask = 0, cmask = 0;
          // s > v[KM-1] and s >= tau  <=>  s >= max(tau, succ(v[KM-1]))
          const float thr = fmaxf(thr_base, succ_f32(R.v[KM - 1]));
          const float cthr = RS::CLEAN ? (owner ? succ_f32(R.cv[KM - 1]) : INFINITY) : 0.f;
          // this row's 16 Gumbel values: four streaming 16-byte loads (read once)
          float gv[NOISY ? 16 : 1];
          if constexpr (NOISY) {
            const float* gp = owner ? grow + key0 + cc : nullptr;
            if (owner && nv == 16 && (reinterpret_cast<uintptr_t>(gp) & 15) == 0) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float4 v4 = __ldcs(reinterpret_cast<const float4*>(gp) + q);
                gv[4 * q] = v4.x;
                gv[4 * q + 1] = v4.y;
                gv[4 * q + 2] = v4.z;
                gv[4 * q + 3] = v4.w;
              }
            } else {
#pragma unroll
              for (int t = 0; t < 16; ++t) gv[t] = (owner && t < nv) ? gp[t] : 0.f;
            }
          }
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const float cosv = __uint_as_float(r[t]);
            float score = __fmul_rn(cosv, T);                          // memory.py:150
            if constexpr (QS) score = __fmul_rn(score, ql);            // memory.py:151-152
            float s_sel = score;
            if constexpr (NOISY) {
              s_sel = __fadd_rn(score, __fmul_rn(D.noise_coef, gv[t]));   // memory.py:158
              scr[t] = score;
            }
            sel[t] = s_sel;
            if (s_sel >= thr) mask |= 1u << t;
            if constexpr (RS::CLEAN) {
              if (score >= cthr) cmask |= 1u << t;
            }
            if constexpr (BAL) {
              if (owner && t < nv) {
                const float p = D.btgrad ? score : __fmul_rn(cosv, T);  // memory.py:211
                if (p > R.rmax) {
                  R.rsum = R.rsum * expf(R.rmax - p) + 1.f;
                  R.rmax = p;
                } else {
                  R.rsum += expf(p - R.rmax);
                }
              }
            }
          }
          if (nv < 16) {
            mask &= (1u << nv) - 1u;
            cmask &= (1u << nv) - 1u;
          }
          while (__any_sync(FULL, mask != 0)) {
            if (mask) {
              const uint32_t low = mask & (0u - mask);
              mask ^= low;
              const int t = low_bit_index16(low);
              const float s = pick16(sel, t);
              if (s > R.v[KM - 1]) {
                if constexpr (NOISY)
                  list_insert3<KM>(R.v, R.ix, R.sc, s, key0 + cc + t, pick16(scr, t));
                else
                  list_insert<KM>(R.v, R.ix, s, key0 + cc + t);
              }
            }
          }
          if constexpr (RS::CLEAN) {
            while (__any_sync(FULL, cmask != 0)) {
              if (cmask) {
                const uint32_t low = cmask & (0u - cmask);
                cmask ^= low;
                const int t = low_bit_index16(low);
                const float s = pick16(scr, t);
                if (s > R.cv[KM - 1]) list_insert<KM>(R.cv, R.cix, s, key0 + cc + t);
              }
            }
          }
        }
        }  // general path
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&ctl->tempty[acc]);
        acc ^= 1;
        if (acc == 0) aph ^= 1;
      }
      if (!ok) break;

      // ---- merge the two column halves of each row (warp pair of a quarter)
      uint64_t* pb = &ctl->pair[quarter];
      if constexpr (FAST16) {
        // through the thread pair's own candidate slots (warp w + 4 is the
        // partner of warp w): no other thread touches them
        if (hf == 1) {
#pragma unroll
          for (int j = 0; j < KM; ++j) {
            fbuf[j * 256] = R.v[j];
            fbuf[(KM + j) * 256] = __int_as_float(R.ix[j]);
          }
        }
        if (!tc::pair_sync(pb, pph, lane, abort, err)) break;
        if (hf == 0 && owner) {
          float ov[KM];
          int oi[KM];
#pragma unroll
          for (int j = 0; j < KM; ++j) {
            ov[j] = fbuf[128 + j * 256];
            oi[j] = __float_as_int(fbuf[128 + (KM + j) * 256]);
          }
          merge_top_pairs<KM>(R.v, R.ix, ov, oi);
        }
      } else {
      if (hf == 1) {
#pragma unroll
        for (int j = 0; j < KM; ++j) {
          mv[r_in_tile * KM + j] = R.v[j];
          mi[r_in_tile * KM + j] = R.ix[j];
          if constexpr (NOISY) mx[r_in_tile * KM + j] = R.sc[j];
        }
        if constexpr (BAL) {
          mrow[2 * r_in_tile] = R.rmax;
          mrow[2 * r_in_tile + 1] = R.rsum;
        }
      }
      if (!tc::pair_sync(pb, pph, lane, abort, err)) break;
      if (hf == 0) {
        bool done = !owner;
        for (int j = 0; __any_sync(FULL, !done) && j < KM; ++j) {
          if (!done) {
            const float s = mv[r_in_tile * KM + j];
            const int i = mi[r_in_tile * KM + j];
            if (ranks_before(s, i, R.v[KM - 1], R.ix[KM - 1])) {
              if constexpr (NOISY)
                list_insert_any3<KM>(R.v, R.ix, R.sc, s, i, mx[r_in_tile * KM + j]);
              else
                list_insert_any<KM>(R.v, R.ix, s, i);
            } else {
              done = true;  // the other list is sorted: nothing further can enter
            }
          }
        }
        if constexpr (BAL) {
          const float m2 = mrow[2 * r_in_tile], s2 = mrow[2 * r_in_tile + 1];
          const float mm = fmaxf(R.rmax, m2);
          R.rsum = (R.rsum > 0.f ? R.rsum * expf(R.rmax - mm) : 0.f) + (s2 > 0.f ? s2 * expf(m2 - mm) : 0.f);
          R.rmax = mm;
        }
      }
      if constexpr (RS::CLEAN) {
        if (!tc::pair_sync(pb, pph, lane, abort, err)) break;
        if (hf == 1) {
#pragma unroll
          for (int j = 0; j < KM; ++j) {
            mv[r_in_tile * KM + j] = R.cv[j];
            mi[r_in_tile * KM + j] = R.cix[j];
          }
        }
        if (!tc::pair_sync(pb, pph, lane, abort, err)) break;
        if (hf == 0) {
          bool done = !owner;
          for (int j = 0; __any_sync(FULL, !done) && j < KM; ++j) {
            if (!done) {
              const float s = mv[r_in_tile * KM + j];
              const int i = mi[r_in_tile * KM + j];
              if (ranks_before(s, i, R.cv[KM - 1], R.cix[KM - 1]))
                list_insert_any<KM>(R.cv, R.cix, s, i);
              else
                done = true;
            }
          }
        }
      }
      }  // general merge
      if (hf == 0 && owner) {
        const int64_t o = row * D.k;
        if (D.k == KM && KM % 4 == 0) {
          // whole list: 16-byte stores (rows are k * 4 bytes apart)
#pragma unroll
          for (int j = 0; j < KM; j += 4) {
            *reinterpret_cast<int4*>(sub_idx + o + j) = make_int4(R.ix[j], R.ix[j + 1], R.ix[j + 2], R.ix[j + 3]);
            *reinterpret_cast<float4*>(sub_sel + o + j) = make_float4(R.v[j], R.v[j + 1], R.v[j + 2], R.v[j + 3]);
            if constexpr (NOISY)
              *reinterpret_cast<float4*>(sub_score + o + j) = make_float4(R.sc[j], R.sc[j + 1], R.sc[j + 2], R.sc[j + 3]);
            if constexpr (RS::CLEAN)
              *reinterpret_cast<int4*>(clean_idx + o + j) = make_int4(R.cix[j], R.cix[j + 1], R.cix[j + 2], R.cix[j + 3]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < KM; ++j) {
            if (j < D.k) {
              sub_idx[o + j] = R.ix[j];
              sub_sel[o + j] = R.v[j];
              if constexpr (NOISY) sub_score[o + j] = R.sc[j];
              if constexpr (RS::CLEAN) clean_idx[o + j] = R.cix[j];
            }
          }
        }
        if constexpr (BAL) {
          row_max[row] = R.rmax;
          row_sum[row] = R.rsum;
        }
      }
      if (!tc::pair_sync(pb, pph, lane, abort, err)) break;   // the merge buffer is reused by the next unit
    }
  }

  tc::pipe_finish(ctl, tmem_base);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

inline int bn_for(const Dims& D) {
  // k = 32 lists need a 48 KB merge buffer: use 128-key chunks to make room
  const int cap = D.kmax >= 32 ? 128 : 256;
  return D.n >= cap ? cap : ((D.n + 15) / 16) * 16;
}

// The exact top-16 fast path runs for clean k <= 16 selections without
// balance statistics.
inline bool fast_path(const Dims& D, bool bal) { return D.kmax == 16 && !D.noisy && !bal; }

// Epilogue shared memory: the row-merge buffer, aliased with the 32-slot
// per-thread (score, key) candidate buffer of the fast path.
inline uint32_t merge_bytes(const Dims& D, bool bal) {
  const uint32_t per = 8u + (D.noisy ? 4u : 0u);
  const uint32_t merge = TC_M * D.kmax * per + TC_M * 8u;
  const uint32_t fast = fast_path(D, bal) ? 64u * 4u * (TC_THREADS - 64) : 0u;
  return merge > fast ? merge : fast;
}

// 16-element K stages (64-byte swizzle): three 48 KB stages leave room for
// the fast path's 64 KB candidate buffer.
constexpr int SCORE_BK = 16;

TcShape tc_shape(const Dims& D, bool bal) {
  TcShape S;
  S.P = tc::pipe_shape(bn_for(D), D.half, merge_bytes(D, bal), SCORE_BK);
  S.m_tiles = (int)((D.M + TC_M - 1) / TC_M);
  S.mt0 = 0;
  S.n_chunks = (D.n + S.P.BN - 1) / S.P.BN;
  S.merge_off = 1024 + S.P.stages * S.P.stage_bytes;
  return S;
}

template <int KM, bool NOISY, bool BAL, bool QS>
cudaError_t launch_tc_t(const Dims& D, const Work& W, const float* gumbel, cudaStream_t s, int mt0, int mtn,
                        int max_ctas) {
  TcShape S = tc_shape(D, BAL);
  if (mtn > 0) {   // a range of 128-token tiles
    S.mt0 = mt0;
    S.m_tiles = mtn;
  }
  if (S.P.stages < 2) return cudaErrorInvalidConfiguration;
  CUtensorMap m[4];
  cudaError_t e;
  const uint64_t arows = (uint64_t)D.M * D.H * 2, brows = (uint64_t)D.n * D.H * 2;
  if ((e = make_tmap_f32(&m[0], W.q_hi, arows, D.half, TC_M, SCORE_BK)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[1], W.q_lo, arows, D.half, TC_M, SCORE_BK)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[2], W.k_hi, brows, D.half, S.P.BN, SCORE_BK)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[3], W.k_lo, brows, D.half, S.P.BN, SCORE_BK)) != cudaSuccess) return e;
  const size_t smem = 1024 + (size_t)S.merge_off + merge_bytes(D, BAL);
  auto kern = score_topk_tc_kernel<KM, NOISY, BAL, QS>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
    return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (max_ctas > 0 && max_ctas < sms) sms = max_ctas;
  const int units = S.m_tiles * D.H * 2;
  const int grid = units < sms ? units : sms;
  kern<<<grid, TC_THREADS, smem, s>>>(m[0], m[1], m[2], m[3], D, S, W.qlen, gumbel, W.scal, W.sub_idx, W.sub_score,
                                      W.sub_sel, W.clean_idx, W.row_max, W.row_sum, W.err);
  count_launch();
  return cudaGetLastError();
}

template <int KM, bool QS>
cudaError_t launch_tc_q(const Dims& D, const Work& W, const float* gumbel, bool bal, cudaStream_t s, int mt0,
                        int mtn, int mc) {
  if (D.noisy)
    return bal ? launch_tc_t<KM, true, true, QS>(D, W, gumbel, s, mt0, mtn, mc)
               : launch_tc_t<KM, true, false, QS>(D, W, gumbel, s, mt0, mtn, mc);
  return bal ? launch_tc_t<KM, false, true, QS>(D, W, gumbel, s, mt0, mtn, mc)
             : launch_tc_t<KM, false, false, QS>(D, W, gumbel, s, mt0, mtn, mc);
}

template <int KM>
cudaError_t launch_tc_k(const Dims& D, const Work& W, const float* gumbel, bool bal, cudaStream_t s, int mt0,
                        int mtn, int mc) {
  return D.qscale ? launch_tc_q<KM, true>(D, W, gumbel, bal, s, mt0, mtn, mc)
                  : launch_tc_q<KM, false>(D, W, gumbel, bal, s, mt0, mtn, mc);
}

}  // namespace

cudaError_t make_tmap_f32(CUtensorMap* map, const float* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                          uint32_t box_k) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (box_k != 16 && box_k != 32) return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * sizeof(float)};
  cuuint32_t box[2] = {box_k, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, box_k == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_tmap_f32_2d(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer, uint64_t pitch,
                             uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch * sizeof(float)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

bool score_tc_supported(const Dims& D) {
  // the tensor maps' boxes (128 query rows, BN key rows) must fit inside the
  // [H*2*M, half] / [H*2*n, half] matrices
  const int BN = bn_for(D);
  return D.half % TC_K == 0 && D.half >= TC_K && D.M * D.H * 2 >= TC_M && (int64_t)D.n * D.H * 2 >= BN &&
         D.M * D.H * 2 < (1ll << 31);
}

cudaError_t launch_score_topk_tc(const Dims& D, const Work& W, const float* gumbel, bool want_balance,
                                 cudaStream_t s, int mt0, int mtn, int max_ctas) {
  switch (D.kmax) {
    case 4: return launch_tc_k<4>(D, W, gumbel, want_balance, s, mt0, mtn, max_ctas);
    case 8: return launch_tc_k<8>(D, W, gumbel, want_balance, s, mt0, mtn, max_ctas);
    case 16: return launch_tc_k<16>(D, W, gumbel, want_balance, s, mt0, mtn, max_ctas);
    case 32: return launch_tc_k<32>(D, W, gumbel, want_balance, s, mt0, mtn, max_ctas);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ml
