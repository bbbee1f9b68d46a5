// Backward of the balance term (memory.py:205-214 differentiated) on the
// tensor cores, with the cosines kept in TMEM.
//
// For one codebook hc the term needs, over every token row m and every key j,
//   cos[m, j] = q_hat[m] . k_hat[j]                      (3xTF32 MMA, K = half)
//   p = cos * ps,  s = softmax_j(p),  ps = T (or T q_len under
//   balance_temperature_grad),
//   d cos[m, j] = ps * s_j (cnt_j dscale - sum_i cnt_i dscale s_i) / M,
//   d q_hat[m] += sum_j d cos[m, j] k_hat[j]              (3xTF32 MMA, K = n)
//   d k_hat[j]  = sum_m d cos[m, j] q_hat[m]               (3xTF32 GEMM, K = M)
// (plus the row's temperature / q_len gradient under balance_temperature_grad).
//
// bal_bwd_tc_kernel, one persistent CTA per SM, one work unit per
// (codebook, 128-token tile):
//   warp 0   TMA producer: q_hat K stages and the sub-key chunks streamed
//            against each, then the transposed sub-keys, 32 keys per block,
//            of the d q_hat MMA (one six-block ring shared with the
//            epilogue's d cos blocks);
//   warp 1   MMA issuer: the 128 x n cosine tile into TMEM columns [0, n),
//            then d q_hat (128 x half) into columns [0, half) -- issued only
//            after the epilogue has read those cosine columns;
//   warps 2-9 epilogue, one TMEM lane (token row) per thread, two warps per
//            lane quarter taking alternate 32-key chunks: row max and sums
//            (combined across the pair), then per chunk d cos -> tf32 hi / lo, written
//            (a) into a shared-memory A-operand slot (128-byte swizzle,
//            K-major) for the d q_hat MMA and (b) as float32, transposed, to
//            global memory, 32 consecutive tokens per store, as the A operand
//            of the d k_hat GEMM; finally the tile's d q_hat is stored (the
//            query norm backward adds it to the routing share).
// The routing backward's sparse d cos entries are then added into the
// transposed d cos (sparse_into_dct_kernel) and the d k_hat GEMM -- one launch
// of the operand-splitting GEMM (gemm_raw_tc.cu), batched over the codebooks,
// reading the unit queries in place, K slices added in order -- gives the
// whole sub-key gradient, dense and sparse parts together.
// The [H*2, M, n] cosine / d cos matrices never reach HBM.
#include "bal_bwd_tc.cuh"
#include "backbone.cuh"
#include "gemm_any.cuh"
#include "tc_common.cuh"

namespace ml {

namespace {

constexpr int BB_EPI_WARPS = 8;                     // two per TMEM lane quarter
constexpr int BB_HALF_WARPS = BB_EPI_WARPS / 2;     // the warps of one chunk parity: one per quarter
constexpr int BB_THREADS = 64 + 32 * BB_EPI_WARPS;
constexpr uint32_t BB_TILE = 128 * 32 * 4;          // 128 rows x 32 tf32, 128-byte rows
constexpr uint32_t BB_BLOCK = 2 * BB_TILE;          // one ring block: a hi / lo pair of tiles
constexpr int BB_BLOCKS = 6;                        // ring depth (>= 1 + 128-key chunks)
constexpr uint32_t BB_XCH = 8192;                   // row-statistics exchange of the warp pairs
constexpr int BB_WCNT = 256;                        // counts per epilogue warp: its n / 2 <= 256 keys
constexpr uint32_t BB_CNTS = BB_EPI_WARPS * BB_WCNT * 4;
constexpr uint32_t BB_SMEM = 2048 + BB_BLOCKS * BB_BLOCK + BB_XCH + BB_CNTS;
constexpr float BB_LOG2E = 1.4426950408889634f;

// One ring of 32 KB blocks carries, per work unit and in this order,
//   for each K stage kc of the cosine MMA: Q(kc) = q_hat hi / lo [128 x 32],
//     then K(kc, jc) = sub-key hi / lo [128 keys x 32] for every key chunk jc
//     (Q(kc) stays resident while its key chunks stream past);
//   for each 32-key chunk c of the d q_hat MMA: KT(c) = transposed sub-keys
//     hi / lo [half x 32 keys], then D(c) = d cos hi / lo [128 x 32 keys],
//     which the epilogue writes instead of TMA.
// Producer, MMA issuer and epilogue walk the same block sequence, so a
// block's position fixes its slot (pos % BB_BLOCKS) and phase.  full[] is
// completed by 4 arrivals: the producer's expect_tx arrive plus 3 plain
// arrives for a TMA block, one per epilogue warp of the chunk's parity for a
// D block; empty[] by the MMA's commit.
// The two epilogue warps of a lane quarter (same 32 rows) take the even and
// the odd 32-key chunks and combine their row statistics through shared
// memory (pair[] barriers, two arrivals each).
struct BalCtl {
  uint64_t full[BB_BLOCKS], empty[BB_BLOCKS];
  uint64_t sfull, sread, dqfull, tempty, pair[4];
  uint32_t tmem_base;
  int abort;
};

struct BalArgs {
  int64_t M;
  int HC, n, half;
  int m_tiles;          // 128-token tiles
  int64_t Mp;           // row pitch of the transposed d cos (m_tiles * 128)
  float dscale;
  int btgrad, qscale;
  const float* cnt;     // [HC][n] clean top-k counts
  const float* qlen;    // [M][HC]
  const float* scal;    // [1] temperature
  float* dqbal;         // [M][HC][half] the balance term's d q_hat
  float* dT_row;        // [HC][M]
  float* dql_row;       // [M][HC] or nullptr
  float* dct;           // [HC][n][Mp] d cos, transposed
  int* err;
};

// 2^x (PTX ex2.approx.ftz.f32).  The softmax works in base 2: exp(p) =
// 2^(p log2 e), with log2 e folded into the row's score scale, so each
// exponential is one FFMA and one ex2.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Bounded rendezvous of the two warps of a lane quarter.
__device__ __forceinline__ bool pair_sync(uint64_t* bar, uint32_t& parity, int lane, volatile int* abort, int* err) {
  __syncwarp();
  if (lane == 0) tc::mbar_arrive(bar);
  const bool ok = tc::mbar_wait(bar, parity, abort, err, 19);
  parity ^= 1;
  return __all_sync(FULL, ok);
}

__device__ __forceinline__ void ring_at(uint32_t pos, int& s, uint32_t& ph) {
  s = (int)(pos % BB_BLOCKS);
  ph = (pos / BB_BLOCKS) & 1;
}

// 3xTF32 MMAs of one 32-deep K stage: d (+)= A_hi B_hi + A_hi B_lo + A_lo B_hi.
__device__ __forceinline__ void mma_stage(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
                                          uint32_t idesc, bool first) {
#pragma unroll
  for (int k8 = 0; k8 < 4; ++k8) {
    const uint32_t off = k8 * 32;
    const uint64_t dah = tc::sdesc_k_sw128(a_hi + off), dal = tc::sdesc_k_sw128(a_lo + off);
    const uint64_t dbh = tc::sdesc_k_sw128(b_hi + off), dbl = tc::sdesc_k_sw128(b_lo + off);
    tc::mma_tf32(d, dah, dbh, idesc, (first && k8 == 0) ? 0u : 1u);
    tc::mma_tf32(d, dah, dbl, idesc, 1);
    tc::mma_tf32(d, dal, dbh, idesc, 1);
  }
}

__global__ void __launch_bounds__(BB_THREADS, 1)
    bal_bwd_tc_kernel(const __grid_constant__ CUtensorMap tQ_hi, const __grid_constant__ CUtensorMap tQ_lo,
                      const __grid_constant__ CUtensorMap tK_hi, const __grid_constant__ CUtensorMap tK_lo,
                      const __grid_constant__ CUtensorMap tKT_hi, const __grid_constant__ CUtensorMap tKT_lo,
                      BalArgs A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BalCtl* ctl = reinterpret_cast<BalCtl*>(smem);
  uint8_t* ring = smem + 1024;
  // [2 parities][128 rows][8]: row statistics at 0-2, temperature / q_len gradient shares at 4-5
  float* xch = reinterpret_cast<float*>(ring + BB_BLOCKS * BB_BLOCK);
  // [8 epilogue warps][256]: the warp's counts (x dscale) of its chunks, 32 per chunk
  float* cnts = xch + BB_XCH / 4;
  volatile int* abort = &ctl->abort;
  int* err = A.err;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = A.HC * A.m_tiles;
  const int nb = A.n / 128;                // 128-key chunks of the cosine MMA
  const int kq = A.half / 32;              // K stages of the cosine MMA
  const int nch = A.n / 32;                // 32-key chunks of the d q_hat MMA
  const uint32_t per_unit = (uint32_t)(kq * (1 + nb) + 2 * nch);   // ring blocks per unit

  if (threadIdx.x == 0) {
    for (int s = 0; s < BB_BLOCKS; ++s) {
      tc::mbar_init(&ctl->full[s], BB_HALF_WARPS);
      tc::mbar_init(&ctl->empty[s], 1);
    }
    for (int q = 0; q < 4; ++q) tc::mbar_init(&ctl->pair[q], 2);
    tc::mbar_init(&ctl->sfull, 1);
    tc::mbar_init(&ctl->dqfull, 1);
    tc::mbar_init(&ctl->sread, BB_EPI_WARPS);
    tc::mbar_init(&ctl->tempty, BB_EPI_WARPS);
    ctl->abort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(&ctl->tmem_base, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = ctl->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tc::prefetch_tmap(&tQ_hi);
      tc::prefetch_tmap(&tQ_lo);
      tc::prefetch_tmap(&tK_hi);
      tc::prefetch_tmap(&tK_lo);
      tc::prefetch_tmap(&tKT_hi);
      tc::prefetch_tmap(&tKT_lo);
      uint32_t pos = 0;
      // claim the next block for a TMA load of `bytes`; nullptr on timeout
      auto claim = [&](uint32_t bytes, uint64_t*& bar) -> uint8_t* {
        int s;
        uint32_t ph;
        ring_at(pos++, s, ph);
        if (!tc::mbar_wait(&ctl->empty[s], ph ^ 1, abort, err, 17)) return nullptr;
        bar = &ctl->full[s];
        tc::mbar_expect_tx(bar, bytes);
        for (int i = 1; i < BB_HALF_WARPS; ++i) tc::mbar_arrive(bar);
        return ring + (size_t)s * BB_BLOCK;
      };
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int hc = u / A.m_tiles, mt = u - hc * A.m_tiles;
        const int qrow = (int)(hc * A.M + (int64_t)mt * 128);
        uint64_t* bar;
        for (int kc = 0; kc < kq; ++kc) {
          uint8_t* b = claim(2 * BB_TILE, bar);
          if (!b) return;
          tc::tma_load_2d(b, &tQ_hi, bar, kc * 32, qrow);
          tc::tma_load_2d(b + BB_TILE, &tQ_lo, bar, kc * 32, qrow);
          for (int jc = 0; jc < nb; ++jc) {
            if (!(b = claim(2 * BB_TILE, bar))) return;
            tc::tma_load_2d(b, &tK_hi, bar, kc * 32, hc * A.n + jc * 128);
            tc::tma_load_2d(b + BB_TILE, &tK_lo, bar, kc * 32, hc * A.n + jc * 128);
          }
        }
        for (int c = 0; c < nch; ++c) {
          uint8_t* b = claim(2 * (uint32_t)A.half * 128, bar);
          if (!b) return;
          tc::tma_load_2d(b, &tKT_hi, bar, c * 32, hc * A.half);
          tc::tma_load_2d(b + A.half * 128, &tKT_lo, bar, c * 32, hc * A.half);
          ++pos;   // D(c): written by the epilogue
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc1 = tc::idesc_tf32(128, 128), idesc2 = tc::idesc_tf32(128, A.half);
      uint32_t pos = 0, it = 0;
      // wait for the next block; its slot in s
      auto take = [&](int& s) -> bool {
        uint32_t ph;
        ring_at(pos++, s, ph);
        if (!tc::mbar_wait(&ctl->full[s], ph, abort, err, 18)) return false;
        tc::fence_after_sync();
        return true;
      };
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
        // TMEM free: the epilogue has finished the previous unit
        if (!tc::mbar_wait(&ctl->tempty, (it & 1) ^ 1, abort, err, 18)) return;
        tc::fence_after_sync();
        for (int kc = 0; kc < kq; ++kc) {
          int sa, sb;
          if (!take(sa)) return;
          const uint32_t a_hi = tc::smem_u32(ring + (size_t)sa * BB_BLOCK), a_lo = a_hi + BB_TILE;
          for (int jc = 0; jc < nb; ++jc) {
            if (!take(sb)) return;
            const uint32_t b_hi = tc::smem_u32(ring + (size_t)sb * BB_BLOCK), b_lo = b_hi + BB_TILE;
            mma_stage(tmem_base + (uint32_t)(jc * 128), a_hi, a_lo, b_hi, b_lo, idesc1, kc == 0);
            tc::mma_commit(&ctl->empty[sb]);
          }
          tc::mma_commit(&ctl->empty[sa]);
        }
        tc::mma_commit(&ctl->sfull);   // cosines complete
        for (int c = 0; c < nch; ++c) {
          int sk, sd;
          if (!take(sk) || !take(sd)) return;
          // d q_hat overwrites cosine columns [0, half): the epilogue has read them
          if (c == 0 && !tc::mbar_wait(&ctl->sread, it & 1, abort, err, 18)) return;
          tc::fence_after_sync();
          const uint32_t a_hi = tc::smem_u32(ring + (size_t)sd * BB_BLOCK), a_lo = a_hi + BB_TILE;
          const uint32_t b_hi = tc::smem_u32(ring + (size_t)sk * BB_BLOCK), b_lo = b_hi + A.half * 128;
          mma_stage(tmem_base, a_hi, a_lo, b_hi, b_lo, idesc2, c == 0);
          tc::mma_commit(&ctl->empty[sk]);
          tc::mma_commit(&ctl->empty[sd]);
        }
        tc::mma_commit(&ctl->dqfull);   // d q_hat complete
      }
    }
  } else {
    const int quarter = warp & 3;
    const int hf = (warp - 2) >> 2;                    // this warp's chunk parity
    const int r = quarter * 32 + lane;                 // TMEM lane = row of the tile
    const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const float T = A.scal[0];
    const float invM = 1.0f / (float)A.M;
    const int Q = A.half / 32;                         // cosine chunks under the d q_hat accumulator
    // the last chunk of this parity below Q (-1: none) -- after reading it the
    // warp tells the MMA issuer that d q_hat may overwrite those columns
    const int my_last = (Q - 1 - hf) >= 0 ? Q - 1 - ((Q - 1 - hf) & 1) : -1;
    uint64_t* pbar = &ctl->pair[quarter];
    uint32_t pph = 0;
    float* mine = xch + (hf * 128 + r) * 8;
    const float* other = xch + ((hf ^ 1) * 128 + r) * 8;
    float* cw = cnts + (warp - 2) * BB_WCNT;           // chunk hf + 2 i at cw + 32 i
    uint32_t it = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
      const int hc = u / A.m_tiles, mt = u - hc * A.m_tiles;
      const int64_t m = (int64_t)mt * 128 + r;
      const bool owner = m < A.M;
      const float ql = (A.qscale && owner) ? A.qlen[m * A.HC + hc] : 1.f;
      const float ps = A.btgrad ? T * ql : T;
      const float psl = ps * BB_LOG2E;                 // score scale in base 2 (ps > 0)
      const float* cn = A.cnt + (int64_t)hc * A.n;
      // this warp's counts into its shared-memory slice while the cosines are
      // computed (the warp's reads of the previous unit's counts are done)
      {
        float cr[BB_WCNT / 32];
#pragma unroll
        for (int i = 0; i < BB_WCNT / 32; ++i) cr[i] = hf + 2 * i < nch ? __ldg(cn + (hf + 2 * i) * 32 + lane) : 0.f;
        __syncwarp();
#pragma unroll
        for (int i = 0; i < BB_WCNT / 32; ++i)
          if (hf + 2 * i < nch) cw[i * 32 + lane] = cr[i] * A.dscale;
        __syncwarp();
      }
      if (!__all_sync(FULL, tc::mbar_wait(&ctl->sfull, it & 1, abort, err, 19))) break;
      tc::fence_after_sync();
      // one pass over this warp's chunks: running max, sum of exp and the
      // count-weighted sum (memory.py:210-214), in base 2; a chunk's counts
      // are 8 broadcast float4 loads; TMEM loads run one chunk ahead.
      float mx = -INFINITY, sum = 0.f, sdp = 0.f;
      auto stats = [&](const uint32_t (&v)[32], const float* cs) {
        float vmax = -INFINITY;
#pragma unroll
        for (int t = 0; t < 32; ++t) vmax = fmaxf(vmax, __uint_as_float(v[t]));
        const float nm = fmaxf(mx, vmax * psl);        // = max_t (v_t psl): psl > 0
        const float sc = ex2(mx - nm);                 // 0 on the first chunk
        sum *= sc;
        sdp *= sc;
        const float4* c4 = reinterpret_cast<const float4*>(cs);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 cq = c4[q];
          const float cv[4] = {cq.x, cq.y, cq.z, cq.w};
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const float e = ex2(fmaf(__uint_as_float(v[4 * q + e4]), psl, -nm));
            sum += e;
            sdp = fmaf(e, cv[e4], sdp);
          }
        }
        mx = nm;
      };
      uint32_t va[32], vb[32];
      // chunks hf, hf + 2, ...: nch / 2 of them, an even number (nch % 4 == 0);
      // chunk c's counts at cw + 32 (c >> 1)
      tc::tmem_ld32(taddr + hf * 32, va);
      for (int c = hf; c < nch; c += 4) {
        tc::tmem_wait_ld_regs(va);
        tc::tmem_ld32(taddr + (c + 2) * 32, vb);
        stats(va, cw + (c >> 1) * 32);
        tc::tmem_wait_ld_regs(vb);
        if (c + 4 < nch) tc::tmem_ld32(taddr + (c + 4) * 32, va);
        stats(vb, cw + ((c + 2) >> 1) * 32);
      }
      // combine the pair's statistics, the even chunks' first (both warps get the same values)
      mine[0] = mx;
      mine[1] = sum;
      mine[2] = sdp;
      if (!pair_sync(pbar, pph, lane, abort, err)) break;
      {
        const float m0 = hf ? other[0] : mx, s0 = hf ? other[1] : sum, d0 = hf ? other[2] : sdp;
        const float m1 = hf ? mx : other[0], s1 = hf ? sum : other[1], d1 = hf ? sdp : other[2];
        mx = fmaxf(m0, m1);
        const float e0 = ex2(m0 - mx), e1 = ex2(m1 - mx);
        sum = s0 * e0 + s1 * e1;
        sdp = d0 * e0 + d1 * e1;
      }
      sdp /= sum;                                      // sum_i dP_i s_i
      // d p_j = e_j / sum (dP_j - sdp) / M with e_j = exp(p_j - max); the row's
      // constant factors folded into one (zero for a padding row), times sg(T)
      // when d cos is T d p_j
      const float gsc = owner ? (A.btgrad ? 1.0f / sum * invM : 1.0f / sum * invM * T) : 0.f;
      const float Tq = T * ql;
      // this row's column of the transposed d cos
      float* gd = A.dct + ((int64_t)hc * A.n) * A.Mp + (int64_t)mt * 128 + r;
      float dTr = 0.f, dqr = 0.f;
      const uint32_t dpos0 = it * per_unit + (uint32_t)(kq * (1 + nb)) + 1;   // position of D(0)
      if (my_last < 0) {   // no chunk of this parity under the accumulator
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&ctl->sread);
      }
      // chunk c of d cos: into the ring block D(c) and, transposed, to global memory
      auto dcos = [&](int c, const uint32_t (&v)[32]) -> bool {
        float hi[32], lo[32];
        const float4* c4 = reinterpret_cast<const float4*>(cw + (c >> 1) * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 cq = c4[q];
          const float cv[4] = {cq.x, cq.y, cq.z, cq.w};
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const int t = 4 * q + e4;
            const float cosv = __uint_as_float(v[t]);
            const float e = ex2(fmaf(cosv, psl, -mx));
            const float g = e * (cv[e4] - sdp) * gsc;   // d p_j (T d p_j without btgrad)
            float dc = g;
            if (A.btgrad) {
              dTr += g * cosv * ql;
              dqr += g * cosv * T;
              dc = g * Tq;
            }
            // transposed d cos: key (c 32 + t)'s row, 32 consecutive tokens per warp store
            gd[(int64_t)(c * 32 + t) * A.Mp] = dc;
            hi[t] = tc::to_tf32_int(dc);
            lo[t] = tc::to_tf32_int(dc - hi[t]);
          }
        }
        if (c == my_last) {   // columns [0, half) read: the d q_hat MMA may overwrite them
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&ctl->sread);
        }
        int s;
        uint32_t ph;
        ring_at(dpos0 + 2 * (uint32_t)c, s, ph);
        if (!__all_sync(FULL, tc::mbar_wait(&ctl->empty[s], ph ^ 1, abort, err, 19))) return false;
        // K-major 128-byte-swizzled row r of the block: 16-byte chunk q at (q ^ (r & 7))
        uint8_t* rowp = ring + (size_t)s * BB_BLOCK + r * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int at = ((q ^ (r & 7)) << 4);
          *reinterpret_cast<float4*>(rowp + at) = make_float4(hi[4 * q], hi[4 * q + 1], hi[4 * q + 2], hi[4 * q + 3]);
          *reinterpret_cast<float4*>(rowp + BB_TILE + at) =
              make_float4(lo[4 * q], lo[4 * q + 1], lo[4 * q + 2], lo[4 * q + 3]);
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&ctl->full[s]);
        return true;
      };
      bool ok = true;
      tc::tmem_ld32(taddr + hf * 32, va);
      for (int c = hf; ok && c < nch; c += 4) {
        tc::tmem_wait_ld_regs(va);
        tc::tmem_ld32(taddr + (c + 2) * 32, vb);
        ok = dcos(c, va);
        tc::tmem_wait_ld_regs(vb);
        if (ok && c + 4 < nch) tc::tmem_ld32(taddr + (c + 4) * 32, va);
        ok = ok && dcos(c + 2, vb);
      }
      if (!ok) break;
      // the row's temperature / q_len gradient: the pair's two shares, even chunks first
      mine[4] = dTr;
      mine[5] = dqr;
      if (!pair_sync(pbar, pph, lane, abort, err)) break;
      if (hf == 0 && owner) {
        A.dT_row[(int64_t)hc * A.M + m] = dTr + other[4];
        if (A.dql_row) A.dql_row[m * A.HC + hc] = dqr + other[5];
      }
      if (!__all_sync(FULL, tc::mbar_wait(&ctl->dqfull, it & 1, abort, err, 19))) break;
      tc::fence_after_sync();
      // this codebook's share of d q_hat, stored (the query norm backward adds
      // it); the pair takes alternate 32-column pieces
      float* dq = A.dqbal + (m * A.HC + hc) * A.half;
      for (int c0 = hf * 32; c0 < A.half; c0 += 64) {
        uint32_t v[32];
        tc::tmem_ld32(taddr + c0, v);
        tc::tmem_wait_ld();
        if (owner) {
#pragma unroll
          for (int t = 0; t < 32; t += 4)
            *reinterpret_cast<float4*>(dq + c0 + t) = make_float4(__uint_as_float(v[t]), __uint_as_float(v[t + 1]),
                                                                  __uint_as_float(v[t + 2]), __uint_as_float(v[t + 3]));
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ctl->tempty);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, 512);
  }
}

// The routing backward's sparse slot-score gradient (memory.py:162-178: one
// d cos per distinct selected sub-key of a (token, codebook) row) added into
// the transposed d cos matrix, so that one GEMM gives the whole sub-key
// gradient.  One thread per entry; a row's entries have distinct keys and
// rows own distinct columns, so no two threads touch one element.
__global__ void sparse_into_dct_kernel(const int* __restrict__ ent_slot, const float* __restrict__ ent_w, int64_t F,
                                       int k, int HC, int64_t Mp, float* __restrict__ dct) {
  const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= F) return;
  const float w = ent_w[f];
  if (w == 0.f) return;                       // padding (its key repeats the codebook's first)
  const int64_t m = f / ((int64_t)k * HC);    // entries are [M][HC][k]
  float* p = dct + (int64_t)ent_slot[f] * Mp + m;
  *p += w;
}

}  // namespace

bool bal_bwd_tc_supported(const Dims& D) {
  return D.n % 128 == 0 && D.n <= 512 && (D.half == 32 || D.half == 64 || D.half == 128) && D.M >= 128 &&
         (int64_t)D.H * 2 * D.M < (1ll << 31);
}

BalBwdPlan bal_bwd_plan(const Dims& D, int sms) {
  BalBwdPlan P{};
  const int64_t HC = D.H * 2, n = D.n, half = D.half;
  P.m_tiles = (int)((D.M + 127) / 128);
  P.Mp = (int64_t)P.m_tiles * 128;
  // K slices of the d k_hat GEMM (K = tokens)
  int64_t S, per;
  raw_slices(HC * (n / 128), (D.M + 31) / 32, HC * n * half, sms, (size_t)1 << 40, &S, &per);
  P.S = (int)S;
  P.kq_slice = (int)per;
  P.q_floats = HC * D.M * half;
  P.k_floats = HC * n * half;
  P.dct_floats = HC * n * P.Mp;
  P.part_floats = P.S > 1 ? (int64_t)P.S * HC * n * half : 0;
  return P;
}

cudaError_t launch_bal_bwd_tc(const Dims& D, const BalBwdPlan& P, const BalBwdBufs& B, float coef, cudaStream_t s) {
  if (D.M == 0) return cudaSuccess;
  const int HC = D.H * 2, n = D.n, half = D.half;
  cudaError_t e;
  // transposed unit sub-keys [hc][half][n] (B operand of the d q_hat MMA)
  if ((e = launch_gather_split(B.keys_n, half, n, 1, half, n, 1, half, B.kt_hi, B.kt_lo, HC, (int64_t)n * half,
                               (int64_t)half * n, s)) != cudaSuccess)
    return e;
  CUtensorMap m[6];
  if ((e = make_tmap_f32(&m[0], B.q_hi, (uint64_t)HC * D.M, half, 128)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[1], B.q_lo, (uint64_t)HC * D.M, half, 128)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[2], B.k_hi, (uint64_t)HC * n, half, 128)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[3], B.k_lo, (uint64_t)HC * n, half, 128)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[4], B.kt_hi, (uint64_t)HC * half, n, half)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[5], B.kt_lo, (uint64_t)HC * half, n, half)) != cudaSuccess) return e;
  BalArgs A{};
  A.M = D.M;
  A.HC = HC;
  A.n = n;
  A.half = half;
  A.m_tiles = P.m_tiles;
  A.Mp = P.Mp;
  A.dscale = coef * (float)n / (float)HC / (float)(D.M * D.k);   // dP = coef n / (2H) f, f = cnt / (M k)
  A.btgrad = D.btgrad;
  A.qscale = D.qscale;
  A.cnt = B.cnt;
  A.qlen = B.qlen;
  A.scal = B.scal;
  A.dqbal = B.dqbal;
  A.dT_row = B.dT_row;
  A.dql_row = B.dql_row;
  A.dct = B.dct;
  A.err = B.err;
  if ((e = cudaFuncSetAttribute(bal_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BB_SMEM)) !=
      cudaSuccess)
    return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int units = HC * P.m_tiles;
  bal_bwd_tc_kernel<<<units < sms ? units : sms, BB_THREADS, BB_SMEM, s>>>(m[0], m[1], m[2], m[3], m[4], m[5], A);
  count_launch();
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // + the routing backward's sparse entries
  {
    const int64_t F = D.M * HC * D.k;
    sparse_into_dct_kernel<<<(unsigned)((F + 255) / 256), 256, 0, s>>>(B.ent_slot, B.ent_w, F, D.k, HC, P.Mp, B.dct);
    count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  // d k_hat[hc] = d cos[hc]^T Q_hat[hc] (K = tokens), one batch per codebook
  const int64_t ldq = (int64_t)HC * half;
  if (!gemm_raw_supported(B.dct, P.Mp, 1, B.qn, ldq, 1, n, half, D.M)) return cudaErrorInvalidValue;
  if (P.S == 1)
    return launch_gemm_raw(B.dct, P.Mp, 1, B.qn, ldq, 1, n, half, D.M, 1, P.kq_slice, B.dkhat, 0, half, nullptr,
                           false, B.err, s, HC, (int64_t)HC * n, ldq, (int64_t)n * half);
  if ((e = launch_gemm_raw(B.dct, P.Mp, 1, B.qn, ldq, 1, n, half, D.M, P.S, P.kq_slice, B.part,
                           (int64_t)HC * n * half, half, nullptr, false, B.err, s, HC, (int64_t)HC * n, ldq,
                           (int64_t)n * half)) != cudaSuccess)
    return e;
  return launch_sum_slices(B.part, P.S, (int64_t)HC * n, half, B.dkhat, half, false, s);
}

}  // namespace ml
