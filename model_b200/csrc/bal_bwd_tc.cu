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
//   warp 0   TMA producer: q_hat tile x sub-key chunk operands of the cosine
//            MMA, then the transposed sub-keys, 32 keys per stage, of the
//            d q_hat MMA (a two-stage ring);
//   warp 1   MMA issuer: the 128 x n cosine tile into TMEM columns [0, n),
//            then d q_hat (128 x half) into columns [0, half) -- issued only
//            after the epilogue has read those cosine columns;
//   warps 2-5 epilogue, one TMEM lane (token row) per thread: row max, then
//            the sums, then per 32-key chunk d cos -> tf32 hi / lo, written
//            (a) into a shared-memory A-operand slot (128-byte swizzle,
//            K-major) for the d q_hat MMA and (b) transposed to global
//            memory, 32 consecutive tokens per store, as the A operand of the
//            d k_hat GEMM; finally d q_hat is added into the caller's
//            gradient.
// The d k_hat GEMM is one launch of the sliced 3xTF32 GEMM (gemm_tc.cu) over
// (token slice, codebook) pairs; the slices are added in order.
// The [H*2, M, n] cosine / d cos matrices never reach HBM.
#include "bal_bwd_tc.cuh"
#include "backbone.cuh"
#include "gemm_any.cuh"
#include "tc_common.cuh"

namespace ml {

namespace {

constexpr int BB_EPI_WARPS = 4;
constexpr int BB_THREADS = 64 + 32 * BB_EPI_WARPS;
constexpr int BB_RING = 2;                          // TMA ring stages
constexpr int BB_ASLOTS = 3;                        // d cos operand slots (>= half / 32 - 1)
constexpr uint32_t BB_TILE = 128 * 32 * 4;          // 128 rows x 32 tf32, 128-byte rows
constexpr uint32_t BB_STAGE = 4 * BB_TILE;          // A hi / lo + B hi / lo (B rows <= 128)
constexpr uint32_t BB_ASLOT = 2 * BB_TILE;          // d cos hi / lo
constexpr uint32_t BB_SMEM = 2048 + BB_RING * BB_STAGE + BB_ASLOTS * BB_ASLOT;

struct BalCtl {
  uint64_t full[BB_RING], empty[BB_RING];
  uint64_t afull[BB_ASLOTS], aempty[BB_ASLOTS];
  uint64_t sfull, sread, dqfull, tempty;
  uint32_t tmem_base;
  int abort;
};

struct BalArgs {
  int64_t M;
  int HC, n, half;
  int m_tiles;          // tiles per codebook, padded to whole token slices
  int Ks;               // tokens per slice of the transposed d cos (multiple of 128)
  float dscale;
  int btgrad, qscale;
  const float* cnt;     // [HC][n] clean top-k counts
  const float* qlen;    // [M][HC]
  const float* scal;    // [1] temperature
  float* dqhat;         // [M][HC][half], accumulated
  float* dT_row;        // [HC][M]
  float* dql_row;       // [M][HC] or nullptr
  float* dct_hi;        // [S][HC][n][Ks]
  float* dct_lo;
  int* err;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
  uint8_t* aslots = ring + BB_RING * BB_STAGE;
  volatile int* abort = &ctl->abort;
  int* err = A.err;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = A.HC * A.m_tiles;
  const int BN1 = A.n < 128 ? A.n : 128;   // keys per cosine MMA
  const int kq = A.half / 32;              // K stages of the cosine MMA
  const int nch = A.n / 32;                // 32-key chunks

  if (threadIdx.x == 0) {
    for (int s = 0; s < BB_RING; ++s) {
      tc::mbar_init(&ctl->full[s], 1);
      tc::mbar_init(&ctl->empty[s], 1);
    }
    for (int s = 0; s < BB_ASLOTS; ++s) {
      tc::mbar_init(&ctl->afull[s], BB_EPI_WARPS);
      tc::mbar_init(&ctl->aempty[s], 1);
    }
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
      int s = 0;
      uint32_t ph = 0;
      auto next = [&]() {
        if (++s == BB_RING) {
          s = 0;
          ph ^= 1;
        }
      };
      const int tiles = (int)((A.M + 127) / 128);
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int hc = u / A.m_tiles, mt = u - hc * A.m_tiles;
        // a padding tile (whole slices of the transposed d cos) reads real rows; its output is masked
        const int qrow = (int)(hc * A.M + (int64_t)(mt < tiles ? mt : 0) * 128);
        // cosine MMA operands: q_hat rows (codebook-major) and sub-key rows
        for (int jc = 0; jc < A.n / BN1; ++jc)
          for (int kc = 0; kc < kq; ++kc) {
            if (!tc::mbar_wait(&ctl->empty[s], ph ^ 1, abort, err, 17)) return;
            uint8_t* st = ring + (size_t)s * BB_STAGE;
            tc::mbar_expect_tx(&ctl->full[s], 2 * BB_TILE + 2 * (uint32_t)BN1 * 128);
            tc::tma_load_2d(st, &tQ_hi, &ctl->full[s], kc * 32, qrow);
            tc::tma_load_2d(st + BB_TILE, &tQ_lo, &ctl->full[s], kc * 32, qrow);
            tc::tma_load_2d(st + 2 * BB_TILE, &tK_hi, &ctl->full[s], kc * 32, hc * A.n + jc * BN1);
            tc::tma_load_2d(st + 2 * BB_TILE + BN1 * 128, &tK_lo, &ctl->full[s], kc * 32, hc * A.n + jc * BN1);
            next();
          }
        // d q_hat MMA operand: transposed sub-keys [half rows x 32 keys]
        for (int c = 0; c < nch; ++c) {
          if (!tc::mbar_wait(&ctl->empty[s], ph ^ 1, abort, err, 17)) return;
          uint8_t* st = ring + (size_t)s * BB_STAGE;
          tc::mbar_expect_tx(&ctl->full[s], 2 * (uint32_t)A.half * 128);
          tc::tma_load_2d(st, &tKT_hi, &ctl->full[s], c * 32, hc * A.half);
          tc::tma_load_2d(st + A.half * 128, &tKT_lo, &ctl->full[s], c * 32, hc * A.half);
          next();
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc1 = tc::idesc_tf32(128, BN1), idesc2 = tc::idesc_tf32(128, A.half);
      int s = 0, cg = 0;
      uint32_t ph = 0, it = 0;
      auto next = [&]() {
        if (++s == BB_RING) {
          s = 0;
          ph ^= 1;
        }
      };
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
        // TMEM free: the epilogue has finished the previous unit
        if (!tc::mbar_wait(&ctl->tempty, (it & 1) ^ 1, abort, err, 18)) return;
        tc::fence_after_sync();
        for (int jc = 0; jc < A.n / BN1; ++jc) {
          const uint32_t d = tmem_base + (uint32_t)(jc * BN1);
          for (int kc = 0; kc < kq; ++kc) {
            if (!tc::mbar_wait(&ctl->full[s], ph, abort, err, 18)) return;
            tc::fence_after_sync();
            const uint32_t a_hi = tc::smem_u32(ring + (size_t)s * BB_STAGE);
            const uint32_t a_lo = a_hi + BB_TILE, b_hi = a_hi + 2 * BB_TILE, b_lo = b_hi + BN1 * 128;
#pragma unroll
            for (int k8 = 0; k8 < 4; ++k8) {
              const uint32_t off = k8 * 32;
              const uint64_t dah = tc::sdesc_k_sw128(a_hi + off), dal = tc::sdesc_k_sw128(a_lo + off);
              const uint64_t dbh = tc::sdesc_k_sw128(b_hi + off), dbl = tc::sdesc_k_sw128(b_lo + off);
              tc::mma_tf32(d, dah, dbh, idesc1, (kc | k8) != 0);
              tc::mma_tf32(d, dah, dbl, idesc1, 1);
              tc::mma_tf32(d, dal, dbh, idesc1, 1);
            }
            tc::mma_commit(&ctl->empty[s]);
            next();
          }
        }
        tc::mma_commit(&ctl->sfull);   // cosines complete
        for (int c = 0; c < nch; ++c, ++cg) {
          const int slot = cg % BB_ASLOTS;
          const uint32_t use = (uint32_t)(cg / BB_ASLOTS);
          if (!tc::mbar_wait(&ctl->afull[slot], use & 1, abort, err, 18)) return;
          // d q_hat overwrites cosine columns [0, half): the epilogue has read them
          if (c == 0 && !tc::mbar_wait(&ctl->sread, it & 1, abort, err, 18)) return;
          if (!tc::mbar_wait(&ctl->full[s], ph, abort, err, 18)) return;
          tc::fence_after_sync();
          const uint32_t a_hi = tc::smem_u32(aslots + (size_t)slot * BB_ASLOT), a_lo = a_hi + BB_TILE;
          const uint32_t b_hi = tc::smem_u32(ring + (size_t)s * BB_STAGE), b_lo = b_hi + A.half * 128;
#pragma unroll
          for (int k8 = 0; k8 < 4; ++k8) {
            const uint32_t off = k8 * 32;
            const uint64_t dah = tc::sdesc_k_sw128(a_hi + off), dal = tc::sdesc_k_sw128(a_lo + off);
            const uint64_t dbh = tc::sdesc_k_sw128(b_hi + off), dbl = tc::sdesc_k_sw128(b_lo + off);
            tc::mma_tf32(tmem_base, dah, dbh, idesc2, (c | k8) != 0);
            tc::mma_tf32(tmem_base, dah, dbl, idesc2, 1);
            tc::mma_tf32(tmem_base, dal, dbh, idesc2, 1);
          }
          tc::mma_commit(&ctl->empty[s]);
          tc::mma_commit(&ctl->aempty[slot]);
          next();
        }
        tc::mma_commit(&ctl->dqfull);   // d q_hat complete
      }
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                 // TMEM lane = row of the tile
    const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const float T = A.scal[0];
    const float invM = 1.0f / (float)A.M;
    const int Q = A.half / 32;                         // cosine chunks under the d q_hat accumulator
    int cg = 0;
    uint32_t it = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
      const int hc = u / A.m_tiles, mt = u - hc * A.m_tiles;
      const int64_t m = (int64_t)mt * 128 + r;
      const bool owner = m < A.M;
      const float ql = (A.qscale && owner) ? A.qlen[m * A.HC + hc] : 1.f;
      const float ps = A.btgrad ? T * ql : T;
      const float* cn = A.cnt + (int64_t)hc * A.n;
      if (!__all_sync(FULL, tc::mbar_wait(&ctl->sfull, it & 1, abort, err, 19))) break;
      tc::fence_after_sync();
      // row max, then the sum of exp and the count-weighted sum (memory.py:210-214)
      float mx = -INFINITY;
      for (int c0 = 0; c0 < A.n; c0 += 32) {
        uint32_t v[32];
        tc::tmem_ld32(taddr + c0, v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) mx = fmaxf(mx, __uint_as_float(v[t]) * ps);
      }
      float sum = 0.f, sdp = 0.f;
      for (int c0 = 0; c0 < A.n; c0 += 32) {
        uint32_t v[32];
        tc::tmem_ld32(taddr + c0, v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const float e = expf(__uint_as_float(v[t]) * ps - mx);
          sum += e;
          sdp += e * __ldg(cn + c0 + t) * A.dscale;
        }
      }
      sdp /= sum;                                      // sum_i dP_i s_i
      const float inv = 1.0f / sum;
      // the slice of the transposed d cos this tile lands in
      const int64_t tok0 = (int64_t)mt * 128;
      const int64_t sl = tok0 / A.Ks, kk = tok0 - sl * A.Ks + r;
      float* gh = A.dct_hi + ((sl * A.HC + hc) * A.n) * (int64_t)A.Ks + kk;
      float* gl = A.dct_lo + ((sl * A.HC + hc) * A.n) * (int64_t)A.Ks + kk;
      float dTr = 0.f, dqr = 0.f;
      bool ok = true;
      for (int c = 0; c < nch; ++c, ++cg) {
        uint32_t v[32];
        tc::tmem_ld32(taddr + c * 32, v);
        tc::tmem_wait_ld();
        float hi[32], lo[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const float cosv = __uint_as_float(v[t]);
          const float sj = expf(cosv * ps - mx) * inv;
          const float g = sj * (__ldg(cn + c * 32 + t) * A.dscale - sdp) * invM;   // d p_j
          float dc;
          if (A.btgrad) {
            dTr += g * cosv * ql;
            dqr += g * cosv * T;
            dc = g * T * ql;
          } else {
            dc = g * T;                                // sg(T)
          }
          dc = owner ? dc : 0.f;
          hi[t] = tc::to_tf32(dc);
          lo[t] = tc::to_tf32(dc - hi[t]);
        }
        if (c == Q - 1) {   // columns [0, half) read: the d q_hat MMA may overwrite them
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&ctl->sread);
        }
        const int slot = cg % BB_ASLOTS;
        const uint32_t use = (uint32_t)(cg / BB_ASLOTS);
        if (!__all_sync(FULL, tc::mbar_wait(&ctl->aempty[slot], (use & 1) ^ 1, abort, err, 19))) {
          ok = false;
          break;
        }
        // K-major 128-byte-swizzled row r of the slot: 16-byte chunk q at (q ^ (r & 7))
        uint8_t* rowp = aslots + (size_t)slot * BB_ASLOT + r * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int at = ((q ^ (r & 7)) << 4);
          *reinterpret_cast<float4*>(rowp + at) = make_float4(hi[4 * q], hi[4 * q + 1], hi[4 * q + 2], hi[4 * q + 3]);
          *reinterpret_cast<float4*>(rowp + BB_TILE + at) =
              make_float4(lo[4 * q], lo[4 * q + 1], lo[4 * q + 2], lo[4 * q + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&ctl->afull[slot]);
        // transposed d cos: key j's row, 32 consecutive tokens per warp store
        const int64_t kb = (int64_t)c * 32 * A.Ks;
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          gh[kb + (int64_t)t * A.Ks] = hi[t];
          gl[kb + (int64_t)t * A.Ks] = lo[t];
        }
      }
      if (!ok) break;
      if (!__all_sync(FULL, tc::mbar_wait(&ctl->dqfull, it & 1, abort, err, 19))) break;
      tc::fence_after_sync();
      float* dq = A.dqhat + (m * A.HC + hc) * A.half;
      for (int c0 = 0; c0 < A.half; c0 += 32) {
        uint32_t v[32];
        tc::tmem_ld32(taddr + c0, v);
        tc::tmem_wait_ld();
        if (owner) {
#pragma unroll
          for (int t = 0; t < 32; t += 4) {
            float4 x = *reinterpret_cast<float4*>(dq + c0 + t);
            x.x += __uint_as_float(v[t]);
            x.y += __uint_as_float(v[t + 1]);
            x.z += __uint_as_float(v[t + 2]);
            x.w += __uint_as_float(v[t + 3]);
            *reinterpret_cast<float4*>(dq + c0 + t) = x;
          }
        }
      }
      if (owner) {
        A.dT_row[(int64_t)hc * A.M + m] = dTr;
        if (A.dql_row) A.dql_row[m * A.HC + hc] = dqr;
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

}  // namespace

bool bal_bwd_tc_supported(const Dims& D) {
  return D.n % 128 == 0 && D.n <= 512 && (D.half == 32 || D.half == 64 || D.half == 128) && D.M >= 1 &&
         (int64_t)D.H * 2 * D.M < (1ll << 31);
}

BalBwdPlan bal_bwd_plan(const Dims& D, int sms) {
  BalBwdPlan P{};
  const int64_t HC = D.H * 2, n = D.n, half = D.half;
  const int64_t tiles = (D.M + 127) / 128;
  // token slices of the d k_hat GEMM: enough (slice, codebook, key tile) units to fill the SMs
  const int64_t per = HC * ((n + 127) / 128);
  int64_t S = 1;
  while (S < tiles && per * S < 2 * sms && S < 16) S *= 2;
  const int64_t tps = (tiles + S - 1) / S;            // tiles per slice
  P.S = (int)((tiles + tps - 1) / tps);
  P.Ks = (int)(tps * 128);
  P.m_tiles = P.S * (int)tps;
  const int64_t Kp = (int64_t)P.S * P.Ks;
  P.q_floats = HC * D.M * half;
  P.k_floats = HC * n * half;
  P.qt_floats = HC * half * Kp;
  P.dct_floats = HC * n * Kp;
  P.part_floats = (int64_t)P.S * HC * n * half;
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
  // transposed unit queries [slice][hc * half][Ks] (B operand of the d k_hat GEMM)
  if ((e = launch_gather_split(B.qn, (int64_t)HC * half, D.M, 1, (int64_t)HC * half, P.Ks, P.S, (int64_t)HC * half,
                               B.qt_hi, B.qt_lo, 1, 0, 0, s)) != cudaSuccess)
    return e;
  CUtensorMap m[6];
  const int BN1 = n < 128 ? n : 128;
  if ((e = make_tmap_f32(&m[0], B.q_hi, (uint64_t)HC * D.M, half, 128)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[1], B.q_lo, (uint64_t)HC * D.M, half, 128)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[2], B.k_hi, (uint64_t)HC * n, half, BN1)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[3], B.k_lo, (uint64_t)HC * n, half, BN1)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[4], B.kt_hi, (uint64_t)HC * half, n, half)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[5], B.kt_lo, (uint64_t)HC * half, n, half)) != cudaSuccess) return e;
  BalArgs A{};
  A.M = D.M;
  A.HC = HC;
  A.n = n;
  A.half = half;
  A.m_tiles = P.m_tiles;
  A.Ks = P.Ks;
  A.dscale = coef * (float)n / (float)HC / (float)(D.M * D.k);   // dP = coef n / (2H) f, f = cnt / (M k)
  A.btgrad = D.btgrad;
  A.qscale = D.qscale;
  A.cnt = B.cnt;
  A.qlen = B.qlen;
  A.scal = B.scal;
  A.dqhat = B.dqhat;
  A.dT_row = B.dT_row;
  A.dql_row = B.dql_row;
  A.dct_hi = B.dct_hi;
  A.dct_lo = B.dct_lo;
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
  // d k_hat[hc] = sum over slices of d cos[slice, hc]^T Q_hat[slice, hc]
  if ((e = launch_dense_tc_sliced(B.dct_hi, B.dct_lo, n, n, P.Ks, B.qt_hi, B.qt_lo, half, half, P.S * HC, B.part,
                                  B.err, s)) != cudaSuccess)
    return e;
  return launch_sum_slices(B.part, P.S, (int64_t)HC * n, half, B.dkhat, half, false, s);
}

}  // namespace ml
