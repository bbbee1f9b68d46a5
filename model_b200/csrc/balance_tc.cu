// Balance-loss column sums on the tensor cores (memory.py:210-214):
// P[h, c, i] = mean over tokens of softmax(p)[m, h, c, i] with
// p = cos * T (or the full scores under balance_temperature_grad).  Each
// work unit (128-token tile, codebook) passes twice over the codebook's keys
// with the same 3xTF32 MMAs as the score kernel (TMA-fed, TMEM
// accumulators): pass 1 keeps every row's online max and sum of
// exp(p - max) (the two warps of a lane quarter combine their column halves
// through shared memory), pass 2 turns each TMEM row into
// exp(p - max) / sum.  Column sums over a warp's 32 rows come from a
// butterfly transpose-reduction (31 shuffles per 32 columns, fixed order)
// and are written per (tile, lane quarter); the finalize kernel adds the
// partials in a fixed order.
#include "tc_pipeline.cuh"

namespace ml {

namespace {

constexpr int EPI_WARPS = 8;
constexpr int BT_THREADS = 64 + 32 * EPI_WARPS;
constexpr int BT_BN = 256;

// v[i] holds this lane's row value of column i (32 columns); returns the
// sum over the warp's 32 rows of column `lane`.
__device__ __forceinline__ float column_sums32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = up ? v[i] : v[i + o];
      const float keep = up ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(FULL, send, o);
    }
  }
  return v[0];
}

template <bool PQ>   // PQ: p carries q_len (balance_temperature_grad with query_scale)
__global__ void __launch_bounds__(BT_THREADS, 1)
    balance_tc_kernel(const __grid_constant__ CUtensorMap tA_hi, const __grid_constant__ CUtensorMap tA_lo,
                      const __grid_constant__ CUtensorMap tB_hi, const __grid_constant__ CUtensorMap tB_lo, Dims D,
                      tc::PipeShape P, int m_tiles, int n_chunks, const float* __restrict__ qlen,
                      const float* __restrict__ scal, float* __restrict__ p_part, int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  tc::PipeCtl* ctl = reinterpret_cast<tc::PipeCtl*>(smem);
  uint8_t* tiles = smem + 1024;
  float* mrow = reinterpret_cast<float*>(tiles + (size_t)P.stages * P.stage_bytes);   // [2 halves][128][max, sum]
  volatile int* abort = &ctl->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HC = D.H * 2;
  const int units = m_tiles * HC;
  auto coords = [&](int u, int& arow, int& brow0, int& nch) {
    const int hc = u / m_tiles, mt = u - hc * m_tiles;
    arow = (int)(hc * D.M + (int64_t)mt * tc::PIPE_M);
    brow0 = hc * D.n;
    nch = 2 * n_chunks;                       // pass 1: row max / sum, pass 2: column sums
  };
  const uint32_t tmem_base = tc::pipe_init(ctl, P, EPI_WARPS);
  if (warp == 0) {
    if (lane == 0) tc::pipe_produce(ctl, P, tiles, units, &tA_hi, &tA_lo, &tB_hi, &tB_lo, coords, err, n_chunks);
  } else if (warp == 1) {
    if (lane == 0) tc::pipe_mma(ctl, P, tiles, units, tmem_base, coords, err);
  } else {
    const int quarter = warp & 3, hf = (warp - 2) >> 2;
    const int half_bn = P.BN >> 1;
    const int r_in_tile = quarter * 32 + lane;
    const float T = scal[0];
    uint64_t* pb = &ctl->pair[quarter];
    int acc = 0;
    uint32_t aph = 0, pph = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      const int hc = u / m_tiles, mt = u - hc * m_tiles;
      const int h = hc >> 1, c = hc & 1;
      const int64_t m = (int64_t)mt * tc::PIPE_M + r_in_tile;
      const bool owner = m < D.M;
      const int64_t row = (m * D.H + h) * 2 + c;
      const float ql = (PQ && owner) ? qlen[row] : 1.f;
      float* dst = p_part + ((int64_t)(mt * 4 + quarter) * HC + hc) * D.n;
      float rmax = -INFINITY, rsum = 0.f, rinv = 0.f;
      for (int j = 0; j < 2 * n_chunks; ++j) {
        if (!__all_sync(FULL, tc::mbar_wait(&ctl->tfull[acc], aph, abort, err, 16))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const bool pass2 = j >= n_chunks;
        const int key0 = (pass2 ? j - n_chunks : j) * P.BN;
        const int valid = min(P.BN, D.n - key0);
        const int cb = hf * half_bn, ce = min(cb + half_bn, valid);
        const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * tc::PIPE_ACC_STRIDE);
        for (int cc = cb; cc < ce; cc += 32) {
          uint32_t r[32];
          tc::tmem_ld32(taddr + cc, r);
          tc::tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            float p = __fmul_rn(__uint_as_float(r[t]), T);              // memory.py:211 cos * sg(T)
            if (PQ) p = __fmul_rn(p, ql);                               //   or the full scores
            v[t] = (cc + t < ce) ? p : -INFINITY;
          }
          if (!pass2) {
            float cmax = v[0];
#pragma unroll
            for (int t = 1; t < 32; ++t) cmax = fmaxf(cmax, v[t]);
            const float nmax = fmaxf(rmax, cmax);
            float cs = 0.f;
#pragma unroll
            for (int t = 0; t < 32; ++t) cs += __expf(v[t] - nmax);
            rsum = (rmax == -INFINITY ? 0.f : rsum * __expf(rmax - nmax)) + cs;
            rmax = nmax;
          } else {
#pragma unroll
            for (int t = 0; t < 32; ++t) v[t] = owner ? __expf(v[t] - rmax) * rinv : 0.f;   // softmax entry
            const float colsum = column_sums32(v, lane);
            if (cc + lane < ce) dst[key0 + cc + lane] = colsum;
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&ctl->tempty[acc]);
        acc ^= 1;
        if (acc == 0) aph ^= 1;
        if (j == n_chunks - 1) {
          // the row's two column halves: combine (max, sum) in half order
          mrow[(hf * tc::PIPE_M + r_in_tile) * 2] = rmax;
          mrow[(hf * tc::PIPE_M + r_in_tile) * 2 + 1] = rsum;
          if (!tc::pair_sync(pb, pph, lane, abort, err)) {
            ok = false;
            break;
          }
          const float m0 = mrow[r_in_tile * 2], s0 = mrow[r_in_tile * 2 + 1];
          const float m1 = mrow[(tc::PIPE_M + r_in_tile) * 2], s1 = mrow[(tc::PIPE_M + r_in_tile) * 2 + 1];
          rmax = fmaxf(m0, m1);
          rsum = (m0 == -INFINITY ? 0.f : s0 * __expf(m0 - rmax)) + (m1 == -INFINITY ? 0.f : s1 * __expf(m1 - rmax));
          rinv = 1.0f / rsum;
        }
      }
      // both halves have read mrow before either writes it for the next unit
      if (ok && !tc::pair_sync(pb, pph, lane, abort, err)) ok = false;
    }
  }
  tc::pipe_finish(ctl, tmem_base);
}

}  // namespace

// Partial column sums land in p_part[(tile * 4 + quarter)][H * 2][n]; the
// number of partial planes is returned in *planes.
cudaError_t launch_balance_tc(const Dims& D, const Work& W, int* planes, cudaStream_t s) {
  const int m_tiles = (int)((D.M + tc::PIPE_M - 1) / tc::PIPE_M);
  *planes = m_tiles * 4;
  if (D.M == 0) return cudaSuccess;
  const int BN = D.n >= BT_BN ? BT_BN : ((D.n + 15) / 16) * 16;
  tc::PipeShape P = tc::pipe_shape(BN, D.half, 2 * tc::PIPE_M * 2 * sizeof(float));
  if (P.stages < 2) return cudaErrorInvalidConfiguration;
  const int n_chunks = (D.n + BN - 1) / BN;
  CUtensorMap m[4];
  cudaError_t e;
  const uint64_t arows = (uint64_t)D.M * D.H * 2, brows = (uint64_t)D.n * D.H * 2;
  if ((e = make_tmap_f32(&m[0], W.q_hi, arows, D.half, tc::PIPE_M)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[1], W.q_lo, arows, D.half, tc::PIPE_M)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[2], W.k_hi, brows, D.half, BN)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[3], W.k_lo, brows, D.half, BN)) != cudaSuccess) return e;
  const size_t smem = 2048 + (size_t)P.stages * P.stage_bytes + 2 * tc::PIPE_M * 2 * sizeof(float);
  auto kern = (D.btgrad && D.qscale) ? balance_tc_kernel<true> : balance_tc_kernel<false>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
    return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int units = m_tiles * D.H * 2;
  kern<<<units < sms ? units : sms, BT_THREADS, smem, s>>>(m[0], m[1], m[2], m[3], D, P, m_tiles, n_chunks, W.qlen,
                                                           W.scal, W.p_part, W.err);
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
