// Backward of one memory layer (model.py:110-119 with memory.py:133-214):
// the gradients of sum(dy * y) + balance_coef * balance_loss that the
// reference trainer's jax.value_and_grad computes with sparse_grad (the
// value table gets none; its rows' gradient is the read-output gradient,
// the "probe" of model.py:114-115).  Routing (the forward's slots and
// weights, its clean top-k counts) carries no gradient; the temperature
// clamp is straight-through (memory.py:141-146).
//
//   route_bwd_kernel   one CTA per token, one warp per head: the read is
//                      recomputed (mem = sum w V[slot], heads in order),
//                      then probe = dmemg * gate, mem * gate, the gate
//                      pre-activation gradient, dw_r = probe . V[slot_r],
//                      the softmax backward, and the slot-score gradient
//                      split onto the two halves' sub-keys (slot = a n + b);
//                      per distinct sub-key it adds dcos k_hat into d q_hat
//                      and emits (sub-key, dcos) entries whose q_hat-weighted
//                      sums are the sparse sub-key gradient; on a
//                      row-sharded table (SH) probe, mem * gate and the
//                      gate gradient come from shard.cu's probe kernel and
//                      each dw_r from the dots its row's owner returned;
//   bal_row_kernel     (balance term, shapes the fused tensor-core kernel of
//                      bal_bwd_tc.cu does not take: n not a multiple of 128,
//                      fewer than 128 tokens) per (token, codebook) row the
//                      softmax of p over all n keys from the recomputed
//                      cosines, and d p = s (dP - sum dP s) / M turned into
//                      d cos;
//   GEMMs              (recomputed projections, Dense-layer gradients, the
//                      dense balance contractions) on the tensor cores as
//                      3xTF32 (gemm_any.cu), long sums split over the SMs
//                      and added back in a fixed order;
//   norm backward      x * rsqrt(|x|^2 + 1e-6) for the queries and sub-keys.
// Every sum runs in a fixed order: results are deterministic.
#include "combine.cuh"
#include "layer_bwd.cuh"
#include "shard.cuh"

namespace ml {

namespace {

__global__ void fill_kernel(float* __restrict__ x, int64_t n, float v) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e < n) x[e] = v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// ---------------------------------------------------------------------------
// route_bwd_kernel: one CTA per token, warp h = pool head.  d <= 1024,
// half <= 128, k <= 32.
// ---------------------------------------------------------------------------
template <typename VT, int VEC, int CH, bool SH>
__global__ void __launch_bounds__(1024) route_bwd_kernel(
    Dims D, const VT* __restrict__ values, const int* __restrict__ slots, const float* __restrict__ weights,
    const float* __restrict__ dmemg, const float* __restrict__ zg, const float* __restrict__ qn,
    const float* __restrict__ qlen, const float* __restrict__ keys_n, const float* __restrict__ scal,
    float* __restrict__ probe, float* __restrict__ memg, float* __restrict__ dzg, float* __restrict__ dqhat,
    float* __restrict__ dqlen, float* __restrict__ dT_part, int* __restrict__ ent_slot, float* __restrict__ ent_w,
    const BwdShard X, const float* __restrict__ mem_fwd) {
  extern __shared__ float bsm[];
  float* red = bsm;                 // [H][d]
  float* dmem_s = bsm + D.H * D.d;  // [d]
  const int64_t m = blockIdx.x;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k = D.k, d = D.d, n = D.n, half = D.half;
  const int64_t ow = (m * D.H + h) * k;
  const int s_in = lane < k ? slots[ow + lane] : 0;
  const bool s_ok = s_in >= 0 && (int64_t)s_in < D.N;   // an id outside the table reads nothing
  const int slot_l = s_ok ? s_in : 0;
  const float w_l = (lane < k && s_ok) ? weights[ow + lane] : 0.f;
  // read (slot + N/2 + 1) % N under shuffle_reads (memory.py:179)
  const int64_t rs_l = D.shuffle ? ((int64_t)slot_l + D.N / 2 + 1) % D.N : (int64_t)slot_l;
  const int groups = d / VEC;
  float dw_l = 0.f;
  if constexpr (SH) {
    // row-sharded table: probe, memg and dzg come from the probe kernel, and
    // dw_r = probe . V[read slot r] from the slot's owner rank, stored in the
    // owner's inbox order (per owner: heads in order, then lanes in order)
    __shared__ int cnt_s[32][MEMLAYER_MAX_SHARDS];
    __shared__ int ok_s;
    const int P = X.world;
    if (threadIdx.x == 0) {
      bool ok = true;
      for (int o = 0; o < P && ok; ++o) ok = wait_epoch(X.flags + o, X.epoch, X.err, 36, X.wait_ns);
      ok_s = ok;
    }
    const int own = (lane < k && s_ok) ? (int)(rs_l % P) : -1;   // an id outside the table has no owner
    const unsigned lt = (1u << lane) - 1u;
    int pos = 0;
    for (int o = 0; o < P; ++o) {
      const unsigned mk = __ballot_sync(FULL, own == o);
      if (own == o) pos = __popc(mk & lt);
      if (lane == 0) cnt_s[h][o] = __popc(mk);
    }
    __syncthreads();
    if (own >= 0 && ok_s) {
      int base = 0;
      for (int hh = 0; hh < h; ++hh) base += cnt_s[hh][own];
      dw_l = __ldcg(X.dots + ((int64_t)own * X.mcap + m) * ((int64_t)D.H * k) + base + pos);
    }
  } else {
  // 1. mem = sum_h sum_r w V[read slot] (memory.py:192), as the forward
  // gather -- unless the forward's read output is given (one pass over the
  // rows instead of two)
  if (!mem_fwd) {
  float acc[CH][VEC];
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[c][v] = 0.f;
#pragma unroll 4
  for (int r = 0; r < k; ++r) {
    const int64_t row = __shfl_sync(FULL, rs_l, r);
    const float wr = __shfl_sync(FULL, w_l, r);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int g = c * 32 + lane;
      if (g < groups) {
        float x[VEC];
        load_group<VT, VEC>(values + row * d + g * VEC, x);
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[c][v] = fmaf(wr, x[v], acc[c][v]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int g = c * 32 + lane;
    if (g < groups)
#pragma unroll
      for (int v = 0; v < VEC; ++v) red[h * d + g * VEC + v] = acc[c][v];
  }
  }
  __syncthreads();
  // 2. gate, probe (d read output), mem * gate, d gate pre-activation (model.py:118-119)
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float mv = 0.f;
    if (mem_fwd)
      mv = mem_fwd[m * d + i];
    else
      for (int hh = 0; hh < D.H; ++hh) mv += red[hh * d + i];
    const float z = zg[m * d + i], sg = sigmoidf_(z), gate = z * sg;
    const float dm_ = dmemg[m * d + i];
    const float dmem = dm_ * gate;
    probe[m * d + i] = dmem;
    memg[m * d + i] = mv * gate;
    dzg[m * d + i] = dm_ * mv * sg * (1.0f + z * (1.0f - sg));     // silu'
    dmem_s[i] = dmem;
  }
  __syncthreads();
  // 3. dw_r = dmem . V[read slot r]; softmax backward (memory.py:178).
  // Four rows at a time: their loads in flight together, their four warp
  // reductions interleaved.
  constexpr int RB = 4;
  for (int r0 = 0; r0 < k; r0 += RB) {
    float s[RB];
#pragma unroll
    for (int b = 0; b < RB; ++b) {
      s[b] = 0.f;
      const int r = r0 + b;
      const int64_t row = __shfl_sync(FULL, rs_l, r < k ? r : 0);
      if (r < k) {
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int g = c * 32 + lane;
          if (g < groups) {
            float x[VEC];
            load_group<VT, VEC>(values + row * d + g * VEC, x);
#pragma unroll
            for (int v = 0; v < VEC; ++v) s[b] = fmaf(dmem_s[g * VEC + v], x[v], s[b]);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int b = 0; b < RB; ++b) s[b] += __shfl_xor_sync(FULL, s[b], o);
#pragma unroll
    for (int b = 0; b < RB; ++b)
      if (lane == r0 + b) dw_l = s[b];
  }
  }
  const float swdw = warp_sum(lane < k ? w_l * dw_l : 0.f);
  const float dss_l = lane < k ? w_l * (dw_l - swdw) : 0.f;
  // 4. slot score = scores[0, a] + scores[1, b]; per half, per distinct sub-key
  const float T = scal[0];
  float dT = 0.f;
  for (int c = 0; c < 2; ++c) {
    const int key_l = c == 0 ? slot_l / n : slot_l % n;
    // lane r owns its key if no earlier lane holds it; its ds sums every lane with the key
    bool own = lane < k;
    float ds = 0.f;
    for (int r = 0; r < k; ++r) {
      const int kr = __shfl_sync(FULL, key_l, r);
      const float dr = __shfl_sync(FULL, dss_l, r);
      if (kr == key_l && lane < k) {
        ds += dr;
        if (r < lane) own = false;
      }
    }
    const int64_t qrow = (m * D.H + h) * 2 + c;
    const int hc = h * 2 + c;
    const float ql = D.qscale ? qlen[qrow] : 1.f;
    const float scale = T * ql;
    constexpr int DV = 4;   // half <= 128: 4 dimensions per lane
    float qv[DV], dq[DV];
#pragma unroll
    for (int e = 0; e < DV; ++e) {
      const int dd = lane + 32 * e;
      qv[e] = dd < half ? qn[qrow * half + dd] : 0.f;
      dq[e] = 0.f;
    }
    float dql = 0.f;
    int j = 0;
    const unsigned owners = __ballot_sync(FULL, own);
    for (int r = 0; r < k; ++r) {
      if (!((owners >> r) & 1u)) continue;
      const int i = __shfl_sync(FULL, key_l, r);
      const float dsr = __shfl_sync(FULL, ds, r);
      const float* kr = keys_n + ((int64_t)hc * n + i) * half;
      float kv[DV], cs = 0.f;
#pragma unroll
      for (int e = 0; e < DV; ++e) {
        const int dd = lane + 32 * e;
        kv[e] = dd < half ? kr[dd] : 0.f;
        cs = fmaf(qv[e], kv[e], cs);
      }
      const float cosv = warp_sum(cs);                           // memory.py:149
      const float dcos = dsr * scale;                            // memory.py:150-152
#pragma unroll
      for (int e = 0; e < DV; ++e) dq[e] = fmaf(dcos, kv[e], dq[e]);
      dT += dsr * cosv * ql;
      dql += dsr * cosv * T;
      if (lane == 0) {
        ent_slot[qrow * k + j] = hc * n + i;
        ent_w[qrow * k + j] = dcos;
      }
      ++j;
    }
    if (lane == 0)
      for (int jj = j; jj < k; ++jj) {   // padding entries add nothing
        ent_slot[qrow * k + jj] = hc * n;
        ent_w[qrow * k + jj] = 0.f;
      }
#pragma unroll
    for (int e = 0; e < DV; ++e) {
      const int dd = lane + 32 * e;
      if (dd < half) dqhat[qrow * half + dd] = dq[e];
    }
    if (lane == 0 && dqlen) dqlen[qrow] = D.qscale ? dql : 0.f;
  }
  if (lane == 0) dT_part[m * D.H + h] = dT;
}

// ---------------------------------------------------------------------------
// Balance term (memory.py:205-214): per (token, codebook) row, C holds the
// cosines over all n keys on entry and d cos on exit; dT_row / dql_row get
// the row's temperature / q_len gradient under balance_temperature_grad.
// One warp per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) bal_row_kernel(Dims D, float* __restrict__ C, const float* __restrict__ cnt,
                                                      const float* __restrict__ qlen, const float* __restrict__ scal,
                                                      float coef, float* __restrict__ dT_row,
                                                      float* __restrict__ dql_row) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);   // hc * M + m
  const int64_t rows = (int64_t)D.H * 2 * D.M;
  if (row >= rows) return;
  const int hc = (int)(row / D.M);
  const int64_t m = row - (int64_t)hc * D.M;
  const int n = D.n;
  const float T = scal[0];
  const int h = hc >> 1, c = hc & 1;
  const float ql = D.qscale ? qlen[(m * D.H + h) * 2 + c] : 1.f;
  float* cr = C + row * n;
  // p = scores (balance_temperature_grad) or cos * sg(T)
  const float ps = D.btgrad ? T * ql : T;
  float mx = -INFINITY;
  for (int j = lane; j < n; j += 32) mx = fmaxf(mx, cr[j] * ps);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  float sum = 0.f, sdp = 0.f;
  const float* cn = cnt + (int64_t)hc * n;
  const float dscale = coef * (float)n / (float)(D.H * 2) / (float)(D.M * D.k);   // dP = coef n/(2H) f, f = cnt/(M k)
  for (int j = lane; j < n; j += 32) {
    const float e = expf(cr[j] * ps - mx);
    sum += e;
    sdp += e * cn[j] * dscale;
  }
  sum = warp_sum(sum);
  sdp = warp_sum(sdp) / sum;                     // sum_i dP_i s_i
  const float inv = 1.0f / sum, invM = 1.0f / (float)D.M;
  float dTr = 0.f, dqr = 0.f;
  for (int j = lane; j < n; j += 32) {
    const float cosv = cr[j];
    const float s = expf(cosv * ps - mx) * inv;
    const float g = s * (cn[j] * dscale - sdp) * invM;   // d p_j
    if (D.btgrad) {
      dTr += g * cosv * ql;
      dqr += g * cosv * T;
      cr[j] = g * T * ql;
    } else {
      cr[j] = g * T;                                  // sg(T): no temperature gradient
    }
  }
  dTr = warp_sum(dTr);
  dqr = warp_sum(dqr);
  if (lane == 0) {
    dT_row[row] = dTr;
    if (dql_row) dql_row[(m * D.H + h) * 2 + c] = dqr;   // the queries' row layout [M, H, 2]
  }
}

// x_hat = x * rsqrt(|x|^2 + 1e-6): dx = r (dx_hat - (x_hat . dx_hat) x_hat)
// (+ dq_len x_hat / sqrt(half) for the queries), one warp per row.
__global__ void __launch_bounds__(256) norm_bwd_kernel(const float* __restrict__ xhat, const float* __restrict__ dxhat,
                                                       const float* __restrict__ rnorm_len, int64_t rows, int half,
                                                       const float* __restrict__ raw, const float* __restrict__ dlen,
                                                       const float* __restrict__ dlen2, float* __restrict__ dx,
                                                       const float* __restrict__ dxhat2) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = xhat + row * half;
  const float* gr = dxhat + row * half;
  const float* g2 = dxhat2 ? dxhat2 + row * half : nullptr;   // a second share of d x_hat (balance term)
  float r;
  if (raw) {   // sub-keys: r from the raw row
    float ss = 0.f;
    for (int i = lane; i < half; i += 32) ss = fmaf(raw[row * half + i], raw[row * half + i], ss);
    r = 1.0f / sqrtf(warp_sum(ss) + 1e-6f);
  } else {     // queries: |q|' = q_len sqrt(half)
    r = 1.0f / (rnorm_len[row] * sqrtf((float)half));
  }
  float dot = 0.f;
  for (int i = lane; i < half; i += 32) dot = fmaf(xr[i], g2 ? gr[i] + g2[i] : gr[i], dot);
  dot = warp_sum(dot);
  const float dl = (dlen ? dlen[row] : 0.f) + (dlen2 ? dlen2[row] : 0.f);
  for (int i = lane; i < half; i += 32)
    dx[row * half + i] = r * ((g2 ? gr[i] + g2[i] : gr[i]) - dot * xr[i]) + dl * xr[i] / sqrtf((float)half);
}

// dkhat[uniq[u]] += rows[u] (distinct ids; padding ids >= N skipped)
__global__ void scatter_rows_kernel(const int* __restrict__ uniq, const float* __restrict__ rows, int64_t cap, int64_t N,
                                    int half, float* __restrict__ dst) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= cap * half) return;
  const int64_t u = e / half;
  const int id = uniq[u];
  if (id < 0 || id >= N) return;
  dst[(int64_t)id * half + (e - u * half)] += rows[e];
}

// dlog_t = T * (sum of the per-(token, head) and per-row partials, in order)
__global__ void __launch_bounds__(1024) dlogt_kernel(const float* __restrict__ a, int64_t na, const float* __restrict__ b,
                                                     int64_t nb, const float* __restrict__ scal, float* __restrict__ out) {
  __shared__ double red[32];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < na; i += blockDim.x) s += (double)a[i];
  for (int64_t i = threadIdx.x; i < nb; i += blockDim.x) s += (double)b[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    *out = (float)(t * (double)scal[0]);   // straight-through clamp: d T / d log_t = T
  }
}

inline int ch_for(int groups) {
  int ch = (groups + 31) / 32;
  return ch <= 1 ? 1 : ch <= 2 ? 2 : ch <= 4 ? 4 : ch <= 8 ? 8 : -1;
}

template <typename VT, int VEC, bool SH>
cudaError_t route_bwd_ch(const Dims& D, const VT* values, const LayerBwd& B, const BwdShard& X, cudaStream_t s) {
  const size_t smem = SH ? 0 : sizeof(float) * ((size_t)D.H * D.d + D.d);
  const dim3 grid((unsigned)D.M), block(32 * D.H);
#define ML_RB(CHV)                                                                                              \
  {                                                                                                             \
    auto kern = route_bwd_kernel<VT, VEC, CHV, SH>;                                                             \
    if (smem > 48 * 1024) {                                                                                     \
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);       \
      if (e != cudaSuccess) return e;                                                                           \
    }                                                                                                           \
    kern<<<grid, block, smem, s>>>(D, values, B.slots, B.weights, B.dmemg, B.zg, B.qn, B.qlen, B.keys_n, B.scal, \
                                   B.probe, B.memg, B.dzg, B.dqhat, B.dqlen, B.dT_part, B.ent_slot, B.ent_w, X,  \
                                   B.mem_fwd);                                                                  \
  }
  switch (ch_for(D.d / VEC)) {
    case 1: ML_RB(1); break;
    case 2: ML_RB(2); break;
    case 4: ML_RB(4); break;
    case 8: ML_RB(8); break;
    default: return cudaErrorInvalidValue;
  }
#undef ML_RB
  count_launch();
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fill(float* x, int64_t n, float v, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, n, v);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_route_bwd(const Dims& D, const void* values, const LayerBwd& B, cudaStream_t s) {
  if (D.M == 0) return cudaSuccess;
  const BwdShard X{};
  if (D.vdtype == MEMLAYER_F16) return route_bwd_ch<__half, 8, false>(D, (const __half*)values, B, X, s);
  if (D.vdtype == MEMLAYER_BF16)
    return route_bwd_ch<__nv_bfloat16, 8, false>(D, (const __nv_bfloat16*)values, B, X, s);
  if (D.d % 4 == 0 && (reinterpret_cast<uintptr_t>(values) & 15) == 0)
    return route_bwd_ch<float, 4, false>(D, (const float*)values, B, X, s);
  return route_bwd_ch<float, 1, false>(D, (const float*)values, B, X, s);
}

cudaError_t launch_route_bwd_sharded(const Dims& D, const LayerBwd& B, const BwdShard& X, cudaStream_t s) {
  if (D.M == 0) return cudaSuccess;
  return route_bwd_ch<float, 4, true>(D, nullptr, B, X, s);
}

cudaError_t launch_bal_rows(const Dims& D, float* C, const float* cnt, const float* qlen, const float* scal, float coef,
                            float* dT_row, float* dql_row, cudaStream_t s) {
  const int64_t rows = (int64_t)D.H * 2 * D.M;
  if (rows == 0) return cudaSuccess;
  bal_row_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(D, C, cnt, qlen, scal, coef, dT_row, dql_row);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_norm_bwd(const float* xhat, const float* dxhat, const float* len, int64_t rows, int half,
                            const float* raw, const float* dlen, const float* dlen2, float* dx, cudaStream_t s,
                            const float* dxhat2) {
  if (rows == 0) return cudaSuccess;
  norm_bwd_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(xhat, dxhat, len, rows, half, raw, dlen, dlen2, dx,
                                                              dxhat2);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_scatter_rows(const int* uniq, const float* rows, int64_t cap, int64_t N, int half, float* dst,
                                cudaStream_t s) {
  if (cap == 0) return cudaSuccess;
  const int64_t n = cap * half;
  scatter_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(uniq, rows, cap, N, half, dst);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_dlogt(const float* a, int64_t na, const float* b, int64_t nb, const float* scal, float* out,
                         cudaStream_t s) {
  dlogt_kernel<<<1, 1024, 0, s>>>(a, na, b, nb, scal, out);
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
