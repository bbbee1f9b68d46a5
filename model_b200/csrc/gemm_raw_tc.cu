// Strided float32 GEMM on the 5th-generation tensor cores that splits its
// operands itself: C (+)= A B (+ bias) with A(i, k) and B(k, j) read as
// stored, in either stride order, by TMA.  Used by the layer backward
// (gemm_any.cu) for the Dense-layer gradients, the recomputed projections
// and d h (model.py:110-119 differentiated).
//
// CTA = 10 warps, persistent over units (K slice, 128-row tile, column tile):
//   warp 0     TMA producer: raw float32 tiles of A [128 x 32 k] and B
//              [BN x 32 k] into a raw ring.  An operand whose k is the
//              contiguous index is loaded K-major with the 128-byte swizzle
//              (the MMA's own layout); one whose row index is contiguous is
//              loaded as [32 k][rows] without swizzle;
//   warp 1     MMA issuer: 128 x BN float32 accumulators, double-buffered in
//              TMEM, 3 kind::tf32 MMAs per K step (hi.hi + hi.lo + lo.hi);
//   warps 2-5  converters: each raw tile -> tf32 hi / lo tiles in the MMA
//              ring (rna_tf32(x), rna_tf32(x - hi)), transposing the
//              row-contiguous ones into the K-major swizzled layout;
//   warps 6-9  epilogue: TMEM lane = output row; 32 x 32 pieces staged in
//              shared memory and written as 4 rows x 128 bytes per store,
//              with the bias added and the destination accumulated when asked.
// A long inner dimension with few output tiles is cut into S K slices (tile
// coordinates, no copies); the partial products are added in slice order by
// the caller.  Every mbarrier wait is bounded.
#include "gemm_any.cuh"
#include "tc_common.cuh"

namespace ml {

namespace {

constexpr int GR_THREADS = 320;
constexpr int GR_CONV_WARPS = 4, GR_EPI_WARPS = 4;
constexpr int GR_RAW = 2, GR_MMA = 2;              // ring depths
constexpr uint32_t GR_TILE = 128 * 32 * 4;         // 16 KB: 128 rows x 32 float32
constexpr uint32_t GR_STG = 32 * 33;               // floats per epilogue warp's staging piece
constexpr uint32_t GR_SMEM = 2048 + GR_RAW * 2 * GR_TILE + GR_MMA * 4 * GR_TILE + GR_EPI_WARPS * GR_STG * 4;

struct GrCtl {
  uint64_t raw_full[GR_RAW], raw_empty[GR_RAW], mma_full[GR_MMA], mma_empty[GR_MMA], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort;
};

struct GrArgs {
  int64_t M, N, K;      // per batch
  int BN;
  int batch;            // independent products: A rows + b a_boff, B rows + b b_boff, C + b c_boff
  int a_boff, b_boff;
  int64_t c_boff;
  int a_kmajor, b_kmajor;   // operand loaded K-major (swizzled) or row-contiguous
  int m_tiles, n_tiles, S, kq_slice;   // kq_slice: 32-element K stages per slice
  float* out;               // slice s writes out + s out_stride (ld) ...
  int64_t out_stride, ld;
  const float* bias;        // ... plus bias[j] (direct mode only)
  int accumulate;           // ... added to the destination (direct mode only)
  int vec;                  // 16-byte stores allowed
  int* err;
};

// Convert one raw tile of `rows` rows into K-major swizzled hi / lo tiles.
__device__ __forceinline__ void convert_tile(const float* raw, bool kmajor, int rows, float* hi, float* lo, int t) {
  if (kmajor) {   // same swizzled layout: elementwise
    const float4* r4 = reinterpret_cast<const float4*>(raw);
    float4* h4 = reinterpret_cast<float4*>(hi);
    float4* l4 = reinterpret_cast<float4*>(lo);
    for (int i = t; i < rows * 8; i += 128) {
      const float4 x = r4[i];
      float4 h, l;
      h.x = tc::to_tf32_int(x.x); l.x = tc::to_tf32_int(x.x - h.x);
      h.y = tc::to_tf32_int(x.y); l.y = tc::to_tf32_int(x.y - h.y);
      h.z = tc::to_tf32_int(x.z); l.z = tc::to_tf32_int(x.z - h.z);
      h.w = tc::to_tf32_int(x.w); l.w = tc::to_tf32_int(x.w - h.w);
      h4[i] = h;
      l4[i] = l;
    }
  } else if (t < rows) {   // raw [32 k][rows]: thread t builds row t
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = raw[k * rows + t];
    uint8_t* hrow = reinterpret_cast<uint8_t*>(hi) + t * 128;
    uint8_t* lrow = reinterpret_cast<uint8_t*>(lo) + t * 128;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 h, l;
      h.x = tc::to_tf32_int(v[4 * q]); l.x = tc::to_tf32_int(v[4 * q] - h.x);
      h.y = tc::to_tf32_int(v[4 * q + 1]); l.y = tc::to_tf32_int(v[4 * q + 1] - h.y);
      h.z = tc::to_tf32_int(v[4 * q + 2]); l.z = tc::to_tf32_int(v[4 * q + 2] - h.z);
      h.w = tc::to_tf32_int(v[4 * q + 3]); l.w = tc::to_tf32_int(v[4 * q + 3] - h.w);
      const int at = (q ^ (t & 7)) << 4;
      *reinterpret_cast<float4*>(hrow + at) = h;
      *reinterpret_cast<float4*>(lrow + at) = l;
    }
  }
}

__global__ void __launch_bounds__(GR_THREADS, 1)
    gemm_raw_tc_kernel(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB, GrArgs G) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GrCtl* ctl = reinterpret_cast<GrCtl*>(smem);
  uint8_t* raw = smem + 1024;                              // [GR_RAW][A, B] raw tiles
  uint8_t* mma = raw + GR_RAW * 2 * GR_TILE;               // [GR_MMA][A hi, A lo, B hi, B lo]
  float* stg_all = reinterpret_cast<float*>(mma + GR_MMA * 4 * GR_TILE);
  volatile int* abort = &ctl->abort;
  int* err = G.err;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_batch = G.m_tiles * G.n_tiles;
  const int per_slice = per_batch * G.batch;
  const int units = per_slice * G.S;
  const uint32_t bbytes = (uint32_t)G.BN * 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GR_RAW; ++s) {
      tc::mbar_init(&ctl->raw_full[s], 1);
      tc::mbar_init(&ctl->raw_empty[s], GR_CONV_WARPS);
    }
    for (int s = 0; s < GR_MMA; ++s) {
      tc::mbar_init(&ctl->mma_full[s], GR_CONV_WARPS);
      tc::mbar_init(&ctl->mma_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&ctl->tfull[b], 1);
      tc::mbar_init(&ctl->tempty[b], GR_EPI_WARPS);
    }
    ctl->abort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(&ctl->tmem_base, 256);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = ctl->tmem_base;

  // unit u = (slice, batch, column tile, row tile), row tile fastest
  auto unit = [&](int u, int& sl, int& b, int& nt, int& mt) {
    sl = u / per_slice;
    int v = u - sl * per_slice;
    b = v / per_batch;
    v -= b * per_batch;
    nt = v / G.m_tiles;
    mt = v - nt * G.m_tiles;
  };
  auto stages_of = [&](int sl) {
    const int64_t k0 = (int64_t)sl * G.kq_slice * 32;
    const int64_t rem = (G.K - k0 + 31) / 32;
    return (int)(rem < G.kq_slice ? rem : G.kq_slice);
  };

  if (warp == 0) {
    if (lane == 0) {
      tc::prefetch_tmap(&tA);
      tc::prefetch_tmap(&tB);
      int s = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        int sl, b, nt, mt;
        unit(u, sl, b, nt, mt);
        const int nk = stages_of(sl);
        const int ar = b * G.a_boff + mt * 128, br = b * G.b_boff + nt * G.BN;
        for (int kc = 0; kc < nk; ++kc) {
          const int k = (sl * G.kq_slice + kc) * 32;
          if (!tc::mbar_wait(&ctl->raw_empty[s], ph ^ 1, abort, err, 11)) return;
          uint8_t* st = raw + (size_t)s * 2 * GR_TILE;
          tc::mbar_expect_tx(&ctl->raw_full[s], GR_TILE + bbytes);
          if (G.a_kmajor)
            tc::tma_load_2d(st, &tA, &ctl->raw_full[s], k, ar);
          else
            tc::tma_load_2d(st, &tA, &ctl->raw_full[s], ar, k);
          if (G.b_kmajor)
            tc::tma_load_2d(st + GR_TILE, &tB, &ctl->raw_full[s], k, br);
          else
            tc::tma_load_2d(st + GR_TILE, &tB, &ctl->raw_full[s], br, k);
          if (++s == GR_RAW) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_tf32(128, G.BN);
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        int sl, b, nt, mt;
        unit(u, sl, b, nt, mt);
        const int nk = stages_of(sl);
        if (!tc::mbar_wait(&ctl->tempty[acc], aph ^ 1, abort, err, 12)) return;
        tc::fence_after_sync();
        const uint32_t d = tmem_base + (uint32_t)(acc * 128);
        for (int kc = 0; kc < nk; ++kc) {
          if (!tc::mbar_wait(&ctl->mma_full[s], ph, abort, err, 13)) return;
          tc::fence_after_sync();
          const uint32_t a_hi = tc::smem_u32(mma + (size_t)s * 4 * GR_TILE), a_lo = a_hi + GR_TILE;
          const uint32_t b_hi = a_hi + 2 * GR_TILE, b_lo = a_hi + 3 * GR_TILE;
#pragma unroll
          for (int k8 = 0; k8 < 4; ++k8) {
            const uint32_t off = k8 * 32;
            const uint64_t dah = tc::sdesc_k_sw128(a_hi + off), dal = tc::sdesc_k_sw128(a_lo + off);
            const uint64_t dbh = tc::sdesc_k_sw128(b_hi + off), dbl = tc::sdesc_k_sw128(b_lo + off);
            tc::mma_tf32(d, dah, dbh, idesc, (kc | k8) != 0);
            tc::mma_tf32(d, dah, dbl, idesc, 1);
            tc::mma_tf32(d, dal, dbh, idesc, 1);
          }
          tc::mma_commit(&ctl->mma_empty[s]);
          if (++s == GR_MMA) {
            s = 0;
            ph ^= 1;
          }
        }
        tc::mma_commit(&ctl->tfull[acc]);
        acc ^= 1;
        if (acc == 0) aph ^= 1;
      }
    }
  } else if (warp < 2 + GR_CONV_WARPS) {
    const int t = threadIdx.x - 64;   // 0..127
    int rs = 0, ms = 0;
    uint32_t rph = 0, mph = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int sl, b, nt, mt;
      unit(u, sl, b, nt, mt);
      const int nk = stages_of(sl);
      bool ok = true;
      for (int kc = 0; kc < nk; ++kc) {
        if (!__all_sync(FULL, tc::mbar_wait(&ctl->raw_full[rs], rph, abort, err, 14)) ||
            !__all_sync(FULL, tc::mbar_wait(&ctl->mma_empty[ms], mph ^ 1, abort, err, 14))) {
          ok = false;
          break;
        }
        const float* ra = reinterpret_cast<const float*>(raw + (size_t)rs * 2 * GR_TILE);
        float* m4 = reinterpret_cast<float*>(mma + (size_t)ms * 4 * GR_TILE);
        convert_tile(ra, G.a_kmajor, 128, m4, m4 + GR_TILE / 4, t);
        convert_tile(ra + GR_TILE / 4, G.b_kmajor, G.BN, m4 + 2 * GR_TILE / 4, m4 + 3 * GR_TILE / 4, t);
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(&ctl->raw_empty[rs]);
          tc::mbar_arrive(&ctl->mma_full[ms]);
        }
        if (++rs == GR_RAW) {
          rs = 0;
          rph ^= 1;
        }
        if (++ms == GR_MMA) {
          ms = 0;
          mph ^= 1;
        }
      }
      if (!ok) break;
    }
  } else {
    const int quarter = warp & 3;
    float* stg = stg_all + (warp - 2 - GR_CONV_WARPS) * GR_STG;
    int acc = 0;
    uint32_t aph = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int sl, b, nt, mt;
      unit(u, sl, b, nt, mt);
      if (!__all_sync(FULL, tc::mbar_wait(&ctl->tfull[acc], aph, abort, err, 15))) break;
      tc::fence_after_sync();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * 128);
      const int64_t row0 = (int64_t)mt * 128 + quarter * 32;
      float* outp = G.out + sl * G.out_stride + b * G.c_boff;
      for (int cc = 0; cc < G.BN; cc += 32) {
        uint32_t v[32];
        tc::tmem_ld32(taddr + cc, v);
        tc::tmem_wait_ld();
        const int64_t col0 = (int64_t)nt * G.BN + cc;
        if (col0 >= G.N) continue;   // warp-uniform
#pragma unroll
        for (int j = 0; j < 32; ++j) stg[lane * 33 + j] = __uint_as_float(v[j]);
        __syncwarp();
        // 4 rows x 32 columns per step: lane -> (row it * 4 + lane / 8, columns 4 (lane % 8) ..)
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int r = it * 4 + (lane >> 3), c = (lane & 7) * 4;
          const int64_t row = row0 + r, col = col0 + c;
          if (row >= G.M) continue;
          float x[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) x[e] = stg[r * 33 + c + e] + ((G.bias && col + e < G.N) ? G.bias[col + e] : 0.f);
          float* dst = outp + row * G.ld + col;
          if (G.vec && col + 4 <= G.N) {
            float4 o = make_float4(x[0], x[1], x[2], x[3]);
            if (G.accumulate) {
              const float4 p = *reinterpret_cast<const float4*>(dst);
              o.x += p.x;
              o.y += p.y;
              o.z += p.z;
              o.w += p.w;
            }
            *reinterpret_cast<float4*>(dst) = o;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (col + e < G.N) dst[e] = G.accumulate ? dst[e] + x[e] : x[e];
          }
        }
        __syncwarp();
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ctl->tempty[acc]);
      acc ^= 1;
      if (acc == 0) aph ^= 1;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem_base, 256);
  }
}

// Operand element (r, k) at base[r sr + k sk]; rows x K.  K-major (sk == 1):
// box 32 k x box_rows, 128-byte swizzle.  Row-contiguous (sr == 1): box
// box_rows x 32 k, no swizzle.
cudaError_t make_operand_map(CUtensorMap* map, const float* base, int64_t rows, int64_t K, int64_t sr, int64_t sk,
                             uint32_t box_rows) {
  if (sk == 1) return make_tmap_f32_2d(map, base, (uint64_t)K, (uint64_t)rows, (uint64_t)sr, 32, box_rows, true);
  return make_tmap_f32_2d(map, base, (uint64_t)rows, (uint64_t)K, (uint64_t)sk, box_rows, 32, false);
}

bool operand_ok(const float* base, int64_t rows, int64_t K, int64_t sr, int64_t sk, int box_rows) {
  if (rows >= (1ll << 31) || K >= (1ll << 31)) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  if (sk == 1) return sr % 4 == 0 && sr >= K && K >= 32 && rows >= box_rows;
  if (sr == 1) return sk % 4 == 0 && sk >= rows && rows >= box_rows && K >= 32;
  return false;
}

}  // namespace

int gemm_raw_bn(int64_t N) { return N >= 128 ? 128 : (int)((N + 15) / 16 * 16); }

bool gemm_raw_supported(const float* A, int64_t sai, int64_t sak, const float* B, int64_t sbk, int64_t sbj,
                        int64_t M, int64_t N, int64_t K) {
  const int BN = gemm_raw_bn(N);
  if (M < 128 || N < 16 || (N < 128 && N % 16) || K < 32 || M >= (1ll << 31) || N >= (1ll << 31)) return false;
  return operand_ok(A, M, K, sai, sak, 128) && operand_ok(B, N, K, sbj, sbk, BN);
}

cudaError_t launch_gemm_raw(const float* A, int64_t sai, int64_t sak, const float* B, int64_t sbk, int64_t sbj,
                            int64_t M, int64_t N, int64_t K, int S, int kq_slice, float* out, int64_t out_stride,
                            int64_t ld, const float* bias, bool accumulate, int* err, cudaStream_t s, int batch,
                            int64_t a_rows, int64_t b_rows, int64_t c_boff) {
  GrArgs G{};
  G.M = M;
  G.N = N;
  G.K = K;
  G.BN = gemm_raw_bn(N);
  G.batch = batch;
  G.a_boff = (int)M;
  G.b_boff = (int)N;
  G.c_boff = c_boff;
  if (batch > 1 && (M % 128 != 0 || N % G.BN != 0)) return cudaErrorInvalidValue;   // whole tiles per batch
  if (a_rows < (int64_t)batch * M) a_rows = (int64_t)batch * M;
  if (b_rows < (int64_t)batch * N) b_rows = (int64_t)batch * N;
  G.a_kmajor = sak == 1;
  G.b_kmajor = sbk == 1;
  G.m_tiles = (int)((M + 127) / 128);
  G.n_tiles = (int)((N + G.BN - 1) / G.BN);
  G.S = S;
  G.kq_slice = kq_slice;
  G.out = out;
  G.out_stride = out_stride;
  G.ld = ld;
  G.bias = bias;
  G.accumulate = accumulate ? 1 : 0;
  G.vec = (ld % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0) && (out_stride % 4 == 0) &&
          (c_boff % 4 == 0);
  G.err = err;
  CUtensorMap ta, tb;
  cudaError_t e;
  if ((e = make_operand_map(&ta, A, a_rows, K, sai, sak, 128)) != cudaSuccess) return e;
  if ((e = make_operand_map(&tb, B, b_rows, K, sbj, sbk, (uint32_t)G.BN)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(gemm_raw_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GR_SMEM)) !=
      cudaSuccess)
    return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int units = G.m_tiles * G.n_tiles * batch * S;
  gemm_raw_tc_kernel<<<units < sms ? units : sms, GR_THREADS, GR_SMEM, s>>>(ta, tb, G);
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
