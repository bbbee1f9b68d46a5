// Projection GEMMs of the memory-layer block on the tensor cores
// (model.py:110-111 router Dense, model.py:118 mem_gate Dense + silu,
// model.py:119 mem_out Dense), float32-faithful through the same 3xTF32
// split as the score kernel: C = A B^T with A [M, K] and B [N, K] both
// K-major, given as tf32 hi / lo halves.
//
// Epilogues (8 warps; TMEM lane = output row; the two warps of a lane
// quarter take the two 128-column halves of the 256-column tile):
//   ROUTER_GATE  columns [0, NR): q = acc + b_router, split per query half
//                into q_len = |q_half| / sqrt(half) and the unit half
//                q_hat = q * rsqrt(|q_half|^2 + 1e-6) (memory.py:136-138),
//                written as tf32 hi / lo in codebook-major [H*2][M][half]
//                for the score kernel (and as float32 [M,H,2,half] when the
//                aux queries are requested);
//                columns [NR, NR + d): gate = silu(acc + b_gate).
//   BIAS         y = acc + bias.
#include "backbone.cuh"
#include "tc_pipeline.cuh"

namespace ml {

namespace {

constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int BN_MAX = 256;

enum { EPI_ROUTER_GATE = 0, EPI_BIAS = 1, EPI_GELU = 2 };

struct ProjArgs {
  int64_t M;
  int N, K;
  const float* bias;   // [N] or nullptr
  // ROUTER_GATE
  int NR;              // router columns H * d_key
  int half;            // d_key / 2 (32, 64 or 128)
  int hc_count;        // H * 2
  float* q_hi;         // [hc][M][half]
  float* q_lo;
  float* qlen;         // [M][hc]
  float* qn;           // [M][hc][half] or nullptr
  float* gate;         // [M][N - NR]
  // BIAS / GELU
  float* out;          // [M][N]
  int bias_smem;       // bias staged in shared memory (N <= BIAS_SMEM_MAX); else read from global
  // split inner dimension (BIAS epilogue): `slices` independent products,
  // slice s reading A rows [s m_pad, +M) and B rows [s n_pad, +N) and
  // writing out + s out_stride
  int slices = 1;
  int64_t m_pad = 0, n_pad = 0, out_stride = 0;
  int accumulate = 0;  // BIAS: out += acc + bias (read-modify-write of the output)
};

constexpr int BIAS_SMEM_MAX = 4096;

// Per-warp staging tile for coalesced epilogue stores: 32 rows x 16 floats,
// row stride 20 floats (conflict-free float4 writes by row-owning lanes).
constexpr int STG_LD = 20;
constexpr int STG_FLOATS = 32 * STG_LD;

// The 32 lanes of a warp each hold 16 consecutive values of their own row
// (row = row0 + lane).  Written through the staging tile so that every
// store instruction covers 8 rows x 64 contiguous bytes instead of 32 rows x
// 16 bytes.  dst0 points at row0's first column; rows >= nrows are skipped;
// with add the destination's values are added (same coalesced pattern).
__device__ __forceinline__ void store16_rows(float* stg, const float (&v)[16], float* dst0, int64_t stride,
                                             int64_t nrows, int lane, bool add = false) {
#pragma unroll
  for (int j = 0; j < 16; j += 4)
    *reinterpret_cast<float4*>(stg + lane * STG_LD + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane >> 2), c = (lane & 3) * 4;
    float4 x = *reinterpret_cast<const float4*>(stg + r * STG_LD + c);
    if (r < nrows) {
      float4* d4 = reinterpret_cast<float4*>(dst0 + r * stride + c);
      if (add) {
        const float4 o = *d4;
        x.x += o.x;
        x.y += o.y;
        x.z += o.z;
        x.w += o.w;
      }
      *d4 = x;
    }
  }
  __syncwarp();
}

// One query half of the warp's 32 rows: q = acc + b_router, q_len and the
// unit half as tf32 hi / lo (+ float32 when requested), memory.py:136-138.
// TMEM is read in pieces of up to 64 columns with one wait each: once for
// |q|^2, once to write.
template <int HALF>
__device__ __forceinline__ void router_half(const ProjArgs& G, uint32_t taddr, int ns, int64_t row0, int lane,
                                            const float* sbias, float* stg) {
  constexpr int P = HALF < 64 ? HALF : 64;
  const int64_t row = row0 + lane;
  const bool rok = row < G.M;
  const int64_t nrows = G.M - row0;
  float ss = 0.f;
#pragma unroll
  for (int p0 = 0; p0 < HALF; p0 += P) {
    uint32_t r[P];
#pragma unroll
    for (int c = 0; c < P; c += 32) tc::tmem_ld32(taddr + p0 + c, *reinterpret_cast<uint32_t(*)[32]>(&r[c]));
    tc::tmem_wait_ld();
#pragma unroll
    for (int t = 0; t < P; ++t) {
      const float q = __uint_as_float(r[t]) + sbias[ns + p0 + t];
      ss = fmaf(q, q, ss);
    }
  }
  const int hc = ns / HALF;                 // head * 2 + half
  const float tt = ss + 1e-6f;
  const float rn = 1.0f / sqrtf(tt);
  if (rok) G.qlen[row * G.hc_count + hc] = sqrtf(tt) / sqrtf((float)HALF);
  // row0's first element in each destination
  float* dhi = G.q_hi ? G.q_hi + ((int64_t)hc * G.M + row0) * HALF : nullptr;
  float* dlo = G.q_hi ? G.q_lo + ((int64_t)hc * G.M + row0) * HALF : nullptr;
  float* dqn = G.qn ? G.qn + (row0 * G.hc_count + hc) * HALF : nullptr;
#pragma unroll
  for (int p0 = 0; p0 < HALF; p0 += P) {
    uint32_t r[P];
#pragma unroll
    for (int c = 0; c < P; c += 32) tc::tmem_ld32(taddr + p0 + c, *reinterpret_cast<uint32_t(*)[32]>(&r[c]));
    tc::tmem_wait_ld();
#pragma unroll
    for (int t = 0; t < P; t += 16) {
      float u[16], h[16], l[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        u[j] = (__uint_as_float(r[t + j]) + sbias[ns + p0 + t + j]) * rn;
        h[j] = tc::to_tf32(u[j]);
        l[j] = tc::to_tf32(u[j] - h[j]);
      }
      if (dhi) {
        store16_rows(stg, h, dhi + p0 + t, HALF, nrows, lane);
        store16_rows(stg, l, dlo + p0 + t, HALF, nrows, lane);
      }
      if (dqn) store16_rows(stg, u, dqn + p0 + t, (int64_t)G.hc_count * HALF, nrows, lane);
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    proj_gemm_tc_kernel(const __grid_constant__ CUtensorMap tA_hi, const __grid_constant__ CUtensorMap tA_lo,
                        const __grid_constant__ CUtensorMap tB_hi, const __grid_constant__ CUtensorMap tB_lo,
                        ProjArgs G, tc::PipeShape P, int m_tiles, int n_tiles, int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  tc::PipeCtl* ctl = reinterpret_cast<tc::PipeCtl*>(smem);
  uint8_t* tiles = smem + 1024;
  // bias vector staged once per CTA (read as a broadcast by every row)
  float* sbias = reinterpret_cast<float*>(tiles + (size_t)P.stages * P.stage_bytes);
  const int nb_s = G.bias_smem ? G.N : 0;   // wide GEMMs (the tied logits) read the bias from global
  for (int i = threadIdx.x; i < nb_s; i += blockDim.x) sbias[i] = G.bias ? G.bias[i] : 0.f;
  volatile int* abort = &ctl->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // per-epilogue-warp staging tiles after the bias vector
  float* stg = sbias + ((nb_s + 255) / 256) * 256 + (warp >= 2 ? (warp - 2) * STG_FLOATS : 0);
  const int per_slice = m_tiles * n_tiles;
  const int units = per_slice * G.slices;
  // unit u = (slice, n tile, m tile), m fastest: neighbouring CTAs share the B tile
  auto coords = [&](int u, int& arow, int& brow0, int& nch) {
    const int sl = u / per_slice, v = u - sl * per_slice;
    const int nt = v / m_tiles, mt = v - nt * m_tiles;
    arow = (int)(sl * G.m_pad) + mt * tc::PIPE_M;
    brow0 = (int)(sl * G.n_pad) + nt * P.BN;
    nch = 1;
  };
  const uint32_t tmem_base = tc::pipe_init(ctl, P, EPI_WARPS);

  if (warp == 0) {
    if (lane == 0) tc::pipe_produce(ctl, P, tiles, units, &tA_hi, &tA_lo, &tB_hi, &tB_lo, coords, err);
  } else if (warp == 1) {
    if (lane == 0) tc::pipe_mma(ctl, P, tiles, units, tmem_base, coords, err);
  } else {
    const int quarter = warp & 3;
    const int hf = (warp - 2) >> 2;
    const int half_bn = P.BN >> 1;
    int acc = 0;
    uint32_t aph = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int sl = u / per_slice, v = u - sl * per_slice;
      const int nt = v / m_tiles, mt = v - nt * m_tiles;
      float* outp = G.out ? G.out + sl * G.out_stride : nullptr;
      const int64_t row0 = (int64_t)mt * tc::PIPE_M + quarter * 32;   // the warp's first row
      const int64_t row = row0 + lane;
      const bool rok = row < G.M;
      if (!__all_sync(FULL, tc::mbar_wait(&ctl->tfull[acc], aph, abort, err, 14))) break;
      tc::fence_after_sync();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * tc::PIPE_ACC_STRIDE);
      const int c0 = hf * half_bn;                 // first tile column of this warp
      const int n0 = nt * P.BN + c0;               // first output column of this warp
      const int ncols = min(half_bn, G.N - n0);    // valid columns of this warp

      if (EPI == EPI_ROUTER_GATE && n0 < G.NR) {
        // router columns: whole query halves (half divides 128, NR % 128 == 0)
        for (int seg = 0; seg < ncols; seg += G.half) {
          if (G.half == 128)
            router_half<128>(G, taddr + c0 + seg, n0 + seg, row0, lane, sbias, stg);
          else if (G.half == 64)
            router_half<64>(G, taddr + c0 + seg, n0 + seg, row0, lane, sbias, stg);
          else
            router_half<32>(G, taddr + c0 + seg, n0 + seg, row0, lane, sbias, stg);
        }
      } else {
        // gate columns (silu) or plain bias columns, 32 at a time
        const int ld = EPI == EPI_ROUTER_GATE ? G.N - G.NR : G.N;
        float* dst0 = EPI == EPI_ROUTER_GATE ? G.gate + row0 * ld + (n0 - G.NR) : outp + row0 * ld + n0;
        float* dst = dst0 + (int64_t)lane * ld;
        const bool vec = (ld & 3) == 0 && (n0 & 3) == 0;
        for (int cc = 0; cc < ncols; cc += 32) {
          uint32_t r[32];
          tc::tmem_ld32(taddr + c0 + cc, r);
          tc::tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int n = n0 + cc + t;
            float x = __uint_as_float(r[t]) +
                      (cc + t < ncols ? (G.bias_smem ? sbias[n] : (G.bias ? __ldg(G.bias + n) : 0.f)) : 0.f);
            if (EPI == EPI_ROUTER_GATE) x = x / (1.0f + expf(-x));      // model.py:118 silu
            if (EPI == EPI_GELU)                                         // model.py:104 nn.gelu (tanh form)
              x = x * (0.5f * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * (x * x * x)))));
            v[t] = x;
          }
#pragma unroll
          for (int g = 0; g < 32; g += 16) {
            if (vec && cc + g + 16 <= ncols) {
              store16_rows(stg, *reinterpret_cast<float(*)[16]>(&v[g]), dst0 + cc + g, ld, G.M - row0, lane,
                           G.accumulate != 0);
            } else if (rok) {
#pragma unroll
              for (int t = 0; t < 16; ++t)
                if (cc + g + t < ncols) dst[cc + g + t] = G.accumulate ? dst[cc + g + t] + v[g + t] : v[g + t];
            }
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ctl->tempty[acc]);
      acc ^= 1;
      if (acc == 0) aph ^= 1;
    }
  }
  tc::pipe_finish(ctl, tmem_base);
}

// The router / gate GEMM keeps 256-column tiles (each warp's 128 columns
// hold whole query halves); narrow GEMMs use 128-column tiles so that more
// CTAs share the work.
inline int bn_for(int EPI, int N) {
  const int cap = EPI == EPI_ROUTER_GATE ? BN_MAX : (N > 256 ? BN_MAX : 128);
  return N >= cap ? cap : ((N + 15) / 16) * 16;
}

template <int EPI>
cudaError_t launch_proj(const ProjArgs& G, const float* a_hi, const float* a_lo, const float* b_hi,
                        const float* b_lo, int* err, cudaStream_t s) {
  if (G.M == 0) return cudaSuccess;
  const int BN = bn_for(EPI, G.N);
  // bias vector (padded to 256 floats) + one staging tile per epilogue warp
  const uint32_t nb_s = G.bias_smem ? (uint32_t)G.N : 0u;
  const uint32_t bias_bytes = (((nb_s + 255) / 256 * 256 * 4 + EPI_WARPS * STG_FLOATS * 4) + 1023) / 1024 * 1024;
  // 32-element K stages (128-byte swizzle).  16-element stages (64-byte
  // swizzle, twice the ring depth) measured the same: the epilogue, not
  // operand latency, bounds this GEMM.
  constexpr int BK = 32;
  tc::PipeShape P = tc::pipe_shape(BN, G.K, bias_bytes, BK);
  if (P.stages < 2) return cudaErrorInvalidConfiguration;
  CUtensorMap m[4];
  cudaError_t e;
  const uint64_t a_rows = G.slices > 1 ? (uint64_t)(G.slices * G.m_pad) : (uint64_t)G.M;
  const uint64_t b_rows = G.slices > 1 ? (uint64_t)(G.slices * G.n_pad) : (uint64_t)G.N;
  if ((e = make_tmap_f32(&m[0], a_hi, a_rows, G.K, tc::PIPE_M, BK)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[1], a_lo, a_rows, G.K, tc::PIPE_M, BK)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[2], b_hi, b_rows, G.K, BN, BK)) != cudaSuccess) return e;
  if ((e = make_tmap_f32(&m[3], b_lo, b_rows, G.K, BN, BK)) != cudaSuccess) return e;
  const size_t smem = 2048 + (size_t)P.stages * P.stage_bytes + bias_bytes;
  auto kern = proj_gemm_tc_kernel<EPI>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
    return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int m_tiles = (int)((G.M + tc::PIPE_M - 1) / tc::PIPE_M), n_tiles = (G.N + BN - 1) / BN;
  const int units = m_tiles * n_tiles * G.slices;
  kern<<<units < sms ? units : sms, THREADS, smem, s>>>(m[0], m[1], m[2], m[3], G, P, m_tiles, n_tiles, err);
  count_launch();
  return cudaGetLastError();
}

// ---- operand preparation ------------------------------------------------------
// x -> (rna_tf32(x), rna_tf32(x - hi)), elementwise.
__global__ void split_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ hi, float* __restrict__ lo) {
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
    float4 h, l;
    h.x = tc::to_tf32(v.x); l.x = tc::to_tf32(v.x - h.x);
    h.y = tc::to_tf32(v.y); l.y = tc::to_tf32(v.y - h.y);
    h.z = tc::to_tf32(v.z); l.z = tc::to_tf32(v.z - h.z);
    h.w = tc::to_tf32(v.w); l.w = tc::to_tf32(v.w - h.w);
    reinterpret_cast<float4*>(hi)[i] = h;
    reinterpret_cast<float4*>(lo)[i] = l;
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    hi[i] = tc::to_tf32(v);
    lo[i] = tc::to_tf32(v - hi[i]);
  }
}

// W [K, N] row-major (a Dense kernel) -> rows [row0, row0 + N) of a K-major
// [*, K] matrix, split into tf32 hi / lo.  32 x 32 tiles through shared memory.
__global__ void transpose_split_kernel(const float* __restrict__ W, int K, int N, float* __restrict__ hi,
                                       float* __restrict__ lo, int row0) {
  __shared__ float t[32][33];
  const int n_base = blockIdx.x * 32, k_base = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int k = k_base + i, n = n_base + threadIdx.x;
    t[i][threadIdx.x] = (k < K && n < N) ? W[(int64_t)k * N + n] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int n = n_base + i, k = k_base + threadIdx.x;
    if (n < N && k < K) {
      const float v = t[threadIdx.x][i];
      const float h = tc::to_tf32(v);
      hi[(int64_t)(row0 + n) * K + k] = h;
      lo[(int64_t)(row0 + n) * K + k] = tc::to_tf32(v - h);
    }
  }
}

__global__ void concat_bias_kernel(const float* __restrict__ a, int na, const float* __restrict__ b, int nb,
                                   float* __restrict__ out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < na + nb; i += gridDim.x * blockDim.x)
    out[i] = i < na ? (a ? a[i] : 0.f) : (b ? b[i - na] : 0.f);
}

}  // namespace

bool proj_tc_supported(const Dims& D) {
  const int NR = D.H * D.dk;
  // NR + d >= 256: 256-column tiles, so each epilogue warp's 128 columns are
  // all router columns (whole query halves, NR % 128 == 0) or all gate columns
  return D.M >= tc::PIPE_M && D.dm % tc::PIPE_K == 0 && D.d % tc::PIPE_K == 0 && NR % 128 == 0 &&
         NR + D.d >= BN_MAX &&
         (NR + D.d) * 4 <= 16384 && D.dm * 4 <= 16384 &&
         (D.half == 32 || D.half == 64 || D.half == 128) && D.d % 16 == 0 && (D.dm >= BN_MAX || D.dm % 16 == 0) &&
         D.M < (1ll << 31);
}

cudaError_t launch_split(const float* x, int64_t n, float* hi, float* lo, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  int64_t blocks = (n / 4 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  split_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, n, hi, lo);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_transpose_split(const float* W, int K, int N, float* hi, float* lo, int row0, cudaStream_t s) {
  dim3 grid((N + 31) / 32, (K + 31) / 32), block(32, 8);
  transpose_split_kernel<<<grid, block, 0, s>>>(W, K, N, hi, lo, row0);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_concat_bias(const float* a, int na, const float* b, int nb, float* out, cudaStream_t s) {
  concat_bias_kernel<<<(na + nb + 255) / 256, 256, 0, s>>>(a, na, b, nb, out);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_router_gate_tc(const Dims& D, const Work& W, const float* bias_rg, float* qn_out,
                                  cudaStream_t s) {
  ProjArgs G{};
  G.M = D.M;
  G.NR = D.H * D.dk;
  G.N = G.NR + D.d;
  G.K = D.dm;
  G.bias = bias_rg;
  G.half = D.half;
  G.hc_count = D.H * 2;
  G.q_hi = W.q_hi;
  G.q_lo = W.q_lo;
  G.qlen = W.qlen;
  G.qn = qn_out;
  G.gate = W.gate;
  G.bias_smem = 1;
  return launch_proj<EPI_ROUTER_GATE>(G, W.h_hi, W.h_lo, W.wrg_hi, W.wrg_lo, W.err, s);
}

cudaError_t launch_out_tc(const Dims& D, const Work& W, const float* b_out, float* y, cudaStream_t s) {
  ProjArgs G{};
  G.M = D.M;
  G.N = D.dm;
  G.K = D.d;
  G.bias = b_out;
  G.out = y;
  G.bias_smem = G.N <= BIAS_SMEM_MAX;
  return launch_proj<EPI_BIAS>(G, W.memg_hi, W.memg_lo, W.wo_hi, W.wo_lo, W.err, s);
}

// ---- general Dense layers of the backbone -------------------------------------

int dense_tc_bn(int N) { return bn_for(EPI_BIAS, N); }

cudaError_t launch_dense_tc_sliced(const float* a_hi, const float* a_lo, int64_t M, int64_t m_pad, int K,
                                   const float* bt_hi, const float* bt_lo, int N, int64_t n_pad, int slices,
                                   float* C, int* err, cudaStream_t s) {
  ProjArgs G{};
  G.M = M;
  G.N = N;
  G.K = K;
  G.bias = nullptr;
  G.out = C;
  G.bias_smem = 0;
  G.slices = slices;
  G.m_pad = m_pad;
  G.n_pad = n_pad;
  G.out_stride = M * N;
  return launch_proj<EPI_BIAS>(G, a_hi, a_lo, bt_hi, bt_lo, err, s);
}

bool dense_tc_supported(int64_t M, int K, int N) {
  return M >= tc::PIPE_M && K % tc::PIPE_K == 0 && K >= tc::PIPE_K && N % 16 == 0 && N >= 16 &&
         M < (1ll << 31);
}

cudaError_t launch_dense_tc(const float* a_hi, const float* a_lo, int64_t M, int K, const float* bt_hi,
                            const float* bt_lo, int N, const float* bias, float* C, int act, int* err,
                            cudaStream_t s, bool accumulate) {
  ProjArgs G{};
  G.M = M;
  G.N = N;
  G.K = K;
  G.bias = bias;
  G.out = C;
  G.bias_smem = N <= BIAS_SMEM_MAX;
  G.accumulate = accumulate ? 1 : 0;
  if (accumulate && act != ACT_NONE) return cudaErrorInvalidValue;
  if (act == ACT_GELU) return launch_proj<EPI_GELU>(G, a_hi, a_lo, bt_hi, bt_lo, err, s);
  if (act != ACT_NONE) return cudaErrorInvalidValue;
  return launch_proj<EPI_BIAS>(G, a_hi, a_lo, bt_hi, bt_lo, err, s);
}

}  // namespace ml
