// Value table in page-locked host memory (the host tier: memory.py:180-183
// with host_pool.fetch, host_pool.py:206-220 and HostPool.gather :117-127).
//
// The reference removes duplicate slots on the device (jnp.unique), copies
// the distinct rows in through a host callback and expands them
// (rows[inv]).  Here the GPU reads the host rows itself, over PCIe / C2C,
// from a table mapped into its address space:
//   1. routing as in the device-table forward (stage 2 writes slots and
//      weights, no gather);
//   2. the read slots are sorted with the stable radix sort of the row
//      gradients: distinct rows ascending, and for every fetch its row;
//   3. one warp per distinct row copies it from host memory into a staging
//      buffer in HBM (16-byte loads, four rows in flight per warp), so each
//      distinct row crosses the host link once per call;
//   4. the weighted mix reads the staged rows with the arithmetic of the
//      device-table gather (per-head fma over the k rows in rank order, heads
//      summed in order): outputs are bit-identical to memlayer_pool_forward
//      on the same table.
#include "combine.cuh"
#include "host_table.cuh"

namespace ml {

namespace {

// Distinct read slots of a small call (F <= TABLE_SMALL_F fetches) in one
// CTA: (read slot, fetch) pairs bitonic-sorted in shared memory (the fetch
// index makes the order stable), segment heads counted with a block scan.
// Writes what the radix pipeline writes: uniq[u] ascending, *n_seg and
// inv[fetch] = u.
__global__ void __launch_bounds__(1024) table_unique_small_kernel(const int* __restrict__ slots, int F, int64_t N,
                                                                  int64_t kadd, int* __restrict__ uniq,
                                                                  int* __restrict__ n_seg, int* __restrict__ inv) {
  __shared__ unsigned long long kv[TABLE_SMALL_F];
  __shared__ int wsum[32];
  int P2 = 1;
  while (P2 < F) P2 <<= 1;
  for (int i = threadIdx.x; i < P2; i += blockDim.x) {
    unsigned long long v = ~0ull;
    if (i < F) {
      const int64_t s = slots[i];
      const int64_t key = kadd > 0 ? (s + kadd) % N : s;   // the read slot (memory.py:179)
      v = ((unsigned long long)key << 32) | (unsigned)i;
    }
    kv[i] = v;
  }
  __syncthreads();
  for (int size = 2; size <= P2; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P2; i += blockDim.x) {
        const int l = i ^ stride;
        if (l > i) {
          const unsigned long long a = kv[i], b = kv[l];
          const bool up = (i & size) == 0;
          if ((a > b) == up) {
            kv[i] = b;
            kv[l] = a;
          }
        }
      }
      __syncthreads();
    }
  // each thread: 4 consecutive sorted entries; exclusive scan of the heads
  constexpr int PER = TABLE_SMALL_F / 1024;
  const int i0 = threadIdx.x * PER;
  int head[PER], cnt = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = i0 + j;
    head[j] = (i < F) && (i == 0 || (kv[i] >> 32) != (kv[i - 1] >> 32));
    cnt += head[j];
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(FULL, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(FULL, w, o);
      if (lane >= o) w += y;
    }
    wsum[lane] = w;   // inclusive over warps
  }
  __syncthreads();
  int run = incl - cnt + (warp > 0 ? wsum[warp - 1] : 0);   // heads before this thread's entries
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = i0 + j;
    if (i >= F) break;
    run += head[j];
    const int u = run - 1;
    if (head[j]) uniq[u] = (int)(kv[i] >> 32);
    inv[(int)(kv[i] & 0xffffffffu)] = u;
  }
  if (threadIdx.x == blockDim.x - 1) *n_seg = wsum[31];
}

// Rows of row_bytes (a multiple of 16) as uint4 words; ROWS rows per warp
// iteration so that several loads are in flight on the host link.
template <int ROWS>
__global__ void __launch_bounds__(256) table_fetch16_kernel(const uint4* __restrict__ table, int64_t row_words,
                                                            const int* __restrict__ uniq, const int* __restrict__ n_seg,
                                                            int64_t n_rows, uint4* __restrict__ staging,
                                                            int* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  const int64_t U = *n_seg;
  const int64_t warps = (int64_t)gridDim.x * 8;
  for (int64_t u0 = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * ROWS; u0 < U; u0 += warps * ROWS) {
    int64_t row[ROWS];
#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
      row[j] = u0 + j < U ? uniq[u0 + j] : -1;
      if (row[j] >= n_rows) {   // only a bug upstream can cause this
        if (lane == 0) atomicCAS(err, 0, 25);
        row[j] = -1;
      }
    }
    for (int64_t w0 = 0; w0 < row_words; w0 += 32) {
      const int64_t w = w0 + lane;
      uint4 x[ROWS];
#pragma unroll
      for (int j = 0; j < ROWS; ++j)
        if (row[j] >= 0 && w < row_words) x[j] = table[row[j] * row_words + w];
#pragma unroll
      for (int j = 0; j < ROWS; ++j)
        if (row[j] >= 0 && w < row_words) staging[(u0 + j) * row_words + w] = x[j];
    }
  }
}

// Rows of any size, element by element (4-byte or 2-byte elements).
template <typename T>
__global__ void __launch_bounds__(256) table_fetch_kernel(const T* __restrict__ table, int d,
                                                          const int* __restrict__ uniq, const int* __restrict__ n_seg,
                                                          int64_t n_rows, T* __restrict__ staging,
                                                          int* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  const int64_t U = *n_seg;
  for (int64_t u = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); u < U; u += (int64_t)gridDim.x * 8) {
    const int64_t row = uniq[u];
    if (row >= n_rows) {
      if (lane == 0) atomicCAS(err, 0, 25);
      continue;
    }
    for (int e = lane; e < d; e += 32) staging[u * d + e] = table[row * d + e];
  }
}

// One CTA per token, one warp per head: out[m] = sum_h sum_r w * staged[inv],
// in the order of combine_gather_kernel.
template <typename VT, int VEC, int CH>
__global__ void __launch_bounds__(1024) table_mix_kernel(Dims D, const VT* __restrict__ staging,
                                                         const int* __restrict__ inv, const float* __restrict__ weights,
                                                         float* __restrict__ out) {
  extern __shared__ float red[];   // [H][d]
  const int64_t m = blockIdx.x;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k = D.k, d = D.d;
  const int64_t ow = (m * D.H + h) * k;
  const int u_l = lane < k ? inv[ow + lane] : -1;
  const float w_l = lane < k ? weights[ow + lane] : 0.f;
  float acc[CH][VEC];
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[c][v] = 0.f;
  const int groups = d / VEC;
#pragma unroll 4
  for (int r = 0; r < k; ++r) {
    const int u = __shfl_sync(FULL, u_l, r);
    const float wr = __shfl_sync(FULL, w_l, r);
    if (u < 0) continue;
    const VT* base = staging + (int64_t)u * d;
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
    out[m * d + i] = o;
  }
}

inline int ch_for(int groups) {
  int ch = (groups + 31) / 32;
  return ch <= 1 ? 1 : ch <= 2 ? 2 : ch <= 4 ? 4 : ch <= 8 ? 8 : -1;
}

template <typename VT, int VEC>
cudaError_t mix_ch(const Dims& D, const VT* staging, const int* inv, const float* weights, float* out,
                   cudaStream_t s) {
  const dim3 grid((unsigned)D.M), block(32 * D.H);
  const size_t smem = (size_t)D.H * D.d * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e;
#define ML_ATTR(CHV)                                                                                        \
  e = cudaFuncSetAttribute(table_mix_kernel<VT, VEC, CHV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
    switch (ch_for(D.d / VEC)) {
      case 1: ML_ATTR(1); break;
      case 2: ML_ATTR(2); break;
      case 4: ML_ATTR(4); break;
      case 8: ML_ATTR(8); break;
      default: return cudaErrorInvalidValue;
    }
#undef ML_ATTR
    if (e != cudaSuccess) return e;
  }
  switch (ch_for(D.d / VEC)) {
    case 1: table_mix_kernel<VT, VEC, 1><<<grid, block, smem, s>>>(D, staging, inv, weights, out); break;
    case 2: table_mix_kernel<VT, VEC, 2><<<grid, block, smem, s>>>(D, staging, inv, weights, out); break;
    case 4: table_mix_kernel<VT, VEC, 4><<<grid, block, smem, s>>>(D, staging, inv, weights, out); break;
    case 8: table_mix_kernel<VT, VEC, 8><<<grid, block, smem, s>>>(D, staging, inv, weights, out); break;
    default: return cudaErrorInvalidValue;
  }
  count_launch();
  return cudaGetLastError();
}

}  // namespace

int64_t table_elem_bytes(int vdtype) { return vdtype == MEMLAYER_F32 ? 4 : 2; }

cudaError_t launch_table_unique_small(const int* slots, int F, int64_t N, int64_t kadd, int* uniq, int* n_seg,
                                      int* inv, cudaStream_t s) {
  if (F < 1 || F > TABLE_SMALL_F) return cudaErrorInvalidValue;
  table_unique_small_kernel<<<1, 1024, 0, s>>>(slots, F, N, kadd, uniq, n_seg, inv);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_table_fetch(const Dims& D, const void* table, const int* uniq, const int* n_seg, int64_t cap,
                               void* staging, int* err, cudaStream_t s) {
  if (cap == 0) return cudaSuccess;
  const int64_t row_bytes = (int64_t)D.d * table_elem_bytes(D.vdtype);
  constexpr int ROWS = 4;
  if (row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(table) & 15) == 0) {
    const int64_t warps = (cap + ROWS - 1) / ROWS;
    const int64_t b = (warps + 7) / 8;
    table_fetch16_kernel<ROWS><<<(unsigned)(b < 148 * 16 ? b : 148 * 16), 256, 0, s>>>(
        (const uint4*)table, row_bytes / 16, uniq, n_seg, D.N, (uint4*)staging, err);
  } else {
    const int64_t b = (cap + 7) / 8;
    const unsigned grid = (unsigned)(b < 148 * 16 ? b : 148 * 16);
    if (D.vdtype == MEMLAYER_F32)
      table_fetch_kernel<float><<<grid, 256, 0, s>>>((const float*)table, D.d, uniq, n_seg, D.N, (float*)staging, err);
    else
      table_fetch_kernel<uint16_t><<<grid, 256, 0, s>>>((const uint16_t*)table, D.d, uniq, n_seg, D.N,
                                                        (uint16_t*)staging, err);
  }
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_table_mix(const Dims& D, const void* staging, const int* inv, const float* weights, float* out,
                             cudaStream_t s) {
  if (D.M == 0) return cudaSuccess;
  if (D.vdtype == MEMLAYER_F16) return mix_ch<__half, 8>(D, (const __half*)staging, inv, weights, out, s);
  if (D.vdtype == MEMLAYER_BF16)
    return mix_ch<__nv_bfloat16, 8>(D, (const __nv_bfloat16*)staging, inv, weights, out, s);
  if (D.d % 4 == 0) return mix_ch<float, 4>(D, (const float*)staging, inv, weights, out, s);
  return mix_ch<float, 1>(D, (const float*)staging, inv, weights, out, s);
}

}  // namespace ml
