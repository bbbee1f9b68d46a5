// Fetched-row gradients and row-wise Adagrad on the touched rows
// (memory_pool_model/train.py:146-172 fetched_row_grads / _merge_rows,
// :378-383 global-norm clip, :396-399 row-wise Adagrad).
//
// A read out[m] = sum_f w_f V[s_f] gives dL/dV[s] = sum over the fetches f
// of slot s of w_f * g[m_f], g = dL/dout.  The fetches of all reads (memory
// layers sharing the pool) are numbered in concatenation order and
//   1. sorted by slot with a stable LSD radix sort of up to 10 bits per pass
//      (per-block digit counts, a per-digit scan, warp-stable scatter), so
//      each slot's fetches stay in fetch order and every sum below has a
//      fixed order;
//   2. cut into segments of equal slot (uniq = the segments' slots,
//      ascending, as jnp.unique returns them);
//   3. summed per segment by one warp per chunk of 64 sorted fetches: a
//      segment inside one chunk is written whole, a segment crossing chunk
//      boundaries leaves one partial per chunk; groups of 32 chunks lying
//      inside one segment are pre-added (one warp per group), and the
//      segment's first chunk adds its head chunks, the group sums and its
//      tail chunks in order -- so a slot fetched by hundreds of thousands of
//      fetches (Zipf-skewed routing) is spread over many warps, its final sum
//      is a few hundred rows long, and the result is still deterministic;
//   4. reduced to the squared norm of all row gradients (fixed order,
//      float64 partials) for the global-norm clip;
//   5. (Adagrad) one warp per touched row: g = scale * row,
//      acc[s] += mean(g^2), V[s] -= lr / (sqrt(acc[s]) + 1e-8) * g.
// g rows (8 KB per token at d = 256) are re-read from L2 per fetch; the
// per-fetch contributions are never materialised.
#include "common.cuh"
#include "rowgrad.cuh"

namespace ml {

namespace {

constexpr int RS_THREADS = 256;
constexpr int RS_ITEMS = 16;
constexpr int RS_TILE = RS_THREADS * RS_ITEMS;   // 4096 keys per sort block
constexpr int RS_WARP_ITEMS = RS_TILE / 8;        // 512 keys per warp
constexpr int SEG_TILE = 1024;                    // flags per scan block
constexpr int CHUNK = 64;                         // sorted fetches per row warp
constexpr int SPAN_GROUP = 32;                    // chunks per pre-added group of a long segment
constexpr int SQ_BLOCKS = 64;
constexpr int MAX_DIGITS = 1024;                 // radix digits per pass (<= 10 bits)
constexpr uint32_t DROPPED = 0x80000000u;        // fetch-id flag: out-of-range slot, contributes zero

// ---- 1. keys: slot of every fetch (an out-of-range id is recorded and its
// fetch is flagged to contribute nothing) ----
__global__ void rg_keys_kernel(RowGradK R, uint32_t* keys, uint32_t* vals, int* err) {
  const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= R.F) return;
  int r = 0;
  while (r + 1 < R.n_reads && f >= R.off[r + 1]) ++r;
  const int s = R.slots[r][f - R.off[r]];
  uint32_t key = R.kworld > 1 ? (uint32_t)((s % R.kworld) * R.kstride + s / R.kworld)
                 : R.kadd > 0 ? (uint32_t)(((int64_t)s + R.kadd) % R.Nslot) : (uint32_t)s;
  uint32_t val = (uint32_t)f;
  if (s < 0 || (int64_t)s >= R.Nslot) {   // only a caller bug can cause this: record it, the fetch adds nothing
    atomicCAS(err, 0, 23);
    key = (uint32_t)(R.N - 1);
    val |= DROPPED;
  }
  keys[f] = key;
  vals[f] = val;
}

// ---- 2. stable LSD radix sort ----
__global__ void __launch_bounds__(RS_THREADS) rs_hist_kernel(const uint32_t* keys, int64_t F, int shift,
                                                             int digits, int nblk, int* hist) {
  __shared__ int cnt[MAX_DIGITS];
  for (int i = threadIdx.x; i < digits; i += RS_THREADS) cnt[i] = 0;
  __syncthreads();
  const int64_t t0 = (int64_t)blockIdx.x * RS_TILE;
  const uint32_t mask = (uint32_t)digits - 1;
  for (int i = threadIdx.x; i < RS_TILE; i += RS_THREADS) {
    const int64_t e = t0 + i;
    if (e < F) atomicAdd(&cnt[(keys[e] >> shift) & mask], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < digits; i += RS_THREADS) hist[(int64_t)i * nblk + blockIdx.x] = cnt[i];
}

// Exclusive scan of n ints in place, one block of 1024 threads.
__global__ void __launch_bounds__(1024) scan_excl_kernel(int* a, int64_t n, int* total) {
  __shared__ int wsum[32];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int64_t per = (n + 1023) / 1024;
  const int64_t b = t * per, e = b + per < n ? b + per : n;
  int s = 0;
  for (int64_t i = b; i < e; ++i) s += a[i];
  // block exclusive scan of the per-thread sums
  int x = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[w] = x;
  __syncthreads();
  if (w == 0) {
    int v = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(FULL, v, o);
      if (lane >= o) v += y;
    }
    wsum[lane] = v;
  }
  __syncthreads();
  int run = x - s + (w > 0 ? wsum[w - 1] : 0);
  for (int64_t i = b; i < e; ++i) {
    const int v = a[i];
    a[i] = run;
    run += v;
  }
  if (total && t == 1023) *total = run;
}

// Exclusive scan of each digit's row of per-block counts (one block per
// digit, in place); dtot[d] = the digit's total.
__global__ void __launch_bounds__(256) rs_digit_scan_kernel(int* hist, int nblk, int* dtot) {
  __shared__ int wsum[8];
  const int d = blockIdx.x, t = threadIdx.x, lane = t & 31, w = t >> 5;
  int* row = hist + (int64_t)d * nblk;
  const int per = (nblk + 255) / 256, b = t * per, e = min(b + per, nblk);
  int s = 0;
  for (int i = b; i < e; ++i) s += row[i];
  int x = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[w] = x;
  __syncthreads();
  int wb = 0;
  for (int i = 0; i < w; ++i) wb += wsum[i];
  int run = wb + x - s;
  for (int i = b; i < e; ++i) {
    const int v = row[i];
    row[i] = run;
    run += v;
  }
  if (t == 255) dtot[d] = wb + x;
}

__global__ void __launch_bounds__(RS_THREADS) rs_scatter_kernel(const uint32_t* kin, const uint32_t* vin, int64_t F,
                                                                int shift, int digits, int nblk, const int* hist,
                                                                const int* dtot, uint32_t* kout, uint32_t* vout) {
  __shared__ int wcnt[8][MAX_DIGITS];
  __shared__ int base[MAX_DIGITS];
  __shared__ int wsum[RS_THREADS / 32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 8 * MAX_DIGITS; i += RS_THREADS) (&wcnt[0][0])[i] = 0;
  // base[d] = keys of smaller digits (exclusive scan of the digit totals)
  //         + keys of digit d in earlier blocks
  {
    constexpr int PER = MAX_DIGITS / RS_THREADS;   // 4 digits per thread
    int v[PER], s = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int dg = threadIdx.x * PER + j;
      v[j] = dg < digits ? dtot[dg] : 0;
      s += v[j];
    }
    int x = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(FULL, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    int run = x - s;
    for (int i = 0; i < w; ++i) run += wsum[i];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int dg = threadIdx.x * PER + j;
      if (dg < digits) base[dg] = run + hist[(int64_t)dg * nblk + blockIdx.x];
      run += v[j];
    }
  }
  __syncthreads();
  const uint32_t mask = (uint32_t)digits - 1;
  const unsigned lt = (1u << lane) - 1u;
  const int64_t w0 = (int64_t)blockIdx.x * RS_TILE + (int64_t)w * RS_WARP_ITEMS;
  uint32_t k[RS_ITEMS], v[RS_ITEMS];
  int rk[RS_ITEMS];
  // stable ranks within the warp, rounds in element order
#pragma unroll
  for (int r = 0; r < RS_ITEMS; ++r) {
    const int64_t e = w0 + r * 32 + lane;
    const bool ok = e < F;
    k[r] = ok ? kin[e] : 0u;
    v[r] = ok ? vin[e] : 0u;
    const int dg = ok ? (int)((k[r] >> shift) & mask) : MAX_DIGITS + lane;   // padding lanes never match
    const unsigned peers = __match_any_sync(FULL, dg);
    rk[r] = ok ? wcnt[w][dg] + __popc(peers & lt) : -1;
    __syncwarp();
    if (ok && (peers & lt) == 0) wcnt[w][dg] += __popc(peers);   // lowest peer lane updates
    __syncwarp();
  }
  __syncthreads();
  // per-digit offsets of the warps in element order
  for (int dgt = threadIdx.x; dgt < digits; dgt += RS_THREADS) {
    int run = 0;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) {
      const int c = wcnt[ww][dgt];
      wcnt[ww][dgt] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < RS_ITEMS; ++r) {
    if (rk[r] < 0) continue;
    const int dg = (int)((k[r] >> shift) & mask);
    const int64_t pos = (int64_t)base[dg] + wcnt[w][dg] + rk[r];
    kout[pos] = k[r];
    vout[pos] = v[r];
  }
}

// ---- 3. segments of equal slot ----
__device__ __forceinline__ bool seg_head(const uint32_t* keys, int64_t i, int64_t Fv) {
  return i < Fv && (i == 0 || keys[i] != keys[i - 1]);
}

__global__ void __launch_bounds__(256) seg_count_kernel(const uint32_t* keys, int64_t F, int* tot) {
  const int64_t Fv = F;
  const int64_t b0 = (int64_t)blockIdx.x * SEG_TILE;
  int c = 0;
  for (int i = threadIdx.x; i < SEG_TILE; i += 256) c += seg_head(keys, b0 + i, Fv);
  c = (int)warp_sum((float)c);   // exact for counts < 2^24
  __shared__ int ws[8];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int i = 0; i < 8; ++i) s += ws[i];
    tot[blockIdx.x] = s;
  }
}

// seg_id of every sorted fetch, seg_start / slot of every segment, and the
// sentinels seg_start[U] = F_valid and *n_seg = U.
__global__ void __launch_bounds__(256) seg_write_kernel(const uint32_t* keys, int64_t F, const int* tot_scanned,
                                                        int nb, int* seg_id, int* seg_start, int* uniq, int* n_seg) {
  __shared__ int ws[8];
  const int64_t Fv = F;
  const int64_t b0 = (int64_t)blockIdx.x * SEG_TILE;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int run = tot_scanned[blockIdx.x];
  // 4 rounds of 256 consecutive flags
  for (int r = 0; r < SEG_TILE / 256; ++r) {
    const int64_t i = b0 + r * 256 + threadIdx.x;
    const int fl = seg_head(keys, i, Fv);
    const unsigned bal = __ballot_sync(FULL, fl);
    const int before = __popc(bal & ((1u << lane) - 1u));
    if (lane == 0) ws[w] = __popc(bal);
    __syncthreads();
    int wb = 0;
    for (int ww = 0; ww < w; ++ww) wb += ws[ww];
    int rt = 0;
    for (int ww = 0; ww < 8; ++ww) rt += ws[ww];
    const int id = run + wb + before + fl - 1;   // inclusive count - 1
    if (i < Fv) {
      seg_id[i] = id;
      if (fl) {
        seg_start[id] = (int)i;
        uniq[id] = (int)keys[i];
      }
    }
    run += rt;
    __syncthreads();
  }
  if (blockIdx.x == nb - 1 && threadIdx.x == 0) {
    *n_seg = run;
    seg_start[run] = (int)Fv;
  }
}

// ---- 4. per-segment sums ----
struct Fetch {
  int seg;
  int token;
  int read;
  float w;
};

__device__ __forceinline__ Fetch load_fetch(const RowGradK& R, const int* seg_id, const uint32_t* vals, int64_t i) {
  Fetch x;
  x.seg = seg_id[i];
  const uint32_t raw = vals[i];
  const int64_t f = raw & ~DROPPED;
  int r = 0;
  while (r + 1 < R.n_reads && f >= R.off[r + 1]) ++r;
  const int64_t lf = f - R.off[r];
  x.read = r;
  x.token = (int)(lf / R.hk);
  x.w = (raw & DROPPED) ? 0.f : R.weights[r][lf];
  return x;
}

template <int VPL>   // floats per lane (d <= 32 * VPL, d % 4 == 0)
__device__ __forceinline__ void add_row(float (&acc)[VPL], const float* g, float w, int d, int lane) {
#pragma unroll
  for (int c = 0; c < VPL / 4; ++c) {
    const int e = (c * 32 + lane) * 4;
    if (e < d) {
      const float4 x = __ldg(reinterpret_cast<const float4*>(g + e));
      acc[4 * c] = fmaf(w, x.x, acc[4 * c]);
      acc[4 * c + 1] = fmaf(w, x.y, acc[4 * c + 1]);
      acc[4 * c + 2] = fmaf(w, x.z, acc[4 * c + 2]);
      acc[4 * c + 3] = fmaf(w, x.w, acc[4 * c + 3]);
    }
  }
}

template <int VPL>
__device__ __forceinline__ void store_row(const float (&acc)[VPL], float* dst, int d, int lane) {
#pragma unroll
  for (int c = 0; c < VPL / 4; ++c) {
    const int e = (c * 32 + lane) * 4;
    if (e < d) *reinterpret_cast<float4*>(dst + e) = make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
  }
}

template <int VPL>
__device__ __forceinline__ float row_sq(const float (&acc)[VPL]) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) s = fmaf(acc[i], acc[i], s);
  return warp_sum(s);
}

// Rows of segment u are complete when the segment lies inside the chunk;
// otherwise the chunk's partial goes to spill[chunk][0] (segment began
// before the chunk) or spill[chunk][1] (segment ends after the chunk).
template <int VPL>
__device__ __forceinline__ void flush(const RowGradK& R, const int* seg_start, int u, int64_t i0, int64_t i1,
                                      const float (&acc)[VPL], int64_t chunk, float* rows, float* rowsq,
                                      float* spill, int lane) {
  const int64_t s0 = seg_start[u], s1 = seg_start[u + 1];
  if (s0 >= i0 && s1 <= i1) {
    store_row<VPL>(acc, rows + (int64_t)u * R.d, R.d, lane);
    const float q = row_sq<VPL>(acc);
    if (lane == 0) rowsq[u] = q;
  } else {
    store_row<VPL>(acc, spill + (chunk * 2 + (s0 < i0 ? 0 : 1)) * R.d, R.d, lane);
  }
}

template <int VPL>
__global__ void __launch_bounds__(256) rg_rows_kernel(RowGradK R, const int* seg_id, const uint32_t* vals,
                                                      const int* seg_start, float* rows, float* rowsq, float* spill) {
  const int lane = threadIdx.x & 31;
  const int64_t chunk = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t Fv = R.F;
  const int64_t i0 = chunk * CHUNK;
  if (i0 >= Fv) return;
  const int64_t i1 = i0 + CHUNK < Fv ? i0 + CHUNK : Fv;
  // the chunk's fetches, two per lane
  Fetch fa = {0, 0, 0, 0.f}, fb = {0, 0, 0, 0.f};
  if (i0 + lane < i1) fa = load_fetch(R, seg_id, vals, i0 + lane);
  if (i0 + 32 + lane < i1) fb = load_fetch(R, seg_id, vals, i0 + 32 + lane);
  const int n = (int)(i1 - i0);
  float acc[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) acc[i] = 0.f;
  int u = __shfl_sync(FULL, fa.seg, 0);
  for (int j = 0; j < n; ++j) {
    const int src = j & 31;
    const bool hi = j >= 32;
    const int seg = __shfl_sync(FULL, hi ? fb.seg : fa.seg, src);
    const int tok = __shfl_sync(FULL, hi ? fb.token : fa.token, src);
    const int rd = __shfl_sync(FULL, hi ? fb.read : fa.read, src);
    const float w = __shfl_sync(FULL, hi ? fb.w : fa.w, src);
    if (seg != u) {
      flush<VPL>(R, seg_start, u, i0, i1, acc, chunk, rows, rowsq, spill, lane);
#pragma unroll
      for (int i = 0; i < VPL; ++i) acc[i] = 0.f;
      u = seg;
    }
    add_row<VPL>(acc, R.grad[rd] + (int64_t)tok * R.d, w, R.d, lane);
  }
  flush<VPL>(R, seg_start, u, i0, i1, acc, chunk, rows, rowsq, spill, lane);
}

// acc += rows p0, p0 + stride, ... (count of them, d floats each) in order;
// the loads are issued SB at a time.
template <int VPL>
__device__ __forceinline__ void add_run(float (&acc)[VPL], const float* p0, int64_t stride, int64_t count, int d,
                                        int lane) {
  constexpr int SB = VPL <= 4 ? 16 : 64 / VPL;
  for (int64_t i = 0; i < count; i += SB) {
    const int nb = count - i < SB ? (int)(count - i) : SB;
    float4 x[SB][VPL / 4];
#pragma unroll
    for (int b = 0; b < SB; ++b)
#pragma unroll
      for (int c = 0; c < VPL / 4; ++c) {
        const int e = (c * 32 + lane) * 4;
        x[b][c] = (b < nb && e < d) ? *reinterpret_cast<const float4*>(p0 + (i + b) * stride + e)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
    for (int b = 0; b < SB; ++b) {
      if (b >= nb) break;
#pragma unroll
      for (int c = 0; c < VPL / 4; ++c) {
        acc[4 * c] += x[b][c].x;
        acc[4 * c + 1] += x[b][c].y;
        acc[4 * c + 2] += x[b][c].z;
        acc[4 * c + 3] += x[b][c].w;
      }
    }
  }
}

// Group g of SPAN_GROUP chunks lying wholly inside one segment (which began
// before the group and reaches its end): the sum of its chunks' partials, in
// chunk order, one warp per group.  A hot row's segment covers thousands of
// chunks; the span kernel then adds group sums instead of chunk partials.
template <int VPL>
__global__ void __launch_bounds__(256) rg_group_kernel(RowGradK R, const int* seg_id, const int* seg_start,
                                                       const float* spill, float* grp, int64_t groups) {
  const int lane = threadIdx.x & 31;
  const int64_t g = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (g >= groups) return;
  const int64_t i0 = g * SPAN_GROUP * CHUNK, i1 = i0 + SPAN_GROUP * CHUNK;
  if (i1 > R.F) return;
  const int u = seg_id[i0];
  if (!(seg_start[u] < i0 && seg_start[u + 1] >= i1)) return;
  float acc[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) acc[i] = 0.f;
  add_run<VPL>(acc, spill + (g * SPAN_GROUP * 2) * R.d, 2 * R.d, SPAN_GROUP, R.d, lane);
  store_row<VPL>(acc, grp + g * R.d, R.d, lane);
}

// One warp per chunk: the chunk where a boundary-crossing segment starts
// adds the partials of every chunk the segment covers: its own tail
// partial, the chunks up to the next group boundary, the group sums of the
// whole groups inside the segment, then the remaining chunks -- a fixed order.
template <int VPL>
__global__ void __launch_bounds__(256) rg_span_kernel(RowGradK R, const int* seg_id, const int* seg_start,
                                                      float* rows, float* rowsq, const float* spill,
                                                      const float* grp) {
  const int lane = threadIdx.x & 31;
  const int64_t chunk = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t Fv = R.F;
  const int64_t i0 = chunk * CHUNK;
  if (i0 >= Fv) return;
  const int64_t i1 = i0 + CHUNK < Fv ? i0 + CHUNK : Fv;
  const int u = seg_id[i1 - 1];
  const int64_t s0 = seg_start[u], s1 = seg_start[u + 1];
  if (!(s0 >= i0 && s1 > i1)) return;
  float acc[VPL];
  const int d = R.d;
#pragma unroll
  for (int i = 0; i < VPL; ++i) acc[i] = 0.f;
  add_run<VPL>(acc, spill + (chunk * 2 + 1) * d, 0, 1, d, lane);
  const int64_t last = (s1 - 1) / CHUNK;
  int64_t c = chunk + 1;
  // head: up to the next group boundary
  int64_t hb = (c + SPAN_GROUP - 1) / SPAN_GROUP * SPAN_GROUP;
  if (hb > last + 1) hb = last + 1;
  add_run<VPL>(acc, spill + (c * 2) * d, 2 * d, hb - c, d, lane);
  c = hb;
  // whole groups inside the segment
  if (c % SPAN_GROUP == 0) {
    const int64_t g0 = c / SPAN_GROUP, gend = s1 / ((int64_t)SPAN_GROUP * CHUNK);
    if (gend > g0) {
      add_run<VPL>(acc, grp + g0 * d, d, gend - g0, d, lane);
      c = gend * SPAN_GROUP;
    }
  }
  // tail
  if (c <= last) add_run<VPL>(acc, spill + (c * 2) * d, 2 * d, last - c + 1, d, lane);
  store_row<VPL>(acc, rows + (int64_t)u * d, d, lane);
  const float q = row_sq<VPL>(acc);
  if (lane == 0) rowsq[u] = q;
}

// ---- 5. squared norm of all rows: float64 partials in a fixed order ----
__global__ void __launch_bounds__(256) rg_sqnorm_kernel(const float* rowsq, const int* n_seg, double* part,
                                                        int* ticket, float* sq_out, double* sq_d) {
  const int U = *n_seg;
  const int per = (U + SQ_BLOCKS - 1) / SQ_BLOCKS;
  const int b0 = blockIdx.x * per, b1 = b0 + per < U ? b0 + per : U;
  __shared__ double sh[256];
  double s = 0.0;
  for (int i = b0 + threadIdx.x; i < b1; i += 256) s += (double)rowsq[i];
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  __shared__ bool last;
  if (threadIdx.x == 0) {
    part[blockIdx.x] = sh[0];
    __threadfence();
    last = atomicAdd(ticket, 1) == SQ_BLOCKS - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    double t = 0.0;
    for (int i = 0; i < SQ_BLOCKS; ++i) t += ((volatile double*)part)[i];
    *sq_d = t;
    if (sq_out) *sq_out = (float)t;
    *ticket = 0;
  }
}

// ---- outputs of fetched_row_grads: padding beyond the U rows ----
__global__ void rg_pad_kernel(const int* n_seg, int64_t cap, int64_t N, int d, int* uniq, float* rows,
                              int* n_unique_out) {
  const int U = *n_seg;
  if (blockIdx.x == 0 && threadIdx.x == 0 && n_unique_out) *n_unique_out = U;
  if (!uniq) return;
  for (int64_t i = U + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < cap; i += (int64_t)gridDim.x * blockDim.x)
    uniq[i] = (int)N;
  if (rows) {
    const int64_t n4 = (cap - U) * d / 4;
    float4* r = reinterpret_cast<float4*>(rows + (int64_t)U * d);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x)
      r[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// ---- Adagrad on the touched rows (train.py:378-383, 396-399) ----
template <int VPL>
__global__ void __launch_bounds__(256) rg_adagrad_kernel(const int* n_seg, const int* uniq, const float* rows,
                                                         const double* sq_d, const float* rest_sq, float clip,
                                                         float lr, int d, float* values, float* accum,
                                                         float* scale_out) {
  const int lane = threadIdx.x & 31;
  const int64_t u = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const double gn2 = *sq_d + (rest_sq ? (double)*rest_sq : 0.0);
  // scale = min(1, clip / (global norm + 1e-6)) in float32, as the reference computes it
  const float gnorm = sqrtf((float)gn2);
  const float scale = fminf(1.f, clip / (gnorm + 1e-6f));
  if (u == 0 && lane == 0 && scale_out) *scale_out = scale;
  if (u >= *n_seg) return;
  const int64_t s = uniq[u];
  float g[VPL];
#pragma unroll
  for (int c = 0; c < VPL / 4; ++c) {
    const int e = (c * 32 + lane) * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e < d) x = *reinterpret_cast<const float4*>(rows + u * d + e);
    g[4 * c] = x.x * scale;
    g[4 * c + 1] = x.y * scale;
    g[4 * c + 2] = x.z * scale;
    g[4 * c + 3] = x.w * scale;
  }
  const float a = accum[s] + row_sq<VPL>(g) / (float)d;        // acc + mean(g^2)
  const float step = lr / (sqrtf(a) + 1e-8f);
  float* v = values + s * d;
#pragma unroll
  for (int c = 0; c < VPL / 4; ++c) {
    const int e = (c * 32 + lane) * 4;
    if (e < d) {
      float4 x = *reinterpret_cast<float4*>(v + e);
      x.x += -step * g[4 * c];
      x.y += -step * g[4 * c + 1];
      x.z += -step * g[4 * c + 2];
      x.w += -step * g[4 * c + 3];
      *reinterpret_cast<float4*>(v + e) = x;
    }
  }
  if (lane == 0) accum[s] = a;
}

// inv[fetch] = its segment (sorted position i holds fetch vals[i])
__global__ void rg_inverse_kernel(const uint32_t* vals, const int* seg_id, int64_t F, int* inv) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= F) return;
  const uint32_t v = vals[i];
  inv[v & ~DROPPED] = (v & DROPPED) ? -1 : seg_id[i];
}

inline int vpl_for(int d) { return d <= 128 ? 4 : d <= 256 ? 8 : d <= 512 ? 16 : 32; }

#define ML_VPL(V, CALL) \
  switch (V) {          \
    case 4: { constexpr int VP = 4; CALL; } break;   \
    case 8: { constexpr int VP = 8; CALL; } break;   \
    case 16: { constexpr int VP = 16; CALL; } break; \
    default: { constexpr int VP = 32; CALL; } break; \
  }

}  // namespace

RowGradLayout rowgrad_layout(int64_t F, int64_t N, int d) {
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  RowGradLayout L{};
  int bits = 1;
  while (bits < 32 && (((int64_t)1 << bits) < N)) ++bits;    // keys in [0, N - 1]
  L.passes = (bits + 9) / 10;
  L.rbits = (bits + L.passes - 1) / L.passes;
  L.nblk = F > 0 ? (F + RS_TILE - 1) / RS_TILE : 1;
  L.nseg_blk = F > 0 ? (F + SEG_TILE - 1) / SEG_TILE : 1;
  L.chunks = F > 0 ? (F + CHUNK - 1) / CHUNK : 1;
  L.cap = F < N ? F : N;
  int64_t o = 0;
  auto take = [&](int64_t bytes) {
    const int64_t at = o;
    o += up(bytes);
    return at;
  };
  L.o_small = take(256);                                  // segment count, ticket
  L.o_err = take(256);                                    // status word (offset 256, as in the forward layouts)
  L.o_keys_a = take(4 * F);
  L.o_vals_a = take(4 * F);
  L.o_keys_b = take(4 * F);
  L.o_vals_b = take(4 * F);
  L.o_hist = take(4 * ((int64_t)1 << L.rbits) * L.nblk);
  L.o_dtot = take(4 * ((int64_t)1 << L.rbits));
  L.o_segtot = take(4 * L.nseg_blk);
  L.o_seg_id = take(4 * F);
  L.o_seg_start = take(4 * (L.cap + 1));
  L.o_uniq = take(4 * L.cap);
  L.o_rows = take(4 * L.cap * d);
  L.o_rowsq = take(4 * L.cap);
  L.o_spill = take(4 * L.chunks * 2 * d);
  L.groups = (L.chunks + SPAN_GROUP - 1) / SPAN_GROUP;
  L.o_grp = take(4 * L.groups * d);
  L.o_part = take(8 * SQ_BLOCKS);
  L.o_sq = take(8);
  L.bytes = o;
  return L;
}

namespace {

// Keys of every fetch, the stable radix passes and the segments; on return
// (*ka, *va) hold the sorted keys / fetch ids.  F > 0.
cudaError_t sort_segments(const RowGradK& R, const RowGradLayout& L, char* ws, uint32_t** ka_out, uint32_t** va_out,
                          int* uniq, cudaStream_t s) {
  int* small = reinterpret_cast<int*>(ws + L.o_small);
  int* err = reinterpret_cast<int*>(ws + L.o_err);
  int* n_seg = small + 1;
  int* dtot = reinterpret_cast<int*>(ws + L.o_dtot);
  uint32_t* ka = reinterpret_cast<uint32_t*>(ws + L.o_keys_a);
  uint32_t* va = reinterpret_cast<uint32_t*>(ws + L.o_vals_a);
  uint32_t* kb = reinterpret_cast<uint32_t*>(ws + L.o_keys_b);
  uint32_t* vb = reinterpret_cast<uint32_t*>(ws + L.o_vals_b);
  int* hist = reinterpret_cast<int*>(ws + L.o_hist);
  int* segtot = reinterpret_cast<int*>(ws + L.o_segtot);
  int* seg_id = reinterpret_cast<int*>(ws + L.o_seg_id);
  int* seg_start = reinterpret_cast<int*>(ws + L.o_seg_start);
  const int64_t F = R.F;
  rg_keys_kernel<<<(unsigned)((F + 255) / 256), 256, 0, s>>>(R, ka, va, err);
  count_launch();
  const int digits = 1 << L.rbits;
  for (int p = 0; p < L.passes; ++p) {
    const int shift = p * L.rbits;
    rs_hist_kernel<<<(unsigned)L.nblk, RS_THREADS, 0, s>>>(ka, F, shift, digits, (int)L.nblk, hist);
    rs_digit_scan_kernel<<<(unsigned)digits, 256, 0, s>>>(hist, (int)L.nblk, dtot);
    rs_scatter_kernel<<<(unsigned)L.nblk, RS_THREADS, 0, s>>>(ka, va, F, shift, digits, (int)L.nblk, hist, dtot, kb,
                                                              vb);
    count_launch(3);
    uint32_t* t = ka; ka = kb; kb = t;
    t = va; va = vb; vb = t;
  }
  // sorted keys / fetch ids are now in (ka, va)
  seg_count_kernel<<<(unsigned)L.nseg_blk, 256, 0, s>>>(ka, F, segtot);
  scan_excl_kernel<<<1, 1024, 0, s>>>(segtot, L.nseg_blk, nullptr);
  seg_write_kernel<<<(unsigned)L.nseg_blk, 256, 0, s>>>(ka, F, segtot, (int)L.nseg_blk, seg_id, seg_start, uniq,
                                                        n_seg);
  count_launch(3);
  *ka_out = ka;
  *va_out = va;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_sort_unique(const RowGradK& R, const RowGradLayout& L, char* ws, int* inv, cudaStream_t s) {
  cudaError_t e;
  if ((e = cudaMemsetAsync(ws + L.o_small, 0, 512, s)) != cudaSuccess) return e;   // counters and status word
  if (R.F == 0) return cudaSuccess;
  uint32_t *ka, *va;
  if ((e = sort_segments(R, L, ws, &ka, &va, reinterpret_cast<int*>(ws + L.o_uniq), s)) != cudaSuccess) return e;
  rg_inverse_kernel<<<(unsigned)((R.F + 255) / 256), 256, 0, s>>>(va, reinterpret_cast<const int*>(ws + L.o_seg_id),
                                                                  R.F, inv);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_rowgrad(const RowGradK& R, const RowGradLayout& L, char* ws, int* uniq_out, float* rows_out,
                           int* n_unique_out, float* sq_out, const RowAdagrad* ada, cudaStream_t s) {
  int* small = reinterpret_cast<int*>(ws + L.o_small);
  int* n_seg = small + 1, *ticket = small + 2;
  uint32_t* ka = nullptr;
  uint32_t* va = nullptr;
  int* seg_id = reinterpret_cast<int*>(ws + L.o_seg_id);
  int* seg_start = reinterpret_cast<int*>(ws + L.o_seg_start);
  int* uniq = uniq_out ? uniq_out : reinterpret_cast<int*>(ws + L.o_uniq);
  float* rows = rows_out ? rows_out : reinterpret_cast<float*>(ws + L.o_rows);
  float* rowsq = reinterpret_cast<float*>(ws + L.o_rowsq);
  float* spill = reinterpret_cast<float*>(ws + L.o_spill);
  double* part = reinterpret_cast<double*>(ws + L.o_part);
  double* sqd = reinterpret_cast<double*>(ws + L.o_sq);
  cudaError_t e;
  if ((e = cudaMemsetAsync(small, 0, 512, s)) != cudaSuccess) return e;   // counters and status word
  const int64_t F = R.F;
  if (F > 0) {
    if ((e = sort_segments(R, L, ws, &ka, &va, uniq, s)) != cudaSuccess) return e;
    const unsigned wblocks = (unsigned)((L.chunks + 7) / 8);
    ML_VPL(vpl_for(R.d), (rg_rows_kernel<VP><<<wblocks, 256, 0, s>>>(R, seg_id, va, seg_start, rows, rowsq,
                                                                      spill)));
    float* grp = reinterpret_cast<float*>(ws + L.o_grp);
    if (L.chunks > SPAN_GROUP) {
      ML_VPL(vpl_for(R.d), (rg_group_kernel<VP><<<(unsigned)((L.groups + 7) / 8), 256, 0, s>>>(R, seg_id, seg_start,
                                                                                               spill, grp, L.groups)));
      count_launch();
    }
    ML_VPL(vpl_for(R.d), (rg_span_kernel<VP><<<wblocks, 256, 0, s>>>(R, seg_id, seg_start, rows, rowsq, spill,
                                                                      grp)));
    count_launch(2);
  }
  rg_sqnorm_kernel<<<SQ_BLOCKS, 256, 0, s>>>(rowsq, n_seg, part, ticket, sq_out, sqd);
  count_launch();
  if (uniq_out || n_unique_out) {
    rg_pad_kernel<<<296, 256, 0, s>>>(n_seg, L.cap, R.N, R.d, uniq_out, rows_out, n_unique_out);
    count_launch();
  }
  if (ada) {
    const unsigned ublocks = (unsigned)((L.cap + 7) / 8 > 0 ? (L.cap + 7) / 8 : 1);
    ML_VPL(vpl_for(R.d), (rg_adagrad_kernel<VP><<<ublocks, 256, 0, s>>>(n_seg, uniq, rows, sqd, ada->rest_sq,
                                                                         ada->clip, ada->lr, R.d, ada->values,
                                                                         ada->accum, ada->scale_out)));
    count_launch();
    if (ada->n_unique_out && !uniq_out)
      if ((e = cudaMemcpyAsync(ada->n_unique_out, n_seg, sizeof(int), cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
        return e;
  }
  return cudaGetLastError();
}

}  // namespace ml
