// Owner-sharded row update of the row-sharded table (training).
//
// The reference trainer keeps the whole table on every device and merges
// the fetched-row gradients of all devices before the update
// (memory_pool_model/train.py:175-206 fetched_row_grads_sharded: a local
// merge per device, an all-gather of the merged rows, a second merge; then
// every device applies the same clip + row-wise Adagrad to its copy).  With
// slot s held only by rank s % world (local row s / world), each row needs
// its gradient on one rank only:
//
//   ROUTE   the local merge runs with owner-grouped sort keys
//           (owner * stride + local row), so this rank's distinct rows come
//           out grouped by owner, ascending by local row; each row goes
//           straight into its owner's inbox over NVLink (row + local row),
//           and the last CTA publishes the per-owner counts and the epoch;
//   GATHER  the owner waits for every source, merges the sources' sorted
//           lists (merge position by binary search: stable by source rank),
//           sums each local row's contributions in source-rank order -- the
//           association of the reference's all-gather + second merge -- and
//           publishes its sum of merged rows^2 (float64) into every rank;
//   REDUCE  every rank adds the owners' partials in rank order (the global
//           norm of the clip, identical on all ranks) and applies row-wise
//           Adagrad to the rows it owns.
//
// Buffers are reused across calls without a reset: a source's next push
// follows its own REDUCE, which waited for every owner's norm partial, and an
// owner publishes that only after it has finished reading its inbox.  Every
// wait is bounded (about 2 s); a wait that gives up records a code in the
// status word and skips its work.
#include "shard.cuh"

namespace ml {

namespace {

__device__ __forceinline__ int lower_bound_i(const int* a, int n, int v) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldcg(a + mid) < v) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ int upper_bound_i(const int* a, int n, int v) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldcg(a + mid) <= v) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// One warp per distinct row of this rank's merge.
__global__ void __launch_bounds__(256) rows_push_kernel(const __grid_constant__ RowShardK K,
                                                        const int* __restrict__ uniq, const float* __restrict__ rows,
                                                        const int* __restrict__ n_seg, int* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  const int U = *n_seg;
  const int d4 = K.d / 4;
  for (int64_t i = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); i < U; i += (int64_t)gridDim.x * 8) {
    const int key = uniq[i];
    const int o = (int)(key / K.stride);
    const int lrow = (int)(key - (int64_t)o * K.stride);
    int lo = 0;
    if (lane == 0) lo = lower_bound_i(uniq, U, (int)(o * K.stride));
    lo = __shfl_sync(FULL, lo, 0);
    const int64_t pos = i - lo;
    if (o >= K.world || pos >= K.cap) {   // only a bug upstream can cause this
      if (lane == 0) atomicCAS(err, 0, 24);
      continue;
    }
    char* ob = K.peer[o];
    if (lane == 0) reinterpret_cast<int*>(ob + K.off.lin)[(int64_t)K.rank * K.cap + pos] = lrow;
    const float4* src = reinterpret_cast<const float4*>(rows + i * K.d);
    float4* dst = reinterpret_cast<float4*>(ob + K.off.rin) + ((int64_t)K.rank * K.cap + pos) * d4;
    for (int e = lane; e < d4; e += 32) dst[e] = src[e];
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  // the last CTA publishes each owner's count, then the epoch
  fence_sys();
  int* ticket = reinterpret_cast<int*>(K.peer[K.rank] + K.off.tickets);
  if (atomicAdd(ticket, 1) != (int)gridDim.x - 1) return;
  *ticket = 0;
  fence_sys();
  for (int o = 0; o < K.world; ++o) {
    const int lo = lower_bound_i(uniq, U, (int)(o * K.stride));
    const int hi = lower_bound_i(uniq, U, (int)((o + 1) * K.stride));
    reinterpret_cast<int*>(K.peer[o] + K.off.cnt)[K.rank] = hi - lo;
    st_release_sys(reinterpret_cast<int*>(K.peer[o] + K.off.flags_in) + K.rank, K.epoch);
  }
}

// Merge position of every inbox entry: entries before (source, i) with local
// row v are the i earlier ones of its own list, those <= v of lower sources
// and those < v of higher sources (each list holds distinct rows).
__global__ void __launch_bounds__(256) rows_rank_kernel(const __grid_constant__ RowShardK K, RowMerge G,
                                                        int* __restrict__ err) {
  __shared__ int ok_s;
  __shared__ int cnt_s[MEMLAYER_MAX_SHARDS];
  const char* mine = K.peer[K.rank];
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int src = 0; src < K.world && ok; ++src)
      ok = wait_epoch(reinterpret_cast<const int*>(mine + K.off.flags_in) + src, K.epoch, err, 33, K.wait_ns);
    ok_s = ok;
  }
  __syncthreads();
  if (!ok_s) {
    if (blockIdx.x == 0 && threadIdx.x == 0) G.small[0] = 0;
    return;
  }
  if (threadIdx.x < K.world) {
    const int c = __ldcg(reinterpret_cast<const int*>(mine + K.off.cnt) + threadIdx.x);
    cnt_s[threadIdx.x] = c < 0 ? 0 : (c > K.cap ? (int)K.cap : c);
  }
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    int T = 0;
    for (int src = 0; src < K.world; ++src) T += cnt_s[src];
    G.small[0] = T;
  }
  const int* lin = reinterpret_cast<const int*>(mine + K.off.lin);
  const int64_t total = (int64_t)K.world * K.cap;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int src = (int)(e / K.cap);
    const int64_t i = e - (int64_t)src * K.cap;
    if (i >= cnt_s[src]) continue;
    const int v = __ldcg(lin + e);
    int64_t pos = i;
    for (int s2 = 0; s2 < K.world; ++s2) {
      if (s2 == src) continue;
      const int* l2 = lin + (int64_t)s2 * K.cap;
      pos += s2 < src ? upper_bound_i(l2, cnt_s[s2], v) : lower_bound_i(l2, cnt_s[s2], v);
    }
    G.mkey[pos] = v;
    G.mref[pos] = (int)e;
  }
}

// One warp per merged entry: the first entry of each local row sums the
// row's contributions in source-rank order.
__global__ void __launch_bounds__(256) rows_sum_kernel(const __grid_constant__ RowShardK K, RowMerge G,
                                                       int* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  if (*(volatile const int*)err == 33) return;   // the merge's wait gave up: positions are incomplete
  const int T = G.small[0];
  const int64_t total = (int64_t)K.world * K.cap;
  const int d4 = K.d / 4;
  const float4* rin = reinterpret_cast<const float4*>(K.peer[K.rank] + K.off.rin);
  for (int64_t p = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); p < T; p += (int64_t)gridDim.x * 8) {
    const int v = G.mkey[p];
    const bool head = p == 0 || G.mkey[p - 1] != v;
    if (!head) {
      if (lane == 0) {
        G.head[p] = 0;
        G.rowsq[p] = 0.f;
      }
      continue;
    }
    int64_t pe = p + 1;
    while (pe < T && pe - p < K.world && G.mkey[pe] == v) ++pe;
    float sq = 0.f;
    for (int e = lane; e < d4; e += 32) {
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int64_t q = p; q < pe; ++q) {
        const int64_t ref = G.mref[q];
        if (ref < 0 || ref >= total) {   // only a bug upstream can cause this
          atomicCAS(err, 0, 24);
          continue;
        }
        const float4 x = __ldcg(rin + ref * d4 + e);
        a.x += x.x;
        a.y += x.y;
        a.z += x.z;
        a.w += x.w;
      }
      reinterpret_cast<float4*>(G.mrow)[p * d4 + e] = a;
      sq = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, sq))));
    }
    sq = warp_sum(sq);
    if (lane == 0) {
      G.head[p] = 1;
      G.rowsq[p] = sq;
    }
  }
}

// This owner's sum of merged rows^2 (fixed thread map, fixed tree, float64)
// and touched-row count; the sum is stored into every rank's buffer and the
// epoch published.
__global__ void __launch_bounds__(1024) rows_publish_kernel(const __grid_constant__ RowShardK K, RowMerge G,
                                                            const int* __restrict__ err) {
  __shared__ double red[32];
  __shared__ int redh[32];
  const int T = G.small[0];
  double s = 0.0;
  int h = 0;
  for (int i = threadIdx.x; i < T; i += 1024) {
    s += (double)G.rowsq[i];
    h += G.head[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(FULL, s, o);
    h += __shfl_xor_sync(FULL, h, o);
  }
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = s;
    redh[threadIdx.x >> 5] = h;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  double t = 0.0;
  int nh = 0;
  for (int w = 0; w < 32; ++w) {
    t += red[w];
    nh += redh[w];
  }
  G.small[1] = nh;
  // a wait of the merge that gave up leaves the peers waiting for this flag
  // too (bounded), so they skip their update as well
  if (*(volatile const int*)err == 33) return;
  for (int o = 0; o < K.world; ++o)
    reinterpret_cast<double*>(K.peer[o] + K.off.sq)[K.rank] = t;
  fence_sys();
  for (int o = 0; o < K.world; ++o)
    st_release_sys(reinterpret_cast<int*>(K.peer[o] + K.off.flags_sq) + K.rank, K.epoch);
}

// scale = min(1, clip / (global norm + 1e-6)) (train.py:378-383); then per
// touched local row acc += mean(g^2), V -= lr / (sqrt(acc) + 1e-8) g
// (train.py:396-399).  One warp per merged entry.
__global__ void __launch_bounds__(256) rows_apply_kernel(const __grid_constant__ RowShardK K, RowMerge G,
                                                         float* __restrict__ values, float* __restrict__ accum,
                                                         float lr, float clip, const float* __restrict__ rest_sq,
                                                         float* __restrict__ scale_out, int* __restrict__ n_unique_out,
                                                         int* __restrict__ err) {
  __shared__ int ok_s;
  __shared__ float scale_s;
  const char* mine = K.peer[K.rank];
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int o = 0; o < K.world && ok; ++o)
      ok = wait_epoch(reinterpret_cast<const int*>(mine + K.off.flags_sq) + o, K.epoch, err, 34, K.wait_ns);
    ok_s = ok;
    if (ok) {
      double gn2 = 0.0;
      const double* sq = reinterpret_cast<const double*>(mine + K.off.sq);
      for (int o = 0; o < K.world; ++o) gn2 += __ldcg(sq + o);     // owners in rank order
      if (rest_sq) gn2 += (double)*rest_sq;
      const float gnorm = sqrtf((float)gn2);
      scale_s = fminf(1.f, clip / (gnorm + 1e-6f));
      if (blockIdx.x == 0) {
        if (scale_out) *scale_out = scale_s;
        if (n_unique_out) *n_unique_out = G.small[1];
      }
    }
  }
  __syncthreads();
  if (!ok_s) return;
  const float scale = scale_s;
  const int lane = threadIdx.x & 31;
  const int T = G.small[0];
  const int d4 = K.d / 4;
  for (int64_t p = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); p < T; p += (int64_t)gridDim.x * 8) {
    if (!G.head[p]) continue;
    const int64_t r = G.mkey[p];
    if (r < 0 || r >= K.rows) {   // only a bug upstream can cause this
      if (lane == 0) atomicCAS(err, 0, 22);
      continue;
    }
    const float4* g4 = reinterpret_cast<const float4*>(G.mrow) + p * d4;
    float q = 0.f;
    for (int e = lane; e < d4; e += 32) {
      float4 g = g4[e];
      g.x *= scale;
      g.y *= scale;
      g.z *= scale;
      g.w *= scale;
      q = fmaf(g.x, g.x, fmaf(g.y, g.y, fmaf(g.z, g.z, fmaf(g.w, g.w, q))));
    }
    q = warp_sum(q);
    const float a = accum[r] + q / (float)K.d;
    const float step = lr / (sqrtf(a) + 1e-8f);
    float4* v4 = reinterpret_cast<float4*>(values + r * K.d);
    for (int e = lane; e < d4; e += 32) {
      const float4 g = g4[e];
      float4 v = v4[e];
      v.x += -step * (g.x * scale);
      v.y += -step * (g.y * scale);
      v.z += -step * (g.z * scale);
      v.w += -step * (g.w * scale);
      v4[e] = v;
    }
    if (lane == 0) accum[r] = a;
  }
}

unsigned warp_grid(int64_t items) {
  const int64_t b = (items + 7) / 8;
  return (unsigned)(b < 1 ? 1 : b < 148 * 8 ? b : 148 * 8);
}

}  // namespace

RowShardOff row_shard_layout(int world, int64_t cap, int d) {
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  RowShardOff o;
  o.flags_in = 0;
  o.flags_sq = 256;
  o.tickets = 512;
  o.cnt = 768;
  o.sq = 1024;
  o.lin = 1280;
  o.rin = o.lin + up((int64_t)world * cap * 4);
  o.bytes = o.rin + up((int64_t)world * cap * d * 4);
  return o;
}

cudaError_t launch_rows_push(const RowShardK& K, const int* uniq, const float* rows, const int* n_seg, int64_t ucap,
                             int* err, cudaStream_t s) {
  rows_push_kernel<<<warp_grid(ucap), 256, 0, s>>>(K, uniq, rows, n_seg, err);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_rows_merge(const RowShardK& K, const RowMerge& G, int* err, cudaStream_t s) {
  const int64_t total = (int64_t)K.world * K.cap;
  const int64_t b = (total + 255) / 256;
  rows_rank_kernel<<<(unsigned)(b < 1 ? 1 : b < 148 * 8 ? b : 148 * 8), 256, 0, s>>>(K, G, err);
  rows_sum_kernel<<<warp_grid(total), 256, 0, s>>>(K, G, err);
  rows_publish_kernel<<<1, 1024, 0, s>>>(K, G, err);
  count_launch(3);
  return cudaGetLastError();
}

cudaError_t launch_rows_apply(const RowShardK& K, const RowMerge& G, float* values, float* accum, float lr,
                              float clip, const float* rest_sq, float* scale_out, int* n_unique_out, int* err,
                              cudaStream_t s) {
  rows_apply_kernel<<<warp_grid((int64_t)K.world * K.cap), 256, 0, s>>>(K, G, values, accum, lr, clip, rest_sq,
                                                                        scale_out, n_unique_out, err);
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
