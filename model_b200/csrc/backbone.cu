// The language model around the memory layer (memory_pool_model/model.py:15-127)
// and its decode step (generate.py:31-34): token + position embedding,
// LayerNorm (fused with the residual add before it), causal multi-head
// attention (whole sequences, and one position against a key / value
// cache), and the status merge of the memory-layer calls.  The Dense layers
// run on the tensor-core GEMM of gemm_tc.cu (or the SIMT GEMM / GEMV for few
// rows), the memory layers through memlayer_layer_forward.
#include <float.h>

#include "backbone.cuh"

namespace ml {

namespace {

// x[m] = embedding[token] + pos_embed[p]: p = m % T (a whole sequence) or
// *pos (one decode step).  A token outside [0, V) records status 26 and
// embeds as zeros.
__global__ void __launch_bounds__(256) embed_kernel(const int* __restrict__ tokens, int64_t M, int T,
                                                    const int* __restrict__ pos, const float* __restrict__ E,
                                                    const float* __restrict__ Pe, int V, int dm, int max_len,
                                                    float* __restrict__ x, int* __restrict__ err) {
  const int64_t m = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (m >= M) return;
  const int tok = tokens[m];
  const int p = pos ? *pos : (int)(m % T);
  const bool ok = tok >= 0 && tok < V && p >= 0 && p < max_len;
  if (!ok && lane == 0) atomicCAS(err, 0, 26);
  for (int j = lane; j < dm; j += 32)
    x[m * dm + j] = ok ? E[(int64_t)tok * dm + j] + Pe[(int64_t)p * dm + j] : 0.f;   // model.py:61-66
}

// x += y (when y is given), then h = LayerNorm(x) (model.py:87,96,124 with
// flax's LayerNorm: eps 1e-6, variance E[x^2] - E[x]^2 clamped at 0,
// (x - mean) * (rsqrt(var + eps) * scale) + bias).  One warp per row.
constexpr int LN_MAX = 32;   // values per lane: d_model <= 1024
__global__ void __launch_bounds__(256) add_ln_kernel(float* __restrict__ x, const float* __restrict__ y,
                                                     const float* __restrict__ scale,
                                                     const float* __restrict__ bias, float* __restrict__ h,
                                                     int64_t M, int dm) {
  const int64_t m = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (m >= M) return;
  float v[LN_MAX];
  float s = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAX; ++i) {
    const int j = lane + 32 * i;
    v[i] = 0.f;
    if (j < dm) {
      float a = x[m * dm + j];
      if (y) {
        a += y[m * dm + j];
        x[m * dm + j] = a;
      }
      v[i] = a;
      s += a;
      s2 = fmaf(a, a, s2);
    }
  }
  s = warp_sum(s);
  s2 = warp_sum(s2);
  const float mean = s / (float)dm;
  const float var = fmaxf(0.f, s2 / (float)dm - mean * mean);
  const float r = 1.0f / sqrtf(var + 1e-6f);
#pragma unroll
  for (int i = 0; i < LN_MAX; ++i) {
    const int j = lane + 32 * i;
    if (j < dm) h[m * dm + j] = (v[i] - mean) * (r * scale[j]) + bias[j];
  }
}

// Causal self-attention of whole sequences (model.py:88-95, flax
// dot_product_attention): qkv [B*T, 3*dm] with the query, key and value of
// head h at columns h*DH, dm + h*DH and 2*dm + h*DH; out [B*T, dm] in the
// same head-major order.  A CTA takes 32 queries of one (batch, head) and
// walks 32-key tiles up to the diagonal with an online softmax (running
// max and sum in float32); 8 threads per query, each scoring 4 keys and
// accumulating DH/8 output dims.
constexpr int AQ = 32, AK = 32;

template <int DH>
__global__ void __launch_bounds__(256) attn_prefill_kernel(const float* __restrict__ qkv, float* __restrict__ out,
                                                           int T, int H) {
  __shared__ float qs[AQ][DH + 1];
  __shared__ float ks[AK][DH + 1];
  __shared__ float vs[AK][DH];
  const int dm = H * DH, ld = 3 * dm;
  const int q0 = blockIdx.x * AQ, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int tid = threadIdx.x, qi = tid >> 3, part = tid & 7;
  const float rs = sqrtf((float)DH);
  for (int e = tid; e < AQ * DH; e += 256) {
    const int r = e / DH, c = e - r * DH;
    const int t = q0 + r;
    qs[r][c] = t < T ? qkv[(b * T + t) * ld + h * DH + c] / rs : 0.f;   // query / sqrt(depth)
  }
  constexpr int OD = DH / 8;
  float acc[OD];
#pragma unroll
  for (int i = 0; i < OD; ++i) acc[i] = 0.f;
  float mrun = -FLT_MAX, lrun = 0.f;
  const int tq = q0 + qi;                          // this thread's query
  const int kend = min(T, q0 + AQ);                // keys past the block's last query are masked for all
  for (int k0 = 0; k0 < kend; k0 += AK) {
    __syncthreads();
    for (int e = tid; e < AK * DH; e += 256) {
      const int r = e / DH, c = e - r * DH;
      const int t = k0 + r;
      const int64_t row = (b * T + (t < T ? t : 0)) * ld;
      ks[r][c] = t < T ? qkv[row + dm + h * DH + c] : 0.f;
      vs[r][c] = t < T ? qkv[row + 2 * dm + h * DH + c] : 0.f;
    }
    __syncthreads();
    float sc[4];
    float mt = -FLT_MAX;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kk = part * 4 + j, tk = k0 + kk;
      float s = 0.f;
#pragma unroll 8
      for (int c = 0; c < DH; ++c) s = fmaf(qs[qi][c], ks[kk][c], s);
      sc[j] = (tk <= tq && tk < T) ? s : -FLT_MAX;   // causal mask
      mt = fmaxf(mt, sc[j]);
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(FULL, mt, o));
    const float mnew = fmaxf(mrun, mt);
    float p[4], ps = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      p[j] = sc[j] == -FLT_MAX ? 0.f : expf(sc[j] - mnew);
      ps += p[j];
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) ps += __shfl_xor_sync(FULL, ps, o);
    const float corr = mrun == -FLT_MAX ? 0.f : expf(mrun - mnew);
    lrun = lrun * corr + ps;
    mrun = mnew;
#pragma unroll
    for (int i = 0; i < OD; ++i) acc[i] *= corr;
    // every key of the tile: its probability from the thread that scored it
#pragma unroll
    for (int src = 0; src < 8; ++src) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pk = __shfl_sync(FULL, p[j], (threadIdx.x & 24) | src);
        const int kk = src * 4 + j;
#pragma unroll
        for (int i = 0; i < OD; ++i) acc[i] = fmaf(pk, vs[kk][part * OD + i], acc[i]);
      }
    }
  }
  if (tq < T) {
    const float inv = 1.0f / lrun;
#pragma unroll
    for (int i = 0; i < OD; ++i) out[(b * T + tq) * dm + h * DH + part * OD + i] = acc[i] * inv;
  }
}

// One decode position (model.py:88-95 with decode=True): the new key and
// value of each batch row go into the layer's cache at *pos, then the query
// attends to cache positions 0..*pos.  qkv [B, 3*dm]; cache_k / cache_v
// [B, max_len, dm]; out [B, dm].  One CTA per (batch row, head).
template <int DH>
__global__ void __launch_bounds__(256) attn_decode_kernel(const float* __restrict__ qkv, float* __restrict__ cache_k,
                                                          float* __restrict__ cache_v, const int* __restrict__ pos,
                                                          int max_len, int H, float* __restrict__ out,
                                                          int* __restrict__ err) {
  extern __shared__ float dsm[];
  float* q = dsm;                 // [DH]
  float* pr = dsm + DH;           // [max_len] scores, then probabilities
  __shared__ float red[8];
  __shared__ float part_s[8][DH];
  const int h = blockIdx.x, dm = H * DH;
  const int64_t b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int p = *pos;
  if (p < 0 || p >= max_len) {
    if (tid == 0) atomicCAS(err, 0, 26);
    for (int c = tid; c < DH; c += 256) out[b * dm + h * DH + c] = 0.f;
    return;
  }
  const float* row = qkv + b * 3 * dm;
  const int64_t cbase = (b * max_len) * dm + h * DH;
  const float rs = sqrtf((float)DH);
  for (int c = tid; c < DH; c += 256) {
    q[c] = row[h * DH + c] / rs;
    cache_k[cbase + (int64_t)p * dm + c] = row[dm + h * DH + c];
    cache_v[cbase + (int64_t)p * dm + c] = row[2 * dm + h * DH + c];
  }
  __syncthreads();
  float mx = -FLT_MAX;
  for (int t = tid; t <= p; t += 256) {
    const float* kr = cache_k + cbase + (int64_t)t * dm;
    float s = 0.f;
    for (int c = 0; c < DH; ++c) s = fmaf(q[c], kr[c], s);
    pr[t] = s;
    mx = fmaxf(mx, s);
  }
  mx = warp_max(mx);
  if (lane == 0) red[w] = mx;
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float sum = 0.f;
  for (int t = tid; t <= p; t += 256) {
    const float e = expf(pr[t] - mx);
    pr[t] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[w] = sum;
  __syncthreads();
  sum = 0.f;
  for (int i = 0; i < 8; ++i) sum += red[i];
  // out[c] = sum_t p_t V[t][c] / sum: the 8 warps split the positions, lanes the dims
  for (int c = lane; c < DH; c += 32) {
    float a = 0.f;
    for (int t = w; t <= p; t += 8) a = fmaf(pr[t], cache_v[cbase + (int64_t)t * dm + c], a);
    part_s[w][c] = a;
  }
  __syncthreads();
  for (int c = tid; c < DH; c += 256) {
    float a = 0.f;
    for (int i = 0; i < 8; ++i) a += part_s[i][c];
    out[b * dm + h * DH + c] = a / sum;
  }
}

// y += z (memory_ffn: the feed-forward and the memory read both feed the residual, model.py:97-121).
__global__ void __launch_bounds__(256) add_kernel(float* __restrict__ y, const float* __restrict__ z, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] += z[i];
}

// Tied logits (model.py:125, embed.attend): C [M, N] = h [M, K] . E [N, K]^T.
// One warp per output column n (the row E[n] read once, coalesced), up to
// 8 rows of h per CTA staged in shared memory; lanes over K, then a warp sum.
constexpr int LG_M = 8;
__global__ void __launch_bounds__(256) logits_gemv_kernel(const float* __restrict__ h, const float* __restrict__ E,
                                                          float* __restrict__ C, int64_t M, int N, int K) {
  extern __shared__ float hs[];   // [LG_M][K]
  const int64_t m0 = (int64_t)blockIdx.y * LG_M;
  const int rows = (int)(M - m0 < LG_M ? M - m0 : LG_M);
  for (int e = threadIdx.x; e < rows * K; e += blockDim.x) hs[e] = h[m0 * K + e];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (n >= N) return;
  float acc[LG_M];
#pragma unroll
  for (int i = 0; i < LG_M; ++i) acc[i] = 0.f;
  const float* er = E + (int64_t)n * K;
  for (int k = lane; k < K; k += 32) {
    const float e = __ldg(er + k);
#pragma unroll
    for (int i = 0; i < LG_M; ++i)
      if (i < rows) acc[i] = fmaf(hs[i * K + k], e, acc[i]);
  }
#pragma unroll
  for (int i = 0; i < LG_M; ++i) {
    if (i >= rows) break;
    const float v = warp_sum(acc[i]);
    if (lane == 0) C[(m0 + i) * N + n] = v;
  }
}

// Keeps the first non-zero status of a model call: a memory-layer call
// resets its own status word, so its code is copied into the model's.
__global__ void merge_status_kernel(const int* __restrict__ from, int* __restrict__ to) {
  if (*from != 0 && *to == 0) *to = *from;
}

}  // namespace

bool attn_supported(int head_dim) { return head_dim == 32 || head_dim == 64; }

cudaError_t launch_embed(const int* tokens, int64_t M, int T, const int* pos, const float* E, const float* Pe, int V,
                         int dm, int max_len, float* x, int* err, cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  embed_kernel<<<(unsigned)((M + 7) / 8), 256, 0, s>>>(tokens, M, T, pos, E, Pe, V, dm, max_len, x, err);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_add_ln(float* x, const float* y, const float* scale, const float* bias, float* h, int64_t M, int dm,
                          cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  if (dm > 32 * LN_MAX) return cudaErrorInvalidValue;
  add_ln_kernel<<<(unsigned)((M + 7) / 8), 256, 0, s>>>(x, y, scale, bias, h, M, dm);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_attn_prefill(const float* qkv, float* out, int64_t B, int T, int H, int DH, cudaStream_t s) {
  if (B == 0 || T == 0) return cudaSuccess;
  const dim3 grid((unsigned)((T + AQ - 1) / AQ), (unsigned)H, (unsigned)B);
  if (DH == 64)
    attn_prefill_kernel<64><<<grid, 256, 0, s>>>(qkv, out, T, H);
  else if (DH == 32)
    attn_prefill_kernel<32><<<grid, 256, 0, s>>>(qkv, out, T, H);
  else
    return cudaErrorInvalidValue;
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_attn_decode(const float* qkv, float* cache_k, float* cache_v, const int* pos, int max_len,
                               int64_t B, int H, int DH, float* out, int* err, cudaStream_t s) {
  if (B == 0) return cudaSuccess;
  const dim3 grid((unsigned)H, (unsigned)B);
  const size_t smem = sizeof(float) * (DH + max_len);
  if (DH == 64)
    attn_decode_kernel<64><<<grid, 256, smem, s>>>(qkv, cache_k, cache_v, pos, max_len, H, out, err);
  else if (DH == 32)
    attn_decode_kernel<32><<<grid, 256, smem, s>>>(qkv, cache_k, cache_v, pos, max_len, H, out, err);
  else
    return cudaErrorInvalidValue;
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_add(float* y, const float* z, int64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int64_t blocks = (n + 255) / 256;
  add_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, s>>>(y, z, n);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_logits_gemv(const float* h, const float* E, float* C, int64_t M, int N, int K, cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  const size_t smem = sizeof(float) * LG_M * K;
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  logits_gemv_kernel<<<dim3((unsigned)((N + 7) / 8), (unsigned)((M + LG_M - 1) / LG_M)), 256, smem, s>>>(h, E, C, M,
                                                                                                       N, K);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_merge_status(const int* from, int* to, cudaStream_t s) {
  merge_status_kernel<<<1, 1, 0, s>>>(from, to);
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
