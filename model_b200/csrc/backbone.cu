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
// (x - mean) * (rsqrt(var + eps) * scale) + bias).  One warp per row, VPL
// values per lane (d_model = 32 * VPL), 16-byte accesses when VPL % 4 == 0.
template <int VPL>
__global__ void __launch_bounds__(256) add_ln_kernel(float* __restrict__ x, const float* __restrict__ y,
                                                     const float* __restrict__ scale,
                                                     const float* __restrict__ bias, float* __restrict__ h,
                                                     int64_t M) {
  constexpr int dm = 32 * VPL;
  constexpr int V4 = VPL % 4 == 0 ? 4 : 1;   // elements per access
  const int64_t m = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (m >= M) return;
  float v[VPL];
  float s = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; i += V4) {
    const int j = (i / V4) * 32 * V4 + lane * V4;   // V4 consecutive columns per access
    if constexpr (V4 == 4) {
      float4 a = *reinterpret_cast<const float4*>(x + m * dm + j);
      if (y) {
        const float4 b = *reinterpret_cast<const float4*>(y + m * dm + j);
        a = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
        *reinterpret_cast<float4*>(x + m * dm + j) = a;
      }
      v[i] = a.x;
      v[i + 1] = a.y;
      v[i + 2] = a.z;
      v[i + 3] = a.w;
    } else {
      float a = x[m * dm + j];
      if (y) {
        a += y[m * dm + j];
        x[m * dm + j] = a;
      }
      v[i] = a;
    }
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    s += v[i];
    s2 = fmaf(v[i], v[i], s2);
  }
  s = warp_sum(s);
  s2 = warp_sum(s2);
  const float mean = s / (float)dm;
  const float var = fmaxf(0.f, s2 / (float)dm - mean * mean);
  const float r = 1.0f / sqrtf(var + 1e-6f);
#pragma unroll
  for (int i = 0; i < VPL; i += V4) {
    const int j = (i / V4) * 32 * V4 + lane * V4;
#pragma unroll
    for (int t = 0; t < V4; ++t) h[m * dm + j + t] = (v[i + t] - mean) * (r * scale[j + t]) + bias[j + t];
  }
}

// Causal self-attention of whole sequences (model.py:88-95, flax
// dot_product_attention): qkv [B*T, 3*dm] with the query, key and value of
// head h at columns h*DH, dm + h*DH and 2*dm + h*DH; out [B*T, dm] in the
// same head-major order.  A CTA takes 64 queries of one (batch, head) and
// walks 64-key tiles up to the diagonal with an online softmax (running max
// and sum in float32).  Both products are register-blocked float32 GEMM
// tiles on 256 threads: S = Q K^T with a 4 x 4 block per thread (16-byte
// shared-memory loads along the head dimension), then O += P V with a
// 4-row x DH/16-column block per thread; the row statistics sit in shared
// memory between the two.
constexpr int AT = 64;   // queries and keys per tile

template <int DH>
__global__ void __launch_bounds__(256) attn_prefill_kernel(const float* __restrict__ qkv, float* __restrict__ out,
                                                           int T, int H) {
  constexpr int LD = DH + 4;      // row stride of Q / K / V tiles (16-byte aligned rows)
  constexpr int LS = AT + 4;      // row stride of the score tile
  constexpr int OC = DH / 16;     // output columns per thread
  extern __shared__ float4 asm_raw[];
  float* qs = reinterpret_cast<float*>(asm_raw);   // [AT][LD], pre-divided by sqrt(DH)
  float* ks = qs + AT * LD;                          // [AT][LD]
  float* vs = ks + AT * LD;                          // [AT][LD]
  float* ps = vs + AT * LD;                          // [AT][LS] scores, then probabilities
  float* mrow = ps + AT * LS;                        // [AT] running max
  float* lrow = mrow + AT;                           // [AT] running sum
  float* crow = lrow + AT;                           // [AT] this tile's rescale of O
  const int dm = H * DH, ld = 3 * dm;
  const int q0 = blockIdx.x * AT, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const float rs = sqrtf((float)DH);
  for (int e = tid; e < AT * DH / 4; e += 256) {
    const int r = e / (DH / 4), c = (e - r * (DH / 4)) * 4;
    const int t = q0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < T) v = *reinterpret_cast<const float4*>(qkv + (b * T + t) * ld + h * DH + c);
    *reinterpret_cast<float4*>(qs + r * LD + c) = make_float4(v.x / rs, v.y / rs, v.z / rs, v.w / rs);
  }
  if (tid < AT) {
    mrow[tid] = -FLT_MAX;
    lrow[tid] = 0.f;
  }
  float o[4][OC];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < OC; ++j) o[i][j] = 0.f;
  const int kend = min(T, q0 + AT);
  for (int k0 = 0; k0 < kend; k0 += AT) {
    __syncthreads();   // previous tile's P / V consumed
    for (int e = tid; e < AT * DH / 4; e += 256) {
      const int r = e / (DH / 4), c = (e - r * (DH / 4)) * 4;
      const int t = k0 + r;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (t < T) {
        const float* row = qkv + (b * T + t) * ld + h * DH + c;
        kv = *reinterpret_cast<const float4*>(row + dm);
        vv = *reinterpret_cast<const float4*>(row + 2 * dm);
      }
      *reinterpret_cast<float4*>(ks + r * LD + c) = kv;
      *reinterpret_cast<float4*>(vs + r * LD + c) = vv;
    }
    __syncthreads();
    // S = Q K^T: thread block rows ty + 16 i, columns tx + 16 j
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
    for (int c = 0; c < DH; c += 4) {
      float4 a[4], bk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(qs + (ty + 16 * i) * LD + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) bk[j] = *reinterpret_cast<const float4*>(ks + (tx + 16 * j) * LD + c);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sc[i][j] = fmaf(a[i].x, bk[j].x, sc[i][j]);
          sc[i][j] = fmaf(a[i].y, bk[j].y, sc[i][j]);
          sc[i][j] = fmaf(a[i].z, bk[j].z, sc[i][j]);
          sc[i][j] = fmaf(a[i].w, bk[j].w, sc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tq = q0 + ty + 16 * i, tk = k0 + tx + 16 * j;
        ps[(ty + 16 * i) * LS + tx + 16 * j] = (tk <= tq && tk < T) ? sc[i][j] : -FLT_MAX;   // causal mask
      }
    __syncthreads();
    // online softmax per row: 4 threads per row, 16 columns each
    {
      const int r = tid >> 2, part = tid & 3;
      float* pr = ps + r * LS + part * 16;
      float mt = -FLT_MAX;
#pragma unroll
      for (int c = 0; c < 16; ++c) mt = fmaxf(mt, pr[c]);
      mt = fmaxf(mt, __shfl_xor_sync(FULL, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(FULL, mt, 2));
      const float mold = mrow[r];
      const float mnew = fmaxf(mold, mt);
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float p = pr[c] == -FLT_MAX ? 0.f : expf(pr[c] - mnew);
        pr[c] = p;
        sum += p;
      }
      sum += __shfl_xor_sync(FULL, sum, 1);
      sum += __shfl_xor_sync(FULL, sum, 2);
      __syncwarp();
      if (part == 0) {
        const float corr = mold == -FLT_MAX ? 0.f : expf(mold - mnew);
        crow[r] = corr;
        lrow[r] = lrow[r] * corr + sum;
        mrow[r] = mnew;
      }
    }
    __syncthreads();
    // O = O * corr + P V: thread rows ty + 16 i, columns tx * OC .. + OC
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float cr = crow[ty + 16 * i];
#pragma unroll
      for (int j = 0; j < OC; ++j) o[i][j] *= cr;
    }
#pragma unroll 2
    for (int k = 0; k < AT; k += 4) {
      float4 pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = *reinterpret_cast<const float4*>(ps + (ty + 16 * i) * LS + k);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        float vr[OC];
        if constexpr (OC % 4 == 0) {
#pragma unroll
          for (int j = 0; j < OC; j += 4) {
            const float4 v4 = *reinterpret_cast<const float4*>(vs + (k + kk) * LD + tx * OC + j);
            vr[j] = v4.x;
            vr[j + 1] = v4.y;
            vr[j + 2] = v4.z;
            vr[j + 3] = v4.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < OC; j += 2) {
            const float2 v2 = *reinterpret_cast<const float2*>(vs + (k + kk) * LD + tx * OC + j);
            vr[j] = v2.x;
            vr[j + 1] = v2.y;
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p = kk == 0 ? pv[i].x : kk == 1 ? pv[i].y : kk == 2 ? pv[i].z : pv[i].w;
#pragma unroll
          for (int j = 0; j < OC; ++j) o[i][j] = fmaf(p, vr[j], o[i][j]);
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ty + 16 * i, tq = q0 + r;
    if (tq >= T) continue;
    const float inv = 1.0f / lrow[r];
    float* dst = out + (b * T + tq) * dm + h * DH + tx * OC;
#pragma unroll
    for (int j = 0; j < OC; j += 2)
      *reinterpret_cast<float2*>(dst + j) = make_float2(o[i][j] * inv, o[i][j + 1] * inv);
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
  const unsigned grid = (unsigned)((M + 7) / 8);
  switch (dm) {
    case 32: add_ln_kernel<1><<<grid, 256, 0, s>>>(x, y, scale, bias, h, M); break;
    case 64: add_ln_kernel<2><<<grid, 256, 0, s>>>(x, y, scale, bias, h, M); break;
    case 128: add_ln_kernel<4><<<grid, 256, 0, s>>>(x, y, scale, bias, h, M); break;
    case 256: add_ln_kernel<8><<<grid, 256, 0, s>>>(x, y, scale, bias, h, M); break;
    case 512: add_ln_kernel<16><<<grid, 256, 0, s>>>(x, y, scale, bias, h, M); break;
    case 1024: add_ln_kernel<32><<<grid, 256, 0, s>>>(x, y, scale, bias, h, M); break;
    default: return cudaErrorInvalidValue;
  }
  count_launch();
  return cudaGetLastError();
}

bool ln_supported(int dm) { return dm == 32 || dm == 64 || dm == 128 || dm == 256 || dm == 512 || dm == 1024; }

template <int DH>
cudaError_t attn_prefill_dh(const float* qkv, float* out, int64_t B, int T, int H, cudaStream_t s) {
  const size_t smem = sizeof(float) * (3 * AT * (DH + 4) + AT * (AT + 4) + 3 * AT);
  const cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((T + AT - 1) / AT), (unsigned)H, (unsigned)B);
  attn_prefill_kernel<DH><<<grid, 256, smem, s>>>(qkv, out, T, H);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_attn_prefill(const float* qkv, float* out, int64_t B, int T, int H, int DH, cudaStream_t s) {
  if (B == 0 || T == 0) return cudaSuccess;
  if (DH == 64) return attn_prefill_dh<64>(qkv, out, B, T, H, s);
  if (DH == 32) return attn_prefill_dh<32>(qkv, out, B, T, H, s);
  return cudaErrorInvalidValue;
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
