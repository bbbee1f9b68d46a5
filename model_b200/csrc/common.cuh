// Shared device helpers and the internal launch descriptors of the memory layer.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "memlayer.h"

namespace ml {

constexpr unsigned FULL = 0xffffffffu;

// Shapes of one call, resolved and validated on the host.
struct Dims {
  int64_t M;       // tokens
  int H;           // heads
  int n;           // sub-keys per half
  int dk;          // d_key
  int half;        // d_key / 2
  int d;           // d_value
  int k;           // top_k
  int kmax;        // compiled list length >= k (4, 8, 16 or 32)
  int dm;          // d_model (layer entry)
  int vdtype;      // memlayer_dtype
  int64_t N;       // n * n
  float noise_coef;  // routing_noise * noise_scale (0 = no selection noise)
  bool noisy;        // selection noise applied
  bool qscale;       // query_scale
  bool btgrad;       // balance_temperature_grad
  bool shuffle;      // shuffle_reads
};

// Device pointers carved out of the caller's workspace.
struct Work {
  float* keys_n = nullptr;     // [H,2,n,half] unit sub-keys
  float* k_hi = nullptr;       // [H*2,n,half] rna_tf32(keys_n)          (tensor-core path)
  float* k_lo = nullptr;       // [H*2,n,half] rna_tf32(keys_n - k_hi)
  float* q_hi = nullptr;       // [H*2,M,half] rna_tf32(qn), codebook-major
  float* q_lo = nullptr;       // [H*2,M,half] rna_tf32(qn - q_hi)
  int* err = nullptr;          // [1] device error code (bounded waits)
  int* fin_ctr = nullptr;      // [1] blocks done in the aux reduction (reset by the prep kernels)
  double* fin_part = nullptr;  // [64] per-block partial sums of the aux reduction
  float* h_hi = nullptr;       // [M,dm] tf32 halves of the hidden state   (tensor-core projections)
  float* h_lo = nullptr;
  float* wrg_hi = nullptr;     // [H*dk + d, dm] router | gate kernels, K-major
  float* wrg_lo = nullptr;
  float* bias_rg = nullptr;    // [H*dk + d] router | gate biases
  float* wo_hi = nullptr;      // [dm, d] output kernel, K-major
  float* wo_lo = nullptr;
  float* memg_hi = nullptr;    // [M,d] tf32 halves of mem * gate
  float* memg_lo = nullptr;
  float* qn = nullptr;         // [M,H,2,half] unit query halves
  float* qlen = nullptr;       // [M,H,2] |q_half| / sqrt(half)
  int* sub_idx = nullptr;      // [M,H,2,k] stage-1 sub-key ids (selection order)
  float* sub_score = nullptr;  // [M,H,2,k] clean scores at sub_idx
  float* sub_sel = nullptr;    // [M,H,2,k] selection scores at sub_idx
  int* clean_idx = nullptr;    // [M,H,2,k] clean top-k (noisy calls with stats)
  float* row_max = nullptr;    // [M,H,2] max of the balance scores per row
  float* row_sum = nullptr;    // [M,H,2] sum of exp(p - max) per row
  float* p_part = nullptr;     // [tiles,H,2,n] per-tile column sums of softmax(p)
  float* clean_cnt = nullptr;  // [H,2,n] clean top-k counts
  float* top1_part = nullptr;  // [M*H] max weight per (token, head)
  float* scal = nullptr;       // [4] temperature, ...
  float* qraw = nullptr;       // [M,H*dk] router output (layer entry)
  float* gate = nullptr;       // [M,d] silu(h W_gate + b_gate) (layer entry)
  float* memg = nullptr;       // [M,d] mem * gate (layer entry)
  int* slots = nullptr;        // [M,H,k] when the caller passes none
  float* weights = nullptr;    // [M,H,k] when the caller passes none
  float* out = nullptr;        // [M,d] when the caller passes none
  int* own_cnt = nullptr;      // [M,world] entries each owner rank gathers (row-sharded pool)
  float* small = nullptr;      // slice top-k lists of the few-token score path
  double* bal_part = nullptr;  // [H*2*n/32] per-block sums of the balance loss
  int* bal_ctr = nullptr;      // [1] blocks done in the balance-loss reduction (reset by its last block)
};

constexpr int SCORE_TM = 128;   // tokens per score tile
constexpr int SCORE_TN = 64;    // sub-keys per chunk

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

// Forward value of the straight-through temperature clamp (memory.py:141-146).
__device__ __forceinline__ float clamped_temperature(float log_t, float min_t, float max_t) {
  float lo = logf(min_t), hi = logf(max_t);
  float c = fminf(fmaxf(log_t, lo), hi);
  return expf(log_t + (c - log_t));
}

// Sorted insertion into a descending register list.  Precondition: s is
// strictly greater than v[KM-1] and i is larger than every index already in
// the list (keys are scanned in increasing order), so equal values keep the
// lower index first, as lax.top_k does.
template <int KM>
__device__ __forceinline__ void list_insert(float (&v)[KM], int (&ix)[KM], float s, int i) {
#pragma unroll
  for (int j = KM - 1; j >= 0; --j) {
    bool down = (j > 0) && (v[j - 1] < s);
    if (down) {
      v[j] = v[j - 1];
      ix[j] = ix[j - 1];
    } else if (v[j] < s) {
      v[j] = s;
      ix[j] = i;
    }
  }
}

template <int KM>
__device__ __forceinline__ void list_insert3(float (&v)[KM], int (&ix)[KM], float (&aux)[KM], float s, int i,
                                             float a) {
#pragma unroll
  for (int j = KM - 1; j >= 0; --j) {
    bool down = (j > 0) && (v[j - 1] < s);
    if (down) {
      v[j] = v[j - 1];
      ix[j] = ix[j - 1];
      aux[j] = aux[j - 1];
    } else if (v[j] < s) {
      v[j] = s;
      ix[j] = i;
      aux[j] = a;
    }
  }
}

// (value desc, index asc) ordering used by every top-k merge.
__device__ __forceinline__ bool ranks_before(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// Value-row element loads (float32 / float16 / bfloat16 storage, float32 math).
template <typename VT>
struct VecLoad;

template <>
struct VecLoad<float> {
  static constexpr int VEC = 4;
  __device__ __forceinline__ static void load(const float* p, float (&o)[4]) {
    float4 t = __ldg(reinterpret_cast<const float4*>(p));
    o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
  }
  __device__ __forceinline__ static float scalar(const float* p) { return __ldg(p); }
};

template <>
struct VecLoad<__half> {
  static constexpr int VEC = 8;
  __device__ __forceinline__ static void load(const __half* p, float (&o)[8]) {
    uint4 t = __ldg(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&t);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  __device__ __forceinline__ static float scalar(const __half* p) { return __half2float(p[0]); }
};

template <>
struct VecLoad<__nv_bfloat16> {
  static constexpr int VEC = 8;
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float (&o)[8]) {
    uint4 t = __ldg(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&t);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  __device__ __forceinline__ static float scalar(const __nv_bfloat16* p) { return __bfloat162float(p[0]); }
};

// memlayer_pool_forward without the intra-call overlap: every launch on
// `stream`, no event or library stream is created.
int32_t pool_forward_single_stream(const memlayer_config* cfg, const memlayer_pool_args* args, void* workspace,
                                   size_t workspace_bytes, void* stream);

// Counts every kernel launch made by this library (memlayer_kernel_launch_count).
void count_launch(int n = 1);

// ---- host-side launchers (one per kernel family) ----
cudaError_t launch_prep_keys(const Dims& D, const float* sub_keys, const float* log_t, float min_t, float max_t,
                             float* keys_n, float* k_hi, float* k_lo, float* scal, int* err, int* fin_ctr,
                             cudaStream_t s);
cudaError_t launch_normalize_queries(const Dims& D, const float* q, float* qn, float* qlen, float* q_hi,
                                     float* q_lo, cudaStream_t s);
bool score_tc_supported(const Dims& D);
// mtn > 0: only the 128-token tiles [mt0, mt0 + mtn); max_ctas > 0 caps the
// persistent grid (leaving SMs to a kernel running beside it)
cudaError_t launch_score_topk_tc(const Dims& D, const Work& W, const float* gumbel, bool want_balance,
                                 cudaStream_t s, int mt0 = 0, int mtn = 0, int max_ctas = 0);
cudaError_t launch_score_topk(const Dims& D, const Work& W, const float* gumbel, bool want_balance,
                              cudaStream_t s);
bool score_small_supported(const Dims& D);
size_t score_small_scratch_bytes(const Dims& D);
cudaError_t launch_score_small(const Dims& D, const Work& W, const float* gumbel, float* scratch, cudaStream_t s);
cudaError_t launch_balance(const Dims& D, const Work& W, float* balance_loss, cudaStream_t s);
cudaError_t launch_balance_tc(const Dims& D, const Work& W, int* planes, cudaStream_t s);
// count > 0: only tokens [m0, m0 + count)
cudaError_t launch_combine_gather(const Dims& D, const Work& W, const void* values, int* slots, float* weights,
                                  float* out, float* mem_gated, float* memg_hi, float* memg_lo, const float* gate,
                                  float* slot_counts, float* subkey_counts, cudaStream_t s, int64_t m0 = 0,
                                  int64_t count = 0);
bool proj_tc_supported(const Dims& D);
cudaError_t launch_split(const float* x, int64_t n, float* hi, float* lo, cudaStream_t s);
cudaError_t launch_transpose_split(const float* W, int K, int N, float* hi, float* lo, int row0, cudaStream_t s);
cudaError_t launch_concat_bias(const float* a, int na, const float* b, int nb, float* out, cudaStream_t s);
cudaError_t launch_router_gate_tc(const Dims& D, const Work& W, const float* bias_rg, float* qn_out, cudaStream_t s);
cudaError_t launch_out_tc(const Dims& D, const Work& W, const float* b_out, float* y, cudaStream_t s);
cudaError_t launch_finalize(const Dims& D, const Work& W, float* top1, float* temperature, cudaStream_t s);
cudaError_t launch_prep_layer(const Dims& D, const Work& W, const float* sub_keys, const float* log_t, float min_t,
                              float max_t, const float* h, const float* w_router, const float* b_router,
                              const float* w_gate, const float* b_gate, const float* w_out, cudaStream_t s);
cudaError_t launch_gemm(const float* A, const float* B, const float* bias, float* C, int64_t M, int N, int K,
                        bool silu, cudaStream_t s);
// Two products of the same A (C0 = A B0 (+ bias0, silu), C1 = A B1 ...): one
// launch for decode-size M, else two launch_gemm calls.
cudaError_t launch_gemm2(const float* A, const float* B0, const float* bias0, float* C0, int N0, bool silu0,
                         const float* B1, const float* bias1, float* C1, int N1, bool silu1, int64_t M, int K,
                         cudaStream_t s);

}  // namespace ml
