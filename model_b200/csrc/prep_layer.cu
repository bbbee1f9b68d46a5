// One-launch operand preparation for the tensor-core layer path: unit
// sub-keys (memory.py:139) with their tf32 halves, the temperature
// (memory.py:141-146), the Dense kernels transposed to K-major tf32 halves
// (router | gate concatenated, output), the concatenated biases and the tf32
// halves of the hidden state.  Blocks are partitioned by job.
#include "tc_common.cuh"

namespace ml {

namespace {

struct LayerPrep {
  const float* sub_keys;
  float* keys_n;
  float* k_hi;
  float* k_lo;
  int64_t key_rows;
  int half;
  const float* log_t;
  float min_t, max_t;
  float* scal;
  int* err;
  int* fin_ctr;
  const float* w_router;   // [dm, NR]
  const float* w_gate;     // [dm, d]
  const float* w_out;      // [d, dm]
  const float* b_router;   // [NR] or nullptr
  const float* b_gate;     // [d] or nullptr
  float* wrg_hi;
  float* wrg_lo;
  float* wo_hi;
  float* wo_lo;
  float* bias_rg;
  int dm, NR, d;
  const float* h;
  float* h_hi;
  float* h_lo;
  int64_t h_n;
  int nb_keys, nb_wr, nb_wg, nb_wo, nb_bias, nb_h;
};

__device__ __forceinline__ void split_store(float v, float* hi, float* lo, int64_t i) {
  const float a = tc::to_tf32(v);
  hi[i] = a;
  lo[i] = tc::to_tf32(v - a);
}

// W [K, N] row-major -> rows [row0, row0 + N) of a K-major matrix, tf32 halves.
__device__ __forceinline__ void transpose_tile(const float* W, int K, int N, float* hi, float* lo, int row0,
                                               int tile, float (*t)[33]) {
  const int tiles_x = (N + 31) / 32;
  const int n_base = (tile % tiles_x) * 32, k_base = (tile / tiles_x) * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int k = k_base + i, n = n_base + tx;
    t[i][tx] = (k < K && n < N) ? W[(int64_t)k * N + n] : 0.f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int n = n_base + i, k = k_base + tx;
    if (n < N && k < K) split_store(t[tx][i], hi, lo, (int64_t)(row0 + n) * K + k);
  }
}

__global__ void __launch_bounds__(256) prep_layer_kernel(LayerPrep P) {
  __shared__ float tile[32][33];
  int b = blockIdx.x;
  if (b < P.nb_keys) {
    // unit sub-keys: one warp per row (memory.py:30-31,139)
    if (b == 0 && threadIdx.x == 0) {
      P.scal[0] = clamped_temperature(P.log_t[0], P.min_t, P.max_t);
      *P.err = 0;
      *P.fin_ctr = 0;
    }
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)b * 8 + (threadIdx.x >> 5);
    if (row >= P.key_rows) return;
    const float* x = P.sub_keys + row * P.half;
    float ss = 0.f;
    for (int i = lane; i < P.half; i += 32) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + 1e-6f);
    for (int i = lane; i < P.half; i += 32) {
      const float v = x[i] * r;
      P.keys_n[row * P.half + i] = v;
      split_store(v, P.k_hi, P.k_lo, row * P.half + i);
    }
    return;
  }
  b -= P.nb_keys;
  if (b < P.nb_wr) return transpose_tile(P.w_router, P.dm, P.NR, P.wrg_hi, P.wrg_lo, 0, b, tile);
  b -= P.nb_wr;
  if (b < P.nb_wg) return transpose_tile(P.w_gate, P.dm, P.d, P.wrg_hi, P.wrg_lo, P.NR, b, tile);
  b -= P.nb_wg;
  if (b < P.nb_wo) return transpose_tile(P.w_out, P.d, P.dm, P.wo_hi, P.wo_lo, 0, b, tile);
  b -= P.nb_wo;
  if (b < P.nb_bias) {
    for (int i = b * 256 + threadIdx.x; i < P.NR + P.d; i += P.nb_bias * 256)
      P.bias_rg[i] = i < P.NR ? (P.b_router ? P.b_router[i] : 0.f) : (P.b_gate ? P.b_gate[i - P.NR] : 0.f);
    return;
  }
  b -= P.nb_bias;
  // hidden state: tf32 halves, float4 grid-stride over this job's blocks
  const int64_t n4 = P.h_n / 4;
  for (int64_t i = (int64_t)b * 256 + threadIdx.x; i < n4; i += (int64_t)P.nb_h * 256) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(P.h) + i);
    float4 hv, lv;
    hv.x = tc::to_tf32(v.x); lv.x = tc::to_tf32(v.x - hv.x);
    hv.y = tc::to_tf32(v.y); lv.y = tc::to_tf32(v.y - hv.y);
    hv.z = tc::to_tf32(v.z); lv.z = tc::to_tf32(v.z - hv.z);
    hv.w = tc::to_tf32(v.w); lv.w = tc::to_tf32(v.w - hv.w);
    reinterpret_cast<float4*>(P.h_hi)[i] = hv;
    reinterpret_cast<float4*>(P.h_lo)[i] = lv;
  }
  for (int64_t i = n4 * 4 + (int64_t)b * 256 + threadIdx.x; i < P.h_n; i += (int64_t)P.nb_h * 256)
    split_store(P.h[i], P.h_hi, P.h_lo, i);
}

}  // namespace

cudaError_t launch_prep_layer(const Dims& D, const Work& W, const float* sub_keys, const float* log_t, float min_t,
                              float max_t, const float* h, const float* w_router, const float* b_router,
                              const float* w_gate, const float* b_gate, const float* w_out, cudaStream_t s) {
  LayerPrep P{};
  P.sub_keys = sub_keys;
  P.keys_n = W.keys_n;
  P.k_hi = W.k_hi;
  P.k_lo = W.k_lo;
  P.key_rows = (int64_t)D.H * 2 * D.n;
  P.half = D.half;
  P.log_t = log_t;
  P.min_t = min_t;
  P.max_t = max_t;
  P.scal = W.scal;
  P.err = W.err;
  P.fin_ctr = W.fin_ctr;
  P.w_router = w_router;
  P.w_gate = w_gate;
  P.w_out = w_out;
  P.b_router = b_router;
  P.b_gate = b_gate;
  P.wrg_hi = W.wrg_hi;
  P.wrg_lo = W.wrg_lo;
  P.wo_hi = W.wo_hi;
  P.wo_lo = W.wo_lo;
  P.bias_rg = W.bias_rg;
  P.dm = D.dm;
  P.NR = D.H * D.dk;
  P.d = D.d;
  P.h = h;
  P.h_hi = W.h_hi;
  P.h_lo = W.h_lo;
  P.h_n = D.M * D.dm;
  // the hi / lo split of the keys is only read by the tensor-core score path
  if (!P.k_hi) return cudaErrorInvalidValue;
  P.nb_keys = (int)((P.key_rows + 7) / 8);
  P.nb_wr = ((P.NR + 31) / 32) * ((P.dm + 31) / 32);
  P.nb_wg = ((P.d + 31) / 32) * ((P.dm + 31) / 32);
  P.nb_wo = ((P.dm + 31) / 32) * ((P.d + 31) / 32);
  P.nb_bias = 1;
  int64_t hb = (P.h_n / 4 + 255) / 256;
  P.nb_h = (int)(hb < 148 * 4 ? (hb < 1 ? 1 : hb) : 148 * 4);
  const int blocks = P.nb_keys + P.nb_wr + P.nb_wg + P.nb_wo + P.nb_bias + P.nb_h;
  prep_layer_kernel<<<blocks, 256, 0, s>>>(P);
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
