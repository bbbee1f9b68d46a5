// C ABI of the language model around the memory layer: memlayer_model_forward
// (MemoryPoolLM.__call__, memory_pool_model/model.py:41-127, inference) and
// memlayer_model_decode_step (one Generator step, generate.py:31-34).  The
// memory layers are memlayer_layer_forward calls on the shared pool.
#include <stdint.h>
#include <string.h>

#include "backbone.cuh"
#include "memlayer.h"

namespace ml {
void count_launch(int n);
cudaError_t launch_split(const float* x, int64_t n, float* hi, float* lo, cudaStream_t s);
cudaError_t launch_transpose_split(const float* W, int K, int N, float* hi, float* lo, int row0, cudaStream_t s);
}  // namespace ml

namespace {

using namespace ml;

constexpr size_t MALIGN = 256;
size_t mup(size_t x) { return (x + MALIGN - 1) / MALIGN * MALIGN; }

#define MM_TRY(x)                                    \
  do {                                               \
    cudaError_t e_ = (x);                            \
    if (e_ != cudaSuccess) return MEMLAYER_ERR_CUDA; \
  } while (0)

struct ModelDims {
  int V, L, dm, H, dh, F, max_len;
  uint32_t mem;
  bool mem_ffn, any_ffn;
};

int check_model(const memlayer_model_config* c, ModelDims* d) {
  if (!c) return MEMLAYER_ERR_BAD_POINTER;
  if (c->vocab_size < 1 || c->max_len < 1 || c->d_model < 1 || c->n_layers < 0 || c->n_layers > MEMLAYER_MAX_LAYERS ||
      c->n_heads < 1 || c->ffn_mult < 1 || c->d_model % c->n_heads)
    return MEMLAYER_ERR_BAD_SHAPE;
  const int dh = c->d_model / c->n_heads;
  if (!attn_supported(dh) || !ln_supported(c->d_model)) return MEMLAYER_ERR_UNSUPPORTED;
  if (c->n_layers < 32 && (c->memory_layers >> c->n_layers)) return MEMLAYER_ERR_BAD_SHAPE;
  d->V = c->vocab_size;
  d->L = c->n_layers;
  d->dm = c->d_model;
  d->H = c->n_heads;
  d->dh = dh;
  d->F = c->d_model * c->ffn_mult;
  d->max_len = c->max_len;
  d->mem = c->memory_layers;
  d->mem_ffn = c->memory_ffn != 0;
  d->any_ffn = false;
  for (int i = 0; i < d->L; ++i)
    if (!((d->mem >> i) & 1u) || d->mem_ffn) d->any_ffn = true;
  if (d->mem && c->pool.d_model != c->d_model) return MEMLAYER_ERR_BAD_SHAPE;
  return MEMLAYER_OK;
}

bool is_mem(const ModelDims& d, int i) { return (d.mem >> i) & 1u; }

memlayer_config pool_cfg(const memlayer_model_config* c, int64_t M) {
  memlayer_config p = c->pool;
  p.tokens = M;
  p.d_model = c->d_model;
  return p;
}

// Workspace regions for M rows.
struct ModelWork {
  size_t o_x, o_h, o_y, o_y2, o_qkv, o_att, o_mid, o_ahi, o_alo, o_whi, o_wlo, o_bias, o_layer, layer_bytes, bytes;
  bool tc;   // the Dense layers run on the tensor cores (enough rows)
};

int model_work(const memlayer_model_config* c, const ModelDims& d, int64_t M, ModelWork* w) {
  ModelWork r{};
  size_t off = 512;   // [256]: the call's status word (where memlayer_workspace_status reads it)
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += mup(bytes);
    return o;
  };
  const size_t row = sizeof(float) * (size_t)M;
  r.o_x = take(row * d.dm);
  r.o_h = take(row * d.dm);
  r.o_y = take(row * d.dm);
  r.o_y2 = take(row * d.dm);
  r.o_qkv = take(row * 3 * d.dm);
  r.o_att = take(row * d.dm);
  r.o_mid = take(d.any_ffn ? row * d.F : 0);
  const int kmax = d.any_ffn && d.F > d.dm ? d.F : d.dm;
  r.tc = dense_tc_supported(M, d.dm, d.dm);
  if (r.tc) {
    r.o_ahi = take(row * kmax);
    r.o_alo = take(row * kmax);
    size_t wmax = (size_t)d.V * d.dm;
    const size_t cand[] = {(size_t)3 * d.dm * d.dm, (size_t)d.dm * d.dm, (size_t)d.F * d.dm};
    for (size_t x : cand) wmax = x > wmax ? x : wmax;
    r.o_whi = take(sizeof(float) * wmax);
    r.o_wlo = take(sizeof(float) * wmax);
  }
  r.o_bias = take(sizeof(float) * 3 * d.dm);
  r.layer_bytes = 0;
  if (d.mem) {
    const memlayer_config p = pool_cfg(c, M);
    int st = memlayer_layer_workspace_size(&p, &r.layer_bytes);
    if (st) return st;
  }
  r.o_layer = take(r.layer_bytes);
  r.bytes = off;
  *w = r;
  return MEMLAYER_OK;
}

struct Ctx {
  char* ws;
  const ModelWork* W;
  cudaStream_t s;
  int* err;
  float* f(size_t off) const { return reinterpret_cast<float*>(ws + off); }
};

// C [M, N] = act(A [M, K] . W + bias).  W is [K, N] (a Dense kernel), or
// [N, K] when nk (the tied embedding).  Tensor cores (3xTF32, operands split
// into the workspace) for enough rows, the SIMT GEMM / GEMV otherwise.
int dense(const Ctx& x, const float* A, int64_t M, int K, const float* W, bool nk, const float* bias, int N, float* C,
          int act) {
  if (M == 0) return MEMLAYER_OK;
  if (x.W->tc && dense_tc_supported(M, K, N)) {
    float *ahi = x.f(x.W->o_ahi), *alo = x.f(x.W->o_alo), *whi = x.f(x.W->o_whi), *wlo = x.f(x.W->o_wlo);
    MM_TRY(launch_split(A, M * K, ahi, alo, x.s));
    if (nk)
      MM_TRY(launch_split(W, (int64_t)N * K, whi, wlo, x.s));
    else
      MM_TRY(launch_transpose_split(W, K, N, whi, wlo, 0, x.s));
    MM_TRY(launch_dense_tc(ahi, alo, M, K, whi, wlo, N, bias, C, act, x.err, x.s));
    return MEMLAYER_OK;
  }
  if (nk) {
    if (bias || act != ACT_NONE) return MEMLAYER_ERR_UNSUPPORTED;
    MM_TRY(launch_logits_gemv(A, W, C, M, N, K, x.s));
    return MEMLAYER_OK;
  }
  MM_TRY(launch_gemm_act(A, W, bias, C, M, N, K, act, x.s));
  return MEMLAYER_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_params(const memlayer_model_config* c, const ModelDims& d, const memlayer_model_params* p) {
  if (!p || !p->embedding || !p->pos_embed || !p->ln_final_scale || !p->ln_final_bias) return MEMLAYER_ERR_BAD_POINTER;
  if (d.L > 0 && !p->layers) return MEMLAYER_ERR_BAD_POINTER;
  for (int i = 0; i < d.L; ++i) {
    const memlayer_block_params& b = p->layers[i];
    if (!b.ln_attn_scale || !b.ln_attn_bias || !b.w_qkv || !b.w_attn_out || !b.ln_ffn_scale || !b.ln_ffn_bias)
      return MEMLAYER_ERR_BAD_POINTER;
    if ((!is_mem(d, i) || d.mem_ffn) && (!b.w_ffn_in || !b.w_ffn_out)) return MEMLAYER_ERR_BAD_POINTER;
    if (is_mem(d, i) && (!b.w_router || !b.w_gate || !b.w_out)) return MEMLAYER_ERR_BAD_POINTER;
  }
  if (d.mem && (!p->sub_keys || !p->log_temperature || !p->values)) return MEMLAYER_ERR_BAD_POINTER;
  (void)c;
  return MEMLAYER_OK;
}

// The feed-forward / memory half of layer i on h -> y (model.py:96-121).
int block_tail(const memlayer_model_config* c, const ModelDims& d, const memlayer_model_params* p, int i,
               const Ctx& x, int64_t M) {
  const memlayer_block_params& b = p->layers[i];
  float *h = x.f(x.W->o_h), *y = x.f(x.W->o_y), *y2 = x.f(x.W->o_y2), *mid = x.f(x.W->o_mid);
  const bool ffn = !is_mem(d, i) || d.mem_ffn;
  int st;
  if (ffn) {
    if ((st = dense(x, h, M, d.dm, b.w_ffn_in, false, b.b_ffn_in, d.F, mid, ACT_GELU))) return st;   // model.py:103
    if ((st = dense(x, mid, M, d.F, b.w_ffn_out, false, b.b_ffn_out, d.dm, y, ACT_NONE))) return st;  // model.py:104
  }
  if (is_mem(d, i)) {
    const memlayer_config pc = pool_cfg(c, M);
    memlayer_layer_args a{};
    a.h = h;
    a.w_router = b.w_router;
    a.b_router = b.b_router;
    a.w_gate = b.w_gate;
    a.b_gate = b.b_gate;
    a.w_out = b.w_out;
    a.b_out = b.b_out;
    a.y = ffn ? y2 : y;
    a.pool.sub_keys = p->sub_keys;
    a.pool.log_temperature = p->log_temperature;
    a.pool.values = p->values;
    a.pool.noise_scale = 1.f;
    char* lws = x.ws + x.W->o_layer;
    if ((st = memlayer_layer_forward(&pc, &a, lws, x.W->layer_bytes, x.s))) return st;   // model.py:108-120
    MM_TRY(launch_merge_status(reinterpret_cast<const int*>(lws + 256), x.err, x.s));
    if (ffn) MM_TRY(launch_add(y, y2, M * d.dm, x.s));
  }
  return MEMLAYER_OK;
}

}  // namespace

extern "C" {

int32_t memlayer_model_workspace_size(const memlayer_model_config* cfg, int64_t tokens, size_t* bytes) {
  ModelDims d;
  int st = check_model(cfg, &d);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  if (tokens < 0) return MEMLAYER_ERR_BAD_SHAPE;
  ModelWork w;
  if ((st = model_work(cfg, d, tokens, &w))) return st;
  *bytes = w.bytes;
  return MEMLAYER_OK;
}

int32_t memlayer_model_cache_size(const memlayer_model_config* cfg, int64_t batch, size_t* bytes) {
  ModelDims d;
  int st = check_model(cfg, &d);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  if (batch < 0) return MEMLAYER_ERR_BAD_SHAPE;
  *bytes = sizeof(float) * (size_t)d.L * 2 * (size_t)batch * d.max_len * d.dm;
  return MEMLAYER_OK;
}

int32_t memlayer_model_forward(const memlayer_model_config* cfg, const memlayer_model_params* p,
                               const int32_t* tokens, int64_t batch, int64_t seq, float* logits, void* workspace,
                               size_t workspace_bytes, void* stream) {
  ModelDims d;
  int st = check_model(cfg, &d);
  if (st) return st;
  if (batch < 0 || seq < 0 || seq > d.max_len) return MEMLAYER_ERR_BAD_SHAPE;
  const int64_t M = batch * seq;
  if ((st = check_params(cfg, d, p))) return st;
  if (M > 0 && (!tokens || !logits)) return MEMLAYER_ERR_BAD_POINTER;
  ModelWork W;
  if ((st = model_work(cfg, d, M, &W))) return st;
  if (!workspace || workspace_bytes < W.bytes || (reinterpret_cast<uintptr_t>(workspace) % MALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  const cudaStream_t s = (cudaStream_t)stream;
  Ctx x{(char*)workspace, &W, s, reinterpret_cast<int*>((char*)workspace + 256)};
  MM_TRY(cudaMemsetAsync(x.err, 0, sizeof(int), s));
  if (M == 0) return MEMLAYER_OK;
  float *X = x.f(W.o_x), *h = x.f(W.o_h), *y = x.f(W.o_y), *qkv = x.f(W.o_qkv), *att = x.f(W.o_att);
  MM_TRY(launch_embed(tokens, M, (int)seq, nullptr, p->embedding, p->pos_embed, d.V, d.dm, d.max_len, X, x.err, s));
  for (int i = 0; i < d.L; ++i) {
    const memlayer_block_params& b = p->layers[i];
    MM_TRY(launch_add_ln(X, i ? y : nullptr, b.ln_attn_scale, b.ln_attn_bias, h, M, d.dm, s));   // model.py:87
    if ((st = dense(x, h, M, d.dm, b.w_qkv, false, b.b_qkv, 3 * d.dm, qkv, ACT_NONE))) return st;
    MM_TRY(launch_attn_prefill(qkv, att, batch, (int)seq, d.H, d.dh, s));                      // model.py:88-94
    if ((st = dense(x, att, M, d.dm, b.w_attn_out, false, b.b_attn_out, d.dm, y, ACT_NONE))) return st;
    MM_TRY(launch_add_ln(X, y, b.ln_ffn_scale, b.ln_ffn_bias, h, M, d.dm, s));               // model.py:95-96
    if ((st = block_tail(cfg, d, p, i, x, M))) return st;                                      // model.py:97-121
  }
  MM_TRY(launch_add_ln(X, d.L ? y : nullptr, p->ln_final_scale, p->ln_final_bias, h, M, d.dm, s));  // model.py:124
  return dense(x, h, M, d.dm, p->embedding, true, nullptr, d.V, logits, ACT_NONE);              // model.py:125
}

int32_t memlayer_model_decode_step(const memlayer_model_config* cfg, const memlayer_model_params* p,
                                   const int32_t* tokens, int64_t batch, const int32_t* pos, void* cache,
                                   float* logits, void* workspace, size_t workspace_bytes, void* stream) {
  ModelDims d;
  int st = check_model(cfg, &d);
  if (st) return st;
  if (batch < 0) return MEMLAYER_ERR_BAD_SHAPE;
  const int64_t M = batch;
  if ((st = check_params(cfg, d, p))) return st;
  if (M > 0 && (!tokens || !logits || !pos || (d.L > 0 && !cache))) return MEMLAYER_ERR_BAD_POINTER;
  if (!al16(cache)) return MEMLAYER_ERR_BAD_POINTER;
  ModelWork W;
  if ((st = model_work(cfg, d, M, &W))) return st;
  if (!workspace || workspace_bytes < W.bytes || (reinterpret_cast<uintptr_t>(workspace) % MALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  const cudaStream_t s = (cudaStream_t)stream;
  Ctx x{(char*)workspace, &W, s, reinterpret_cast<int*>((char*)workspace + 256)};
  MM_TRY(cudaMemsetAsync(x.err, 0, sizeof(int), s));
  if (M == 0) return MEMLAYER_OK;
  float *X = x.f(W.o_x), *h = x.f(W.o_h), *y = x.f(W.o_y), *qkv = x.f(W.o_qkv), *att = x.f(W.o_att);
  MM_TRY(launch_embed(tokens, M, 1, pos, p->embedding, p->pos_embed, d.V, d.dm, d.max_len, X, x.err, s));
  const size_t layer_floats = (size_t)2 * M * d.max_len * d.dm;
  for (int i = 0; i < d.L; ++i) {
    const memlayer_block_params& b = p->layers[i];
    float* ck = reinterpret_cast<float*>(cache) + (size_t)i * layer_floats;
    float* cv = ck + (size_t)M * d.max_len * d.dm;
    MM_TRY(launch_add_ln(X, i ? y : nullptr, b.ln_attn_scale, b.ln_attn_bias, h, M, d.dm, s));
    if ((st = dense(x, h, M, d.dm, b.w_qkv, false, b.b_qkv, 3 * d.dm, qkv, ACT_NONE))) return st;
    MM_TRY(launch_attn_decode(qkv, ck, cv, pos, d.max_len, M, d.H, d.dh, att, x.err, s));
    if ((st = dense(x, att, M, d.dm, b.w_attn_out, false, b.b_attn_out, d.dm, y, ACT_NONE))) return st;
    MM_TRY(launch_add_ln(X, y, b.ln_ffn_scale, b.ln_ffn_bias, h, M, d.dm, s));
    if ((st = block_tail(cfg, d, p, i, x, M))) return st;
  }
  MM_TRY(launch_add_ln(X, d.L ? y : nullptr, p->ln_final_scale, p->ln_final_bias, h, M, d.dm, s));
  return dense(x, h, M, d.dm, p->embedding, true, nullptr, d.V, logits, ACT_NONE);
}

}  // extern "C"
