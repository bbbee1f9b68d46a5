// C ABI of the memory layer (include/memlayer.h): argument validation,
// workspace layout and the launch sequence of one forward call.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>

#include <mutex>
#include <unordered_map>
#include <new>

#include "common.cuh"
#include "host_table.cuh"
#include "layer_bwd.cuh"
#include "keys.cuh"
#include "rowgrad.cuh"
#include "bal_bwd_tc.cuh"
#include "gemm_any.cuh"
#include "shard.cuh"

namespace ml {

static std::atomic<int64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

namespace {

constexpr size_t ALIGN = 256;

inline size_t up(size_t x) { return (x + ALIGN - 1) / ALIGN * ALIGN; }

struct Flags {
  bool layer = false;
  bool balance = false;   // balance_loss requested
  int world = 0;          // ranks of the row-sharded pool (0: single GPU)
};

int check_config(const memlayer_config* c, Dims* D, bool layer) {
  if (!c || !D) return MEMLAYER_ERR_BAD_POINTER;
  if (c->tokens < 0 || c->heads < 1 || c->heads > 32 || c->n_sub_keys < 1 || c->d_key < 2 || c->d_key % 2 ||
      c->d_value < 1 || c->top_k < 1 || c->top_k > c->n_sub_keys)
    return MEMLAYER_ERR_BAD_SHAPE;
  if (c->n_sub_keys > 46340) return MEMLAYER_ERR_BAD_SHAPE;       // n*n must fit int32 slot ids
  if (c->top_k > 32 || c->d_key > 256 || c->d_value > 1024) return MEMLAYER_ERR_UNSUPPORTED;
  if (c->values_dtype != MEMLAYER_F32 && c->values_dtype != MEMLAYER_F16 && c->values_dtype != MEMLAYER_BF16)
    return MEMLAYER_ERR_UNSUPPORTED;
  if (c->values_dtype != MEMLAYER_F32 && c->d_value % 8) return MEMLAYER_ERR_UNSUPPORTED;
  if (c->values_dtype == MEMLAYER_F32 && c->d_value % 4 && c->d_value > 256) return MEMLAYER_ERR_UNSUPPORTED;
  if (layer && c->d_model < 1) return MEMLAYER_ERR_BAD_SHAPE;
  if (!(c->min_temperature > 0.f) || !(c->max_temperature >= c->min_temperature)) return MEMLAYER_ERR_BAD_SHAPE;
  D->M = c->tokens;
  D->H = c->heads;
  D->n = c->n_sub_keys;
  D->dk = c->d_key;
  D->half = c->d_key / 2;
  D->d = c->d_value;
  D->k = c->top_k;
  D->kmax = c->top_k <= 4 ? 4 : c->top_k <= 8 ? 8 : c->top_k <= 16 ? 16 : 32;
  D->dm = c->d_model;
  D->vdtype = c->values_dtype;
  D->N = (int64_t)c->n_sub_keys * c->n_sub_keys;
  D->qscale = c->query_scale != 0;
  D->btgrad = c->balance_temperature_grad != 0;
  D->noise_coef = 0.f;
  D->noisy = false;
  D->shuffle = false;
  return MEMLAYER_OK;
}

// Carve the workspace (ws == nullptr: only measure).  Returns total bytes.
size_t layout(const Dims& D, const Flags& f, char* ws, Work* W) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> void* {
    void* p = ws ? ws + off : nullptr;
    off += up(bytes);
    return p;
  };
  const int64_t rows = D.M * D.H * 2;
  const int64_t tiles = (D.M + SCORE_TM - 1) / SCORE_TM;
  Work w;
  w.scal = (float*)take(4 * sizeof(float));
  w.err = (int*)take(sizeof(int));
  w.fin_ctr = (int*)take(sizeof(int));
  w.fin_part = (double*)take(sizeof(double) * 64);
  w.keys_n = (float*)take(sizeof(float) * D.H * 2 * D.n * D.half);
  w.qn = (float*)take(sizeof(float) * rows * D.half);
  // few tokens (decode): split-key score path; tensor-core tiles need many tokens
  const bool small = score_small_supported(D);
  if (small) w.small = (float*)take(score_small_scratch_bytes(D));
  if (score_tc_supported(D) && !small) {
    w.k_hi = (float*)take(sizeof(float) * D.H * 2 * D.n * D.half);
    w.k_lo = (float*)take(sizeof(float) * D.H * 2 * D.n * D.half);
    w.q_hi = (float*)take(sizeof(float) * rows * D.half);
    w.q_lo = (float*)take(sizeof(float) * rows * D.half);
  }
  w.qlen = (float*)take(sizeof(float) * rows);
  w.sub_idx = (int*)take(sizeof(int) * rows * D.k);
  w.sub_score = (float*)take(sizeof(float) * rows * D.k);
  w.sub_sel = (float*)take(sizeof(float) * rows * D.k);
  w.top1_part = (float*)take(sizeof(float) * D.M * D.H);
  if (f.balance) {
    w.clean_idx = (int*)take(sizeof(int) * rows * D.k);
    w.row_max = (float*)take(sizeof(float) * rows);
    w.row_sum = (float*)take(sizeof(float) * rows);
    w.p_part = (float*)take(sizeof(float) * tiles * 4 * D.H * 2 * D.n);   // 4 lane quarters per tile (TC pass)
    w.clean_cnt = (float*)take(sizeof(float) * D.H * 2 * D.n);
    w.bal_part = (double*)take(sizeof(double) * ((D.H * 2 * D.n + 31) / 32));
    w.bal_ctr = (int*)take(sizeof(int));
  }
  if (f.layer) {
    const int64_t NRD = (int64_t)D.H * D.dk + D.d;
    w.gate = (float*)take(sizeof(float) * D.M * D.d);
    if (proj_tc_supported(D)) {
      w.h_hi = (float*)take(sizeof(float) * D.M * D.dm);
      w.h_lo = (float*)take(sizeof(float) * D.M * D.dm);
      w.wrg_hi = (float*)take(sizeof(float) * NRD * D.dm);
      w.wrg_lo = (float*)take(sizeof(float) * NRD * D.dm);
      w.bias_rg = (float*)take(sizeof(float) * NRD);
      w.wo_hi = (float*)take(sizeof(float) * D.dm * D.d);
      w.wo_lo = (float*)take(sizeof(float) * D.dm * D.d);
      w.memg_hi = (float*)take(sizeof(float) * D.M * D.d);
      w.memg_lo = (float*)take(sizeof(float) * D.M * D.d);
    } else {
      w.qraw = (float*)take(sizeof(float) * D.M * D.H * D.dk);
      w.memg = (float*)take(sizeof(float) * D.M * D.d);
    }
    w.slots = (int*)take(sizeof(int) * D.M * D.H * D.k);
    w.weights = (float*)take(sizeof(float) * D.M * D.H * D.k);
  }
  if (f.world > 0) w.own_cnt = (int*)take(sizeof(int) * D.M * f.world);
  if (W) *W = w;
  return off;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_pool_args(const Dims& D, const memlayer_pool_args* a, bool layer) {
  if (!a) return MEMLAYER_ERR_BAD_POINTER;
  if (!a->sub_keys || !a->log_temperature || !a->values) return MEMLAYER_ERR_BAD_POINTER;
  if (D.M == 0) return MEMLAYER_OK;
  if (!layer && !a->queries) return MEMLAYER_ERR_BAD_POINTER;
  if (!layer && (!a->out || !a->slots || !a->weights)) return MEMLAYER_ERR_BAD_POINTER;
  if (D.vdtype != MEMLAYER_F32 && !aligned16(a->values)) return MEMLAYER_ERR_BAD_POINTER;
  return MEMLAYER_OK;
}

void resolve_noise(Dims* D, const memlayer_config* c, const memlayer_pool_args* a) {
  // memory.py:155-159: select = scores + routing_noise * noise_scale * gumbel (train only)
  const double coef = (double)c->routing_noise * (double)a->noise_scale;
  D->noisy = a->train && c->routing_noise > 0.f && coef != 0.0;
  D->noise_coef = (float)coef;
  D->shuffle = a->shuffle_reads != 0;
}

#define ML_TRY(x)                              \
  do {                                         \
    cudaError_t e_ = (x);                      \
    if (e_ != cudaSuccess) return MEMLAYER_ERR_CUDA; \
  } while (0)

cudaError_t mark(const memlayer_pool_args* a, int i, cudaStream_t s) {
  if (!a->stage_events || !a->stage_events->events[i]) return cudaSuccess;
  return cudaEventRecord((cudaEvent_t)a->stage_events->events[i], s);
}

// Routing from prepared unit queries onward: score + per-half top-k,
// balance statistics, k*k combine + softmax + gather (+ gate), aux finalise.
int aux_stream(cudaStream_t* out);

// Intra-call overlap of the single-GPU forward (score of the second token
// half beside the gather of the first); MEMLAYER_OVERLAP=0 in the
// environment turns it off (stage timing of the bench's roofline pass).
bool overlap_enabled() {
  const char* v = getenv("MEMLAYER_OVERLAP");
  return !(v && v[0] == '0');
}

// Score CTAs of the second part, beside the first part's gather (of 148
// SMs).  The first part is a whole number of rounds of (tile, codebook)
// units over every SM.  configs[0] (64 tiles x 8 codebooks): first part 37
// tiles (296 units = 2 rounds), second part on 108 CTAs: 0.2745 ms per
// step, against 0.2786 for 32 tiles / 100 CTAs, 0.2747 for 37 / 100,
// 0.2750 for 37 / 74, 0.2835 for 32 / 128 and 0.2774 for 18 / 123.
constexpr int OVERLAP_SCORE_CTAS = 108;

// First-part tiles: half of the units rounded up to whole rounds over `sms` CTAs.
int overlap_first_tiles(int mt_all, int hc, int sms) {
  const int units = mt_all * hc;
  const int rounds = (units / 2 + sms - 1) / sms;
  const int mta = rounds * sms / hc;
  return mta >= 1 && mta < mt_all ? mta : mt_all / 2;
}

// Token split of an overlapped call: the first part's score kernel fills
// whole rounds of the SMs, the second part's runs on fewer CTAs beside the
// first part's gather.  0 when the call does not overlap.
int64_t overlap_split(const Dims& D, bool tc_scores, bool balance) {
  const int mt_all = (int)((D.M + SCORE_TM - 1) / SCORE_TM);
  if (!tc_scores || balance || mt_all < 16 || !overlap_enabled()) return 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (int64_t)overlap_first_tiles(mt_all, D.H * 2, sms) * SCORE_TM;
}

// The scatter of a row-sharded call: one per token half; after_a (if set)
// is recorded between the halves.  overlap: the halves split at a tile
// boundary (overlap_split) and the second half's score kernel runs after
// the first half's scatter, beside the first half's gather.
struct ShardRun {
  ShardK half[2];
  bool split;
  bool overlap;
  cudaEvent_t after_a;
};

// With `sh` (row-sharded pool) stage 2 pushes its entries to the owner ranks
// instead of gathering; out / memg / gate are then unused.
int run_route_mix(const Dims& D, const memlayer_pool_args* a, const Work& W, float* qn, int* slots,
                  float* weights, float* out, float* memg, float* memg_hi, float* memg_lo, const float* gate,
                  cudaStream_t s, const ShardRun* sh = nullptr, bool allow_overlap = true) {
  Work w2 = W;
  w2.qn = qn;
  const bool bal = a->balance_loss != nullptr;
  const int mt_all = (int)((D.M + SCORE_TM - 1) / SCORE_TM);
  if (allow_overlap && !sh && W.q_hi && !bal && mt_all >= 16 && overlap_enabled()) {
    // two token halves: the second half's score kernel (on fewer SMs) runs
    // beside the first half's gather (HBM-bound) on a second stream
    cudaStream_t aux = nullptr;
    int st = aux_stream(&aux);
    if (st) return st;
    cudaEvent_t ev[2] = {};
    for (int i = 0; i < 2; ++i)
      if (cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess) {
        if (ev[0]) cudaEventDestroy(ev[0]);
        return MEMLAYER_ERR_CUDA;
      }
    auto body = [&]() -> int {
      int dev = 0, sms = 148;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      const int mta = overlap_first_tiles(mt_all, D.H * 2, sms);
      const int64_t ha = (int64_t)mta * SCORE_TM;
      if (a->slot_counts) ML_TRY(cudaMemsetAsync(a->slot_counts, 0, sizeof(float) * D.N, s));
      if (a->subkey_counts) ML_TRY(cudaMemsetAsync(a->subkey_counts, 0, sizeof(float) * D.H * 2 * D.n, s));
      ML_TRY(launch_score_topk_tc(D, w2, a->gumbel, false, s, 0, mta, 0));
      ML_TRY(cudaEventRecord(ev[0], s));
      ML_TRY(cudaStreamWaitEvent(aux, ev[0], 0));
      ML_TRY(launch_combine_gather(D, w2, a->values, slots, weights, out, memg, memg_hi, memg_lo, gate,
                                   a->slot_counts, a->subkey_counts, aux, 0, ha));
      ML_TRY(cudaEventRecord(ev[1], aux));
      ML_TRY(launch_score_topk_tc(D, w2, a->gumbel, false, s, mta, mt_all - mta, OVERLAP_SCORE_CTAS));
      ML_TRY(mark(a, 3, s));
      ML_TRY(launch_combine_gather(D, w2, a->values, slots, weights, out, memg, memg_hi, memg_lo, gate,
                                   a->slot_counts, a->subkey_counts, s, ha, D.M - ha));
      ML_TRY(cudaStreamWaitEvent(s, ev[1], 0));
      ML_TRY(mark(a, 4, s));
      ML_TRY(launch_finalize(D, w2, a->top1_weight, a->temperature, s));
      return MEMLAYER_OK;
    };
    st = body();
    for (int i = 0; i < 2; ++i) cudaEventDestroy(ev[i]);   // released once their work completes
    return st;
  }
  if (sh && sh->overlap && W.q_hi && !bal) {
    // row-sharded, two halves: score(A), stage 2 + scatter(A), then score(B)
    // on fewer CTAs while the owners gather half A (launched by the caller
    // on the library stream after `after_a`), then stage 2 + scatter(B)
    const int mta = (int)(sh->half[0].t1 / SCORE_TM);
    if (a->slot_counts) ML_TRY(cudaMemsetAsync(a->slot_counts, 0, sizeof(float) * D.N, s));
    if (a->subkey_counts) ML_TRY(cudaMemsetAsync(a->subkey_counts, 0, sizeof(float) * D.H * 2 * D.n, s));
    for (int hf = 0; hf < 2; ++hf) {
      const ShardK& K = sh->half[hf];
      if (hf == 0)
        ML_TRY(launch_score_topk_tc(D, w2, a->gumbel, false, s, 0, mta, 0));
      else
        ML_TRY(launch_score_topk_tc(D, w2, a->gumbel, false, s, mta, mt_all - mta, OVERLAP_SCORE_CTAS));
      if (hf == 1) ML_TRY(mark(a, 3, s));
      if (K.t1 > K.t0)
        ML_TRY(launch_combine_gather(D, w2, nullptr, slots, weights, nullptr, nullptr, nullptr, nullptr, nullptr,
                                     a->slot_counts, a->subkey_counts, s, K.t0, K.t1 - K.t0));
      ML_TRY(launch_shard_scatter(D, K, slots, weights, W.own_cnt, W.err, s));
      if (hf == 0 && sh->after_a) ML_TRY(cudaEventRecord(sh->after_a, s));
    }
    ML_TRY(mark(a, 4, s));
    ML_TRY(launch_finalize(D, w2, a->top1_weight, a->temperature, s));
    return MEMLAYER_OK;
  }
  if (W.q_hi)   // the tensor-core balance pass computes its own row max / sum: the score kernel
                // needs its statistics variant only for the clean top-k of noisy calls
    ML_TRY(launch_score_topk_tc(D, w2, a->gumbel, bal && D.noisy, s));
  else if (W.small && !bal)
    ML_TRY(launch_score_small(D, w2, a->gumbel, W.small, s));
  else
    ML_TRY(launch_score_topk(D, w2, a->gumbel, bal, s));
  if (bal) ML_TRY(launch_balance(D, w2, a->balance_loss, s));
  if (a->slot_counts) ML_TRY(cudaMemsetAsync(a->slot_counts, 0, sizeof(float) * D.N, s));
  if (a->subkey_counts) ML_TRY(cudaMemsetAsync(a->subkey_counts, 0, sizeof(float) * D.H * 2 * D.n, s));
  ML_TRY(mark(a, 3, s));
  if (sh) {
    // stage 2 as on one GPU (routing only), then the entries go to their owners
    for (int hf = 0; hf < (sh->split ? 2 : 1); ++hf) {
      const ShardK& K = sh->half[hf];
      if (K.t1 > K.t0)
        ML_TRY(launch_combine_gather(D, w2, nullptr, slots, weights, nullptr, nullptr, nullptr, nullptr, nullptr,
                                     a->slot_counts, a->subkey_counts, s, K.t0, K.t1 - K.t0));
      ML_TRY(launch_shard_scatter(D, K, slots, weights, W.own_cnt, W.err, s));
      if (hf == 0 && sh->split && sh->after_a) ML_TRY(cudaEventRecord(sh->after_a, s));
    }
  } else
    ML_TRY(launch_combine_gather(D, w2, a->values, slots, weights, out, memg, memg_hi, memg_lo, gate,
                                 a->slot_counts, a->subkey_counts, s));
  ML_TRY(mark(a, 4, s));
  ML_TRY(launch_finalize(D, w2, a->top1_weight, a->temperature, s));
  return MEMLAYER_OK;
}

int prep_keys(const Dims& D, const memlayer_config* c, const memlayer_pool_args* a, const Work& W, cudaStream_t s) {
  ML_TRY(launch_prep_keys(D, a->sub_keys, a->log_temperature, c->min_temperature, c->max_temperature, W.keys_n,
                          W.k_hi, W.k_lo, W.scal, W.err, W.fin_ctr, s));
  return MEMLAYER_OK;
}

// Sharded calls: shapes must be the communicator's, tokens within capacity,
// every peer mapped, and this thread on the communicator's device.
int check_shard(const memlayer_config* c, const void* values, const memlayer_shard_comm* comm) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  if (comm->kind != 0) return MEMLAYER_ERR_BAD_SHAPE;
  const memlayer_config& k = comm->cfg;
  if (c->heads != k.heads || c->n_sub_keys != k.n_sub_keys || c->d_key != k.d_key || c->d_value != k.d_value ||
      c->top_k != k.top_k || c->values_dtype != k.values_dtype || c->tokens > k.tokens)
    return MEMLAYER_ERR_BAD_SHAPE;
  if (c->d_value % 4) return MEMLAYER_ERR_UNSUPPORTED;
  if (!aligned16(values)) return MEMLAYER_ERR_BAD_POINTER;
  for (int p = 0; p < comm->world; ++p)
    if (!comm->peer[p]) return MEMLAYER_ERR_BAD_POINTER;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return MEMLAYER_ERR_CUDA;
  return MEMLAYER_OK;
}

int64_t shard_rows(int64_t pool, int rank, int world) {
  return pool > rank ? (pool - rank + world - 1) / world : 0;
}

ShardK shard_k(const memlayer_shard_comm* comm, const Dims& D) {
  ShardK S{};
  for (int p = 0; p < comm->world; ++p) S.peer[p] = comm->peer[p];
  S.off = comm->off;
  S.rank = comm->rank;
  S.world = comm->world;
  S.mcap = comm->cfg.tokens > 0 ? comm->cfg.tokens : 1;
  S.hk = D.H * D.k;
  S.d = D.d;
  S.rows = shard_rows(D.N, comm->rank, comm->world);
  S.epoch = comm->epoch;
  S.wait_ns = comm->wait_ns;
  S.hf = 0;
  S.t0 = 0;
  S.t1 = D.M;
  S.span = S.mcap;
  return S;
}

// The two token halves of a split call (or the whole call as half 0).
ShardRun shard_run(const memlayer_shard_comm* comm, const Dims& D, bool split, int64_t at = 0) {
  ShardRun R{};
  R.split = split;
  R.overlap = split && at > 0;
  R.half[0] = shard_k(comm, D);
  if (split) {
    const int64_t h0 = at > 0 ? at : (D.M + 1) / 2;
    R.half[0].t1 = h0;
    R.half[0].span = (R.half[0].mcap + 1) / 2;
    R.half[1] = R.half[0];
    R.half[1].hf = 1;
    R.half[1].t0 = h0;
    R.half[1].t1 = D.M;
  }
  return R;
}

// Streams the library keeps per device for work it overlaps with the
// caller's stream (the gathers of split sharded calls, the first token half's
// gather of a single-GPU call); handed out round robin so that calls running
// on different caller streams do not queue behind each other.
int aux_stream(cudaStream_t* out) {
  constexpr int POOL = 4;
  static std::mutex mu;
  static cudaStream_t st[64][POOL] = {};
  static unsigned next[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MEMLAYER_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  const unsigned i = next[dev]++ % POOL;
  if (!st[dev][i] && cudaStreamCreateWithFlags(&st[dev][i], cudaStreamNonBlocking) != cudaSuccess)
    return MEMLAYER_ERR_CUDA;
  *out = st[dev][i];
  return MEMLAYER_OK;
}

// Events of one overlapped split call (released when their work completes).
struct SplitEvents {
  cudaEvent_t e[4] = {};   // push A done, route done, gather A done, gather B done
  int create() {
    for (int i = 0; i < 4; ++i)
      if (cudaEventCreateWithFlags(&e[i], cudaEventDisableTiming) != cudaSuccess) return MEMLAYER_ERR_CUDA;
    return MEMLAYER_OK;
  }
  ~SplitEvents() {
    for (int i = 0; i < 4; ++i)
      if (e[i]) cudaEventDestroy(e[i]);
  }
};

// Gather + reduce of a sharded call.  Overlapped: the gathers run on the
// aux stream (half A after push A, half B after the whole route), the
// reduces on `s` after their half's gather.  `reduce(half)` launches one
// half's reduce.
template <class Reduce>
int shard_gather_reduce(const Dims& D, const ShardRun& R, const void* values, int* err, bool gather, bool reduce,
                        bool overlap, SplitEvents* ev, cudaStream_t s, Reduce reduce_half) {
  const int halves = R.split ? 2 : 1;
  if (overlap) {
    cudaStream_t aux = nullptr;
    int st = aux_stream(&aux);
    if (st) return st;
    ML_TRY(cudaEventRecord(ev->e[1], s));                       // route (and push B) done
    ML_TRY(cudaStreamWaitEvent(aux, ev->e[0], 0));
    ML_TRY(launch_shard_gather(D, R.half[0], values, err, aux));
    ML_TRY(cudaEventRecord(ev->e[2], aux));
    ML_TRY(cudaStreamWaitEvent(aux, ev->e[1], 0));
    ML_TRY(launch_shard_gather(D, R.half[1], values, err, aux));
    ML_TRY(cudaEventRecord(ev->e[3], aux));
    ML_TRY(cudaStreamWaitEvent(s, ev->e[2], 0));
    ML_TRY(reduce_half(R.half[0]));
    ML_TRY(cudaStreamWaitEvent(s, ev->e[3], 0));
    ML_TRY(reduce_half(R.half[1]));
    return MEMLAYER_OK;
  }
  if (gather)
    for (int h = 0; h < halves; ++h) ML_TRY(launch_shard_gather(D, R.half[h], values, err, s));
  if (reduce)
    for (int h = 0; h < halves; ++h) ML_TRY(reduce_half(R.half[h]));
  return MEMLAYER_OK;
}

// MemoryPool.__call__, single GPU (comm == nullptr) or row-sharded.
int pool_impl(const memlayer_config* cfg, const memlayer_pool_args* a, void* workspace, size_t workspace_bytes,
              cudaStream_t s, memlayer_shard_comm* comm, int phases, bool allow_overlap = true,
              bool route_only = false) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  st = check_pool_args(D, a, false);
  if (st) return st;
  if (comm && (st = check_shard(cfg, a->values, comm))) return st;
  resolve_noise(&D, cfg, a);
  if (D.noisy && !a->gumbel && D.M > 0) return MEMLAYER_ERR_BAD_POINTER;
  Flags f;
  f.balance = a->balance_loss != nullptr;
  f.world = comm ? comm->world : 0;
  size_t need = layout(D, f, nullptr, nullptr);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  Work W;
  layout(D, f, (char*)workspace, &W);
  float* qn = a->queries_unit ? a->queries_unit : W.qn;
  if (!comm) {
    memlayer_pool_args ro;
    if (route_only) {   // stage 2 writes slots / weights, no gather
      ro = *a;
      ro.values = nullptr;
      a = &ro;
    }
    ML_TRY(mark(a, 0, s));
    ML_TRY(mark(a, 1, s));
    if ((st = prep_keys(D, cfg, a, W, s))) return st;
    ML_TRY(launch_normalize_queries(D, a->queries, qn, W.qlen, W.q_hi, W.q_lo, s));
    ML_TRY(mark(a, 2, s));
    if ((st = run_route_mix(D, a, W, qn, a->slots, a->weights, route_only ? nullptr : a->out, nullptr, nullptr,
                            nullptr, nullptr, s, nullptr, allow_overlap && !route_only)))
      return st;
    ML_TRY(mark(a, 5, s));
    return MEMLAYER_OK;
  }
  const bool split = (phases & MEMLAYER_PHASE_SPLIT) != 0;
  const bool overlap = split && (phases & MEMLAYER_PHASE_ALL) == MEMLAYER_PHASE_ALL;
  SplitEvents ev;
  if (overlap && (st = ev.create())) return st;
  if (phases & MEMLAYER_PHASE_ROUTE) ++comm->epoch;
  ShardRun R = shard_run(comm, D, split, overlap ? overlap_split(D, W.q_hi != nullptr, f.balance) : 0);
  R.after_a = overlap ? ev.e[0] : nullptr;
  if (phases & MEMLAYER_PHASE_ROUTE) {
    ML_TRY(mark(a, 0, s));
    ML_TRY(mark(a, 1, s));
    if ((st = prep_keys(D, cfg, a, W, s))) return st;
    ML_TRY(launch_normalize_queries(D, a->queries, qn, W.qlen, W.q_hi, W.q_lo, s));
    ML_TRY(mark(a, 2, s));
    if ((st = run_route_mix(D, a, W, qn, a->slots, a->weights, nullptr, nullptr, nullptr, nullptr, nullptr, s, &R)))
      return st;
  }
  auto reduce_half = [&](const ShardK& K) {
    return launch_shard_reduce(D, K, W.own_cnt, nullptr, a->out, nullptr, nullptr, nullptr, W.err, s);
  };
  if ((st = shard_gather_reduce(D, R, a->values, W.err, (phases & MEMLAYER_PHASE_GATHER) != 0,
                                (phases & MEMLAYER_PHASE_REDUCE) != 0, overlap, &ev, s, reduce_half)))
    return st;
  if (phases & MEMLAYER_PHASE_REDUCE) ML_TRY(mark(a, 5, s));
  return MEMLAYER_OK;
}

// Memory-layer block (model.py:108-120), single GPU or row-sharded.
// later_chunk: a chunk after the first of memlayer_layer_forward_host, whose
// sub-key / Dense-kernel preparation and status reset already ran on this
// workspace; only the hidden state is split again.
// route_only: projections and routing (slots, weights, the gate in the
// workspace), no read and no output projection (ROUTE of the staged exchange).
int layer_impl(const memlayer_config* cfg, const memlayer_layer_args* a, void* workspace, size_t workspace_bytes,
               cudaStream_t s, memlayer_shard_comm* comm, int phases, bool later_chunk = false,
               const Work* given = nullptr, bool route_only = false) {
  Dims D;
  int st = check_config(cfg, &D, true);
  if (st) return st;
  if (!a) return MEMLAYER_ERR_BAD_POINTER;
  st = check_pool_args(D, &a->pool, true);
  if (st) return st;
  if (D.M > 0 && (!a->h || !a->w_router || !a->w_gate || !a->w_out || !a->y)) return MEMLAYER_ERR_BAD_POINTER;
  if (!aligned16(a->h) || !aligned16(a->y) || !aligned16(a->mem) || !aligned16(a->pool.out))
    return MEMLAYER_ERR_BAD_POINTER;
  if (comm && (st = check_shard(cfg, a->pool.values, comm))) return st;
  resolve_noise(&D, cfg, &a->pool);
  if (D.noisy && !a->pool.gumbel && D.M > 0) return MEMLAYER_ERR_BAD_POINTER;
  // no tokens on one GPU: no Dense work, only the pool's per-call outputs
  // (temperature, statistics), as the pool entry gives them for no queries
  if (D.M == 0 && !comm && !given) return pool_impl(cfg, &a->pool, workspace, workspace_bytes, s, nullptr,
                                                    MEMLAYER_PHASE_ALL);
  Flags f;
  f.layer = true;
  f.balance = a->pool.balance_loss != nullptr;
  f.world = comm ? comm->world : 0;
  Work W;
  if (given) {
    W = *given;
  } else {
    size_t need = layout(D, f, nullptr, nullptr);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
      return MEMLAYER_ERR_WORKSPACE;
    layout(D, f, (char*)workspace, &W);
  }
  memlayer_pool_args ro;
  const memlayer_pool_args* pa = &a->pool;
  if (route_only) {           // stage 2 writes slots / weights only (no table read)
    ro = a->pool;
    ro.values = nullptr;
    pa = &ro;
  }
  int* slots = pa->slots ? pa->slots : W.slots;
  float* weights = pa->weights ? pa->weights : W.weights;
  float* out = route_only ? nullptr : a->mem ? a->mem : pa->out;
  float* qn = pa->queries_unit ? pa->queries_unit : W.qn;
  const bool route = !comm || (phases & MEMLAYER_PHASE_ROUTE);
  const bool reduce = (!comm || (phases & MEMLAYER_PHASE_REDUCE)) && !route_only;
  const bool split = comm && (phases & MEMLAYER_PHASE_SPLIT) != 0;
  const bool overlap = split && (phases & MEMLAYER_PHASE_ALL) == MEMLAYER_PHASE_ALL;
  SplitEvents ev;
  if (overlap && (st = ev.create())) return st;
  ShardRun R{};
  if (comm) {
    if (route) ++comm->epoch;
    R = shard_run(comm, D, split, overlap ? overlap_split(D, W.q_hi != nullptr, f.balance) : 0);
    R.after_a = overlap ? ev.e[0] : nullptr;
  }
  const ShardRun* sh = comm ? &R : nullptr;
  if (W.h_hi) {
    if (route) {
      ML_TRY(mark(pa, 0, s));
      // tensor-core projections: K-major tf32 halves of the Dense kernels and
      // the hidden state, then one GEMM for router (model.py:110) + gate (:118)
      const int NR = D.H * D.dk;
      if (later_chunk) {
        ML_TRY(launch_split(a->h, D.M * D.dm, W.h_hi, W.h_lo, s));
      } else if (W.k_hi) {
        ML_TRY(launch_prep_layer(D, W, pa->sub_keys, pa->log_temperature, cfg->min_temperature,
                                 cfg->max_temperature, a->h, a->w_router, a->b_router, a->w_gate, a->b_gate,
                                 a->w_out, s));
      } else {
        if ((st = prep_keys(D, cfg, pa, W, s))) return st;
        ML_TRY(launch_transpose_split(a->w_router, D.dm, NR, W.wrg_hi, W.wrg_lo, 0, s));
        ML_TRY(launch_transpose_split(a->w_gate, D.dm, D.d, W.wrg_hi, W.wrg_lo, NR, s));
        ML_TRY(launch_concat_bias(a->b_router, NR, a->b_gate, D.d, W.bias_rg, s));
        ML_TRY(launch_transpose_split(a->w_out, D.d, D.dm, W.wo_hi, W.wo_lo, 0, s));
        ML_TRY(launch_split(a->h, D.M * D.dm, W.h_hi, W.h_lo, s));
      }
      // unit queries in float32 only when the aux output asks or the SIMT score path reads them
      ML_TRY(launch_router_gate_tc(D, W, W.bias_rg, (pa->queries_unit || !W.q_hi) ? qn : nullptr, s));
      ML_TRY(mark(pa, 1, s));
      ML_TRY(mark(pa, 2, s));
      if ((st = run_route_mix(D, pa, W, qn, slots, weights, out, nullptr, W.memg_hi, W.memg_lo, W.gate, s, sh)))
        return st;
    }
    if (comm) {
      auto reduce_half = [&](const ShardK& K) {
        return launch_shard_reduce(D, K, W.own_cnt, W.gate, out, nullptr, W.memg_hi, W.memg_lo, W.err, s);
      };
      if ((st = shard_gather_reduce(D, R, pa->values, W.err, (phases & MEMLAYER_PHASE_GATHER) != 0, reduce, overlap,
                                    &ev, s, reduce_half)))
        return st;
    }
    if (reduce) ML_TRY(launch_out_tc(D, W, a->b_out, a->y, s));                 // model.py:119
  } else {
    // SIMT float32 projections
    if (route) {
      ML_TRY(mark(pa, 0, s));
      if (!later_chunk && (st = prep_keys(D, cfg, pa, W, s))) return st;
      ML_TRY(launch_gemm2(a->h, a->w_router, a->b_router, W.qraw, D.H * D.dk, false,       // model.py:110-111
                          a->w_gate, a->b_gate, W.gate, D.d, true, D.M, D.dm, s));          // model.py:118
      ML_TRY(mark(pa, 1, s));
      ML_TRY(launch_normalize_queries(D, W.qraw, qn, W.qlen, W.q_hi, W.q_lo, s));
      ML_TRY(mark(pa, 2, s));
      if ((st = run_route_mix(D, pa, W, qn, slots, weights, out, W.memg, nullptr, nullptr, W.gate, s, sh)))
        return st;
    }
    if (comm) {
      auto reduce_half = [&](const ShardK& K) {
        return launch_shard_reduce(D, K, W.own_cnt, W.gate, out, W.memg, nullptr, nullptr, W.err, s);
      };
      if ((st = shard_gather_reduce(D, R, pa->values, W.err, (phases & MEMLAYER_PHASE_GATHER) != 0, reduce, overlap,
                                    &ev, s, reduce_half)))
        return st;
    }
    if (reduce) ML_TRY(launch_gemm(W.memg, a->w_out, a->b_out, a->y, D.M, D.dm, D.d, false, s));  // model.py:119
  }
  if (reduce) {
    if (a->mem && pa->out && pa->out != a->mem && D.M > 0)
      ML_TRY(cudaMemcpyAsync(pa->out, a->mem, sizeof(float) * D.M * D.d, cudaMemcpyDeviceToDevice, s));
    ML_TRY(mark(pa, 5, s));
  }
  return MEMLAYER_OK;
}

// ---- host-buffer layer forward: chunked copy / compute pipeline ----
constexpr int64_t HOST_MIN_CHUNK = 256;   // smaller chunks do not pay for their fixed costs

struct HostPlan {
  int chunks;
  int64_t mc;          // tokens per chunk (the last may have fewer)
  size_t work_bytes;   // chunk workspace
  size_t stage_off_y;  // staging: h at work_bytes, y at stage_off_y
  size_t bytes;
};

HostPlan host_plan(const Dims& D, int chunks) {
  HostPlan p{};
  int64_t c = chunks < 1 ? 1 : chunks;
  while (c > 1 && (D.M + c - 1) / c < HOST_MIN_CHUNK) --c;
  p.chunks = (int)c;
  p.mc = D.M > 0 ? (D.M + c - 1) / c : 0;
  Dims Dc = D;
  Dc.M = p.mc;
  Flags f;
  f.layer = true;
  p.work_bytes = layout(Dc, f, nullptr, nullptr);
  p.stage_off_y = p.work_bytes + up(sizeof(float) * D.M * D.dm);
  p.bytes = p.stage_off_y + up(sizeof(float) * D.M * D.dm);
  return p;
}

// Two non-blocking copy streams per device (host-to-device, device-to-host),
// created on first use and kept for the life of the process.
int copy_streams(cudaStream_t* in, cudaStream_t* out) {
  static std::mutex mu;
  static cudaStream_t cs[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MEMLAYER_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < 2; ++i)
    if (!cs[dev][i] && cudaStreamCreateWithFlags(&cs[dev][i], cudaStreamNonBlocking) != cudaSuccess)
      return MEMLAYER_ERR_CUDA;
  *in = cs[dev][0];
  *out = cs[dev][1];
  return MEMLAYER_OK;
}

// Reads of a row-gradient call: shapes, pointers and fetch offsets.
int rowgrad_setup(const memlayer_config* cfg, const memlayer_read* reads, int n_reads, RowGradK* R) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (!reads) return MEMLAYER_ERR_BAD_POINTER;
  if (n_reads < 1 || n_reads > MEMLAYER_MAX_READS) return MEMLAYER_ERR_BAD_SHAPE;
  if (D.d % 4) return MEMLAYER_ERR_UNSUPPORTED;
  *R = RowGradK{};
  R->n_reads = n_reads;
  R->N = D.N;
  R->Nslot = D.N;
  R->hk = D.H * D.k;
  R->d = D.d;
  R->off[0] = 0;
  for (int r = 0; r < n_reads; ++r) {
    const memlayer_read& x = reads[r];
    if (x.tokens < 0) return MEMLAYER_ERR_BAD_SHAPE;
    if (x.tokens > 0 && (!x.slots || !x.weights || !x.grad)) return MEMLAYER_ERR_BAD_POINTER;
    if (!aligned16(x.grad)) return MEMLAYER_ERR_BAD_POINTER;
    R->slots[r] = x.slots;
    R->weights[r] = x.weights;
    R->grad[r] = x.grad;
    R->off[r + 1] = R->off[r] + x.tokens * R->hk;
  }
  R->F = R->off[n_reads];
  if (R->F >= (1LL << 31)) return MEMLAYER_ERR_BAD_SHAPE;   // fetch ids are 32-bit
  return MEMLAYER_OK;
}

}  // namespace

// What memlayer_layer_forward prepared in each workspace (sub-key
// normalisation, Dense-kernel splits): the config and the weight pointers of
// the last successful call, so that memlayer_layer_forward_prepared can refuse
// a workspace prepared for other arguments.  In-place changes of the weights
// cannot be seen here; the caller's contract covers them.
struct Prepared {
  memlayer_config cfg;
  const void* ptr[8];
};
std::mutex g_prep_mu;
std::unordered_map<const void*, Prepared> g_prepared;

Prepared prepared_of(const memlayer_config* cfg, const memlayer_layer_args* a) {
  Prepared p{};
  p.cfg = *cfg;
  const void* v[8] = {a->pool.sub_keys, a->pool.log_temperature, a->w_router, a->b_router,
                      a->w_gate,        a->b_gate,                a->w_out,    a->b_out};
  for (int i = 0; i < 8; ++i) p.ptr[i] = v[i];
  return p;
}

void record_prepared(const void* ws, const memlayer_config* cfg, const memlayer_layer_args* a) {
  std::lock_guard<std::mutex> lk(g_prep_mu);
  g_prepared[ws] = prepared_of(cfg, a);
}

bool is_prepared(const void* ws, const memlayer_config* cfg, const memlayer_layer_args* a) {
  const Prepared want = prepared_of(cfg, a);
  std::lock_guard<std::mutex> lk(g_prep_mu);
  auto it = g_prepared.find(ws);
  return it != g_prepared.end() && memcmp(&it->second, &want, sizeof(Prepared)) == 0;
}

// MemoryPool forward on the caller's stream only: no event, no library
// stream (the allocation-free entry point).
int32_t pool_forward_single_stream(const memlayer_config* cfg, const memlayer_pool_args* args, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  return pool_impl(cfg, args, workspace, workspace_bytes, (cudaStream_t)stream, nullptr, MEMLAYER_PHASE_ALL, false);
}

}  // namespace ml

using namespace ml;

extern "C" {

int32_t memlayer_abi_version(void) { return MEMLAYER_ABI_VERSION; }

int64_t memlayer_kernel_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* memlayer_status_string(int32_t s) {
  switch (s) {
    case MEMLAYER_OK: return "ok";
    case MEMLAYER_ERR_BAD_SHAPE: return "bad shape";
    case MEMLAYER_ERR_BAD_POINTER: return "bad pointer";
    case MEMLAYER_ERR_UNSUPPORTED: return "unsupported setting";
    case MEMLAYER_ERR_WORKSPACE: return "workspace too small";
    case MEMLAYER_ERR_CUDA: return "CUDA error";
    case MEMLAYER_ERR_PEER_TIMEOUT: return "peer timeout";
    default: return "unknown status";
  }
}

int32_t memlayer_pool_workspace_size(const memlayer_config* cfg, size_t* bytes) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  Flags f;
  f.balance = true;  // sized for the largest request
  *bytes = layout(D, f, nullptr, nullptr);
  return MEMLAYER_OK;
}

int32_t memlayer_layer_workspace_size(const memlayer_config* cfg, size_t* bytes) {
  Dims D;
  int st = check_config(cfg, &D, true);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  Flags f;
  f.balance = true;
  f.layer = true;
  *bytes = layout(D, f, nullptr, nullptr);
  return MEMLAYER_OK;
}

int32_t memlayer_pool_forward(const memlayer_config* cfg, const memlayer_pool_args* a, void* workspace,
                              size_t workspace_bytes, void* stream) {
  return pool_impl(cfg, a, workspace, workspace_bytes, (cudaStream_t)stream, nullptr, MEMLAYER_PHASE_ALL);
}

int32_t memlayer_layer_forward(const memlayer_config* cfg, const memlayer_layer_args* a, void* workspace,
                               size_t workspace_bytes, void* stream) {
  const int st = layer_impl(cfg, a, workspace, workspace_bytes, (cudaStream_t)stream, nullptr, MEMLAYER_PHASE_ALL);
  if (st == MEMLAYER_OK) record_prepared(workspace, cfg, a);
  return st;
}

int32_t memlayer_workspace_status(const memlayer_config* cfg, const void* workspace, int32_t* code, void* stream) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (!workspace || !code) return MEMLAYER_ERR_BAD_POINTER;
  Work W;
  layout(D, Flags{}, (char*)workspace, &W);   // the error word sits at the same offset in every layout
  int v = 0;
  ML_TRY(cudaMemcpyAsync(&v, W.err, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  ML_TRY(cudaStreamSynchronize((cudaStream_t)stream));
  *code = v;
  return MEMLAYER_OK;
}

// ---- row-sharded pool ----

// A phase mask of a sharded call: at least one phase, no unknown bit (SPLIT
// only for the forward), and no REDUCE with ROUTE but without GATHER -- the
// reduce would wait for this rank's own gather, which only a later call runs.
static bool phase_mask_ok(int phases, bool allow_split) {
  const int known = MEMLAYER_PHASE_ALL | (allow_split ? MEMLAYER_PHASE_SPLIT : 0);
  if ((phases & MEMLAYER_PHASE_ALL) == 0 || (phases & ~known)) return false;
  return !((phases & MEMLAYER_PHASE_ROUTE) && (phases & MEMLAYER_PHASE_REDUCE) && !(phases & MEMLAYER_PHASE_GATHER));
}

int64_t memlayer_shard_rows(int64_t pool_size, int32_t rank, int32_t world) {
  if (world < 1 || rank < 0 || rank >= world || pool_size < 0) return 0;
  return shard_rows(pool_size, rank, world);
}

int32_t memlayer_shard_comm_create(const memlayer_config* cfg, int32_t rank, int32_t world,
                                   memlayer_shard_comm** comm) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  *comm = nullptr;
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (world < 1 || world > MEMLAYER_MAX_SHARDS || rank < 0 || rank >= world) return MEMLAYER_ERR_BAD_SHAPE;
  if (D.d % 4) return MEMLAYER_ERR_UNSUPPORTED;
  memlayer_shard_comm* c = new (std::nothrow) memlayer_shard_comm;
  if (!c) return MEMLAYER_ERR_CUDA;
  c->rank = rank;
  c->world = world;
  c->cfg = *cfg;
  if (cudaGetDevice(&c->device) != cudaSuccess) {
    delete c;
    return MEMLAYER_ERR_CUDA;
  }
  c->off = shard_layout(world, cfg->tokens > 0 ? cfg->tokens : 1, D.H * D.k, D.d);
  if (cudaMalloc(&c->base, (size_t)c->off.bytes) != cudaSuccess) {
    delete c;
    return MEMLAYER_ERR_CUDA;
  }
  if (cudaMemset(c->base, 0, (size_t)c->off.bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(c->base);
    delete c;
    return MEMLAYER_ERR_CUDA;
  }
  c->peer[rank] = c->base;
  *comm = c;
  return MEMLAYER_OK;
}

int32_t memlayer_shard_comm_info(const memlayer_shard_comm* comm, int32_t* rank, int32_t* world, int32_t* device,
                                 size_t* bytes) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  if (rank) *rank = comm->rank;
  if (world) *world = comm->world;
  if (device) *device = comm->device;
  if (bytes) *bytes = (size_t)comm->off.bytes;
  return MEMLAYER_OK;
}

static_assert(sizeof(cudaIpcMemHandle_t) == MEMLAYER_IPC_HANDLE_BYTES, "IPC handle size");

int32_t memlayer_shard_comm_ipc_handle(const memlayer_shard_comm* comm, void* handle) {
  if (!comm || !handle) return MEMLAYER_ERR_BAD_POINTER;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, comm->base) != cudaSuccess) return MEMLAYER_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return MEMLAYER_OK;
}

int32_t memlayer_shard_comm_open_peers(memlayer_shard_comm* comm, const void* handles) {
  if (!comm || !handles) return MEMLAYER_ERR_BAD_POINTER;
  for (int p = 0; p < comm->world; ++p) {
    if (p == comm->rank || comm->opened[p]) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, (const char*)handles + (size_t)p * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return MEMLAYER_ERR_CUDA;
    comm->peer[p] = (char*)ptr;
    comm->opened[p] = true;
  }
  return MEMLAYER_OK;
}

int32_t memlayer_shard_comm_set_peer(memlayer_shard_comm* comm, int32_t peer, const memlayer_shard_comm* other) {
  if (!comm || !other) return MEMLAYER_ERR_BAD_POINTER;
  if (peer < 0 || peer >= comm->world || peer == comm->rank || comm->opened[peer]) return MEMLAYER_ERR_BAD_SHAPE;
  // peers address each other's buffers with their own offsets: shapes must agree
  if (other->world != comm->world || other->rank != peer || other->kind != comm->kind ||
      other->off.bytes != comm->off.bytes ||
      other->cfg.tokens != comm->cfg.tokens || other->cfg.heads != comm->cfg.heads ||
      other->cfg.top_k != comm->cfg.top_k || other->cfg.d_value != comm->cfg.d_value)
    return MEMLAYER_ERR_BAD_SHAPE;
  comm->peer[peer] = other->base;
  return MEMLAYER_OK;
}

int32_t memlayer_shard_comm_set_wait_budget(memlayer_shard_comm* comm, int64_t nanoseconds) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  if (nanoseconds < 1000 || nanoseconds > 60000000000LL) return MEMLAYER_ERR_BAD_SHAPE;
  comm->wait_ns = nanoseconds;
  return MEMLAYER_OK;
}

int32_t memlayer_shard_comm_destroy(memlayer_shard_comm* comm) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  int st = MEMLAYER_OK;
  for (int p = 0; p < comm->world; ++p)
    if (comm->opened[p] && cudaIpcCloseMemHandle(comm->peer[p]) != cudaSuccess) st = MEMLAYER_ERR_CUDA;
  if (comm->base && cudaFree(comm->base) != cudaSuccess) st = MEMLAYER_ERR_CUDA;
  delete comm;
  return st;
}

// ---- owner-sharded row update ----

int32_t memlayer_shard_comm_create_rowgrad(const memlayer_config* cfg, int32_t n_reads, int32_t rank, int32_t world,
                                           memlayer_shard_comm** comm) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  *comm = nullptr;
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (world < 1 || world > MEMLAYER_MAX_SHARDS || rank < 0 || rank >= world) return MEMLAYER_ERR_BAD_SHAPE;
  if (n_reads < 1 || n_reads > MEMLAYER_MAX_READS) return MEMLAYER_ERR_BAD_SHAPE;
  if (D.d % 4) return MEMLAYER_ERR_UNSUPPORTED;
  if (cfg->values_dtype != MEMLAYER_F32) return MEMLAYER_ERR_UNSUPPORTED;
  memlayer_shard_comm* c = new (std::nothrow) memlayer_shard_comm;
  if (!c) return MEMLAYER_ERR_CUDA;
  c->rank = rank;
  c->world = world;
  c->cfg = *cfg;
  c->kind = 1;
  c->n_reads = n_reads;
  if (cudaGetDevice(&c->device) != cudaSuccess) {
    delete c;
    return MEMLAYER_ERR_CUDA;
  }
  const int64_t stride = (D.N + world - 1) / world;
  const int64_t fetch_cap = (int64_t)n_reads * (cfg->tokens > 0 ? cfg->tokens : 1) * D.H * D.k;
  c->rcap = fetch_cap < stride ? fetch_cap : stride;
  c->roff = row_shard_layout(world, c->rcap, D.d);
  c->off.bytes = c->roff.bytes;
  if (cudaMalloc(&c->base, (size_t)c->roff.bytes) != cudaSuccess) {
    delete c;
    return MEMLAYER_ERR_CUDA;
  }
  if (cudaMemset(c->base, 0, (size_t)c->roff.bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(c->base);
    delete c;
    return MEMLAYER_ERR_CUDA;
  }
  c->peer[rank] = c->base;
  *comm = c;
  return MEMLAYER_OK;
}

namespace {

struct RowPlan {
  RowGradLayout L;
  int64_t o_small, o_mkey, o_mref, o_head, o_rowsq, o_mrow, bytes;
};

RowPlan row_plan(const memlayer_shard_comm* comm, const RowGradK& R) {
  RowPlan P{};
  P.L = rowgrad_layout(R.F, R.N, R.d);
  const int64_t n = (int64_t)comm->world * comm->rcap;
  int64_t o = (int64_t)up((size_t)P.L.bytes);
  auto take = [&](int64_t b) {
    const int64_t at = o;
    o += (int64_t)up((size_t)b);
    return at;
  };
  P.o_small = take(256);
  P.o_mkey = take(4 * n);
  P.o_mref = take(4 * n);
  P.o_head = take(4 * n);
  P.o_rowsq = take(4 * n);
  P.o_mrow = take(4 * n * R.d);
  P.bytes = o;
  return P;
}

// The read descriptors with owner-grouped sort keys for this communicator.
int row_setup(const memlayer_config* cfg, const memlayer_read* reads, int n_reads, const memlayer_shard_comm* comm,
              RowGradK* R) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  if (comm->kind != 1) return MEMLAYER_ERR_BAD_SHAPE;
  int st = rowgrad_setup(cfg, reads, n_reads, R);
  if (st) return st;
  const memlayer_config& k = comm->cfg;
  if (cfg->heads != k.heads || cfg->n_sub_keys != k.n_sub_keys || cfg->d_value != k.d_value ||
      cfg->top_k != k.top_k || n_reads > comm->n_reads)
    return MEMLAYER_ERR_BAD_SHAPE;
  for (int r = 0; r < n_reads; ++r)
    if (reads[r].tokens > (k.tokens > 0 ? k.tokens : 1)) return MEMLAYER_ERR_BAD_SHAPE;
  const int64_t stride = (R->Nslot + comm->world - 1) / comm->world;
  R->kworld = comm->world;
  R->kstride = stride;
  R->N = stride * comm->world;
  return MEMLAYER_OK;
}

RowShardK row_k(const memlayer_shard_comm* comm, const RowGradK& R) {
  RowShardK K{};
  for (int p = 0; p < comm->world; ++p) K.peer[p] = comm->peer[p];
  K.off = comm->roff;
  K.rank = comm->rank;
  K.world = comm->world;
  K.cap = comm->rcap;
  K.stride = R.kstride;
  K.rows = shard_rows(R.Nslot, comm->rank, comm->world);
  K.d = R.d;
  K.epoch = comm->epoch;
  K.wait_ns = comm->wait_ns;
  return K;
}

}  // namespace

int32_t memlayer_shard_rowgrad_workspace_size(const memlayer_shard_comm* comm, int64_t fetches, size_t* bytes) {
  if (!comm || !bytes) return MEMLAYER_ERR_BAD_POINTER;
  if (comm->kind != 1) return MEMLAYER_ERR_BAD_SHAPE;
  if (fetches < 0 || fetches >= (1LL << 31)) return MEMLAYER_ERR_BAD_SHAPE;
  RowGradK R{};
  R.F = fetches;
  R.d = comm->cfg.d_value;
  R.Nslot = (int64_t)comm->cfg.n_sub_keys * comm->cfg.n_sub_keys;
  R.kstride = (R.Nslot + comm->world - 1) / comm->world;
  R.N = R.kstride * comm->world;
  *bytes = (size_t)row_plan(comm, R).bytes;
  return MEMLAYER_OK;
}

int32_t memlayer_row_adagrad_sharded(const memlayer_config* cfg, const memlayer_read* reads, int32_t n_reads,
                                     const memlayer_adagrad_args* args, memlayer_shard_comm* comm, int32_t phases,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  RowGradK R;
  int st = row_setup(cfg, reads, n_reads, comm, &R);
  if (st) return st;
  if (!args || !args->values || !args->accum || !aligned16(args->values)) return MEMLAYER_ERR_BAD_POINTER;
  if (cfg->values_dtype != MEMLAYER_F32) return MEMLAYER_ERR_UNSUPPORTED;
  if (!phase_mask_ok(phases, false)) return MEMLAYER_ERR_BAD_SHAPE;
  for (int p = 0; p < comm->world; ++p)
    if (!comm->peer[p]) return MEMLAYER_ERR_BAD_POINTER;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return MEMLAYER_ERR_CUDA;
  const RowPlan P = row_plan(comm, R);
  if (!workspace || workspace_bytes < (size_t)P.bytes || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  char* ws = (char*)workspace;
  const cudaStream_t s = (cudaStream_t)stream;
  int* err = reinterpret_cast<int*>(ws + P.L.o_err);
  if (phases & MEMLAYER_PHASE_ROUTE) ++comm->epoch;
  const RowShardK K = row_k(comm, R);
  RowMerge G;
  G.small = reinterpret_cast<int*>(ws + P.o_small);
  G.mkey = reinterpret_cast<int*>(ws + P.o_mkey);
  G.mref = reinterpret_cast<int*>(ws + P.o_mref);
  G.head = reinterpret_cast<int*>(ws + P.o_head);
  G.rowsq = reinterpret_cast<float*>(ws + P.o_rowsq);
  G.mrow = reinterpret_cast<float*>(ws + P.o_mrow);
  if (phases & MEMLAYER_PHASE_ROUTE) {
    // local merge with owner-grouped keys; uniq / rows / segment count stay in the workspace
    ML_TRY(launch_rowgrad(R, P.L, ws, nullptr, nullptr, nullptr, nullptr, nullptr, s));
    const int* n_seg = reinterpret_cast<const int*>(ws + P.L.o_small) + 1;
    ML_TRY(launch_rows_push(K, reinterpret_cast<const int*>(ws + P.L.o_uniq),
                            reinterpret_cast<const float*>(ws + P.L.o_rows), n_seg, P.L.cap, err, s));
  }
  if (phases & MEMLAYER_PHASE_GATHER) ML_TRY(launch_rows_merge(K, G, err, s));
  if (phases & MEMLAYER_PHASE_REDUCE)
    ML_TRY(launch_rows_apply(K, G, args->values, args->accum, args->lr, args->grad_clip, args->rest_sq_norm,
                             args->clip_scale, args->n_unique, err, s));
  return MEMLAYER_OK;
}

int32_t memlayer_shard_workspace_size(const memlayer_config* cfg, int32_t world, int32_t layer, size_t* bytes) {
  Dims D;
  int st = check_config(cfg, &D, layer != 0);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  if (world < 1 || world > MEMLAYER_MAX_SHARDS) return MEMLAYER_ERR_BAD_SHAPE;
  Flags f;
  f.balance = true;
  f.layer = layer != 0;
  f.world = world;
  *bytes = layout(D, f, nullptr, nullptr);
  return MEMLAYER_OK;
}

int32_t memlayer_pool_forward_sharded(const memlayer_config* cfg, const memlayer_pool_args* args,
                                      memlayer_shard_comm* comm, int32_t phases, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  if (!phase_mask_ok(phases, true))
    return MEMLAYER_ERR_BAD_SHAPE;
  return pool_impl(cfg, args, workspace, workspace_bytes, (cudaStream_t)stream, comm, phases);
}

int32_t memlayer_layer_forward_sharded(const memlayer_config* cfg, const memlayer_layer_args* args,
                                       memlayer_shard_comm* comm, int32_t phases, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  if (!phase_mask_ok(phases, true))
    return MEMLAYER_ERR_BAD_SHAPE;
  return layer_impl(cfg, args, workspace, workspace_bytes, (cudaStream_t)stream, comm, phases);
}

// ---- fetched-row gradients / row-wise Adagrad ----

int32_t memlayer_rowgrad_workspace_size(const memlayer_config* cfg, int64_t fetches, size_t* bytes) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  if (fetches < 0 || fetches >= (1LL << 31)) return MEMLAYER_ERR_BAD_SHAPE;
  *bytes = (size_t)rowgrad_layout(fetches, D.N, D.d).bytes;
  return MEMLAYER_OK;
}

int32_t memlayer_fetched_row_grads(const memlayer_config* cfg, const memlayer_read* reads, int32_t n_reads,
                                   int32_t* uniq, float* rows, int32_t* n_unique, float* sq_norm,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  RowGradK R;
  int st = rowgrad_setup(cfg, reads, n_reads, &R);
  if (st) return st;
  if ((!uniq && R.F > 0) || !aligned16(rows)) return MEMLAYER_ERR_BAD_POINTER;
  const RowGradLayout L = rowgrad_layout(R.F, R.N, R.d);
  if (!workspace || workspace_bytes < (size_t)L.bytes || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  ML_TRY(launch_rowgrad(R, L, (char*)workspace, uniq, rows, n_unique, sq_norm, nullptr, (cudaStream_t)stream));
  return MEMLAYER_OK;
}

int32_t memlayer_row_adagrad(const memlayer_config* cfg, const memlayer_read* reads, int32_t n_reads,
                             const memlayer_adagrad_args* args, void* workspace, size_t workspace_bytes,
                             void* stream) {
  RowGradK R;
  int st = rowgrad_setup(cfg, reads, n_reads, &R);
  if (st) return st;
  if (!args || !args->values || !args->accum || !aligned16(args->values)) return MEMLAYER_ERR_BAD_POINTER;
  if (cfg->values_dtype != MEMLAYER_F32) return MEMLAYER_ERR_UNSUPPORTED;
  const RowGradLayout L = rowgrad_layout(R.F, R.N, R.d);
  if (!workspace || workspace_bytes < (size_t)L.bytes || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  RowAdagrad A{args->values, args->accum, args->lr, args->grad_clip, args->rest_sq_norm, args->clip_scale,
               args->n_unique};
  ML_TRY(launch_rowgrad(R, L, (char*)workspace, nullptr, nullptr, nullptr, nullptr, &A, (cudaStream_t)stream));
  return MEMLAYER_OK;
}

// ---- value table in page-locked host memory ----

namespace {

struct TablePlan {
  size_t fwd;              // pool-forward workspace (at offset 0: its status word is the call's)
  RowGradLayout L;         // sort of the read slots
  int64_t o_sort, o_inv, o_stage, cap, bytes;
};

TablePlan table_plan(const Dims& D, const Flags& f) {
  TablePlan P{};
  P.fwd = layout(D, f, nullptr, nullptr);
  const int64_t F = D.M * D.H * D.k;
  P.L = rowgrad_layout(F, D.N, 0);
  P.cap = F < D.N ? F : D.N;
  int64_t o = (int64_t)up(P.fwd);
  P.o_sort = o;
  o += (int64_t)up((size_t)P.L.bytes);
  P.o_inv = o;
  o += (int64_t)up((size_t)(4 * F));
  P.o_stage = o;
  o += (int64_t)up((size_t)(P.cap * D.d * table_elem_bytes(D.vdtype)));
  P.bytes = o;
  return P;
}

}  // namespace

int32_t memlayer_host_table_workspace_size(const memlayer_config* cfg, size_t* bytes) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  Flags f;
  f.balance = true;
  *bytes = (size_t)table_plan(D, f).bytes;
  return MEMLAYER_OK;
}

int32_t memlayer_pool_forward_host_table(const memlayer_config* cfg, const memlayer_pool_args* a, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if ((st = check_pool_args(D, a, false))) return st;
  // the table must be readable by this device: page-locked host memory (or device memory)
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, a->values) != cudaSuccess) {
    cudaGetLastError();
    return MEMLAYER_ERR_BAD_POINTER;
  }
  if (attr.type == cudaMemoryTypeUnregistered || !attr.devicePointer) return MEMLAYER_ERR_BAD_POINTER;
  const void* table = attr.devicePointer;
  Flags f;
  f.balance = a->balance_loss != nullptr;
  const TablePlan P = table_plan(D, f);
  if (!workspace || workspace_bytes < (size_t)P.bytes || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  const cudaStream_t s = (cudaStream_t)stream;
  if ((st = pool_impl(cfg, a, workspace, P.fwd, s, nullptr, MEMLAYER_PHASE_ALL, false, true))) return st;
  if (D.M == 0) return MEMLAYER_OK;
  char* ws = (char*)workspace;
  resolve_noise(&D, cfg, a);
  RowGradK R{};
  R.n_reads = 1;
  R.slots[0] = a->slots;
  R.weights[0] = a->weights;
  R.off[0] = 0;
  R.off[1] = D.M * D.H * D.k;
  R.F = R.off[1];
  R.N = D.N;
  R.Nslot = D.N;
  R.hk = D.H * D.k;
  R.d = 0;
  R.kadd = D.shuffle ? D.N / 2 + 1 : 0;   // the read slot (memory.py:179)
  int* inv = reinterpret_cast<int*>(ws + P.o_inv);
  char* sort_ws = ws + P.o_sort;
  if (R.F <= TABLE_SMALL_F)   // decode-size calls: one CTA instead of the radix passes
    ML_TRY(launch_table_unique_small(a->slots, (int)R.F, D.N, R.kadd, reinterpret_cast<int*>(sort_ws + P.L.o_uniq),
                                     reinterpret_cast<int*>(sort_ws + P.L.o_small) + 1, inv, s));
  else
    ML_TRY(launch_sort_unique(R, P.L, sort_ws, inv, s));
  int* err = reinterpret_cast<int*>(ws + 256);   // the forward's status word
  ML_TRY(launch_table_fetch(D, table, reinterpret_cast<const int*>(sort_ws + P.L.o_uniq),
                            reinterpret_cast<const int*>(sort_ws + P.L.o_small) + 1, P.cap, ws + P.o_stage, err, s));
  ML_TRY(launch_table_mix(D, ws + P.o_stage, inv, a->weights, a->out, s));
  return MEMLAYER_OK;
}

// ---- sub-key maintenance ----

int32_t memlayer_key_diversity_workspace_size(const memlayer_config* cfg, size_t* bytes) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  *bytes = (size_t)key_div_layout(D.H * 2, D.n, D.half).bytes;
  return MEMLAYER_OK;
}

int32_t memlayer_key_diversity(const memlayer_config* cfg, const float* sub_keys, float* loss, float* grad,
                               float grad_scale, void* workspace, size_t workspace_bytes, void* stream) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (!sub_keys || (!loss && !grad)) return MEMLAYER_ERR_BAD_POINTER;
  const KeyDivLayout L = key_div_layout(D.H * 2, D.n, D.half);
  if (!workspace || workspace_bytes < (size_t)L.bytes || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  ML_TRY(launch_key_diversity(sub_keys, D.H * 2, D.n, D.half, (char*)workspace, loss, grad, grad_scale,
                              (cudaStream_t)stream));
  return MEMLAYER_OK;
}

int32_t memlayer_revive_dead_keys(const memlayer_config* cfg, const memlayer_revive_args* a, void* stream) {
  Dims D;
  int st = check_config(cfg, &D, false);
  if (st) return st;
  if (!a || !a->sub_keys || !a->usage || !a->queries || !a->pick || !a->noise) return MEMLAYER_ERR_BAD_POINTER;
  if (a->query_tokens < 1) return MEMLAYER_ERR_BAD_SHAPE;
  ML_TRY(launch_revive(a->sub_keys, a->usage, a->queries, a->query_tokens, a->pick, a->noise, D.H * 2, D.n, D.half,
                       a->threshold, a->noise_scale, a->dead, a->moment0, a->moment1, (cudaStream_t)stream));
  return MEMLAYER_OK;
}

// ---- layer backward ----

namespace {

struct BwdPlan {
  RowGradLayout L;
  int64_t F, cap;
  int64_t o_qraw, o_qn, o_qlen, o_keys, o_scal, o_zg, o_dmemg, o_memg, o_dzg, o_dqhat, o_dqlen, o_dT, o_ent_s,
      o_ent_w, o_rg, o_uniq, o_rows, o_dkhat, o_dq, o_cbal, o_dTrow, o_dqlrow, o_ones, o_gemm, bytes;
  size_t gemm_floats;   // scratch of the tensor-core GEMMs (operand halves, slice partials)
  // balance term on the tensor cores (bal_bwd_tc.cu): operand halves and scratch
  bool bal_tc;
  BalBwdPlan bp;
  int64_t o_qhi, o_qlo, o_khi, o_klo, o_kthi, o_ktlo, o_dct, o_bpart, o_dqbal;
};

BwdPlan bwd_plan(const Dims& D, bool balance) {
  BwdPlan P{};
  const int64_t M = D.M, HC = D.H * 2, half = D.half, NK = HC * D.n;
  P.F = M * HC * D.k;
  P.L = rowgrad_layout(P.F, NK, (int)half);
  P.cap = P.F < NK ? P.F : NK;
  int64_t o = 512;   // small words; the status word at 256, as in the forward layouts
  auto take = [&](int64_t b) {
    const int64_t at = o;
    o += (int64_t)up((size_t)(b > 0 ? b : 0));
    return at;
  };
  P.o_qraw = take(4 * M * D.H * D.dk);
  P.o_qn = take(4 * M * HC * half);
  P.o_qlen = take(4 * M * HC);
  P.o_keys = take(4 * NK * half);
  P.o_scal = take(16);
  P.o_zg = take(4 * M * D.d);
  P.o_dmemg = take(4 * M * D.d);
  P.o_memg = take(4 * M * D.d);
  P.o_dzg = take(4 * M * D.d);
  P.o_dqhat = take(4 * M * HC * half);
  P.o_dqlen = take(4 * M * HC);
  P.o_dT = take(4 * M * D.H);
  P.o_ent_s = take(4 * P.F);
  P.o_ent_w = take(4 * P.F);
  // the balance term on the tensor cores: the sub-key entries go through its
  // GEMM, so the segment-sum scratch is not needed
  P.bal_tc = balance && bal_bwd_tc_supported(D);
  P.o_rg = P.bal_tc ? 0 : take(P.L.bytes);
  P.o_uniq = P.bal_tc ? 0 : take(4 * P.cap);
  P.o_rows = P.bal_tc ? 0 : take(4 * P.cap * half);
  P.o_dkhat = take(4 * NK * half);
  P.o_dq = take(4 * M * HC * half);
  if (P.bal_tc) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    P.bp = bal_bwd_plan(D, sms);
    P.o_qhi = take(4 * P.bp.q_floats);
    P.o_qlo = take(4 * P.bp.q_floats);
    P.o_khi = take(4 * P.bp.k_floats);
    P.o_klo = take(4 * P.bp.k_floats);
    P.o_kthi = take(4 * P.bp.k_floats);
    P.o_ktlo = take(4 * P.bp.k_floats);
    P.o_dct = take(4 * P.bp.dct_floats);
    P.o_bpart = take(4 * P.bp.part_floats);
    P.o_dqbal = take(4 * M * HC * half);
  }
  P.o_cbal = (balance && !P.bal_tc) ? take(4 * HC * M * D.n) : 0;
  P.o_dTrow = balance ? take(4 * HC * M) : 0;
  P.o_dqlrow = balance ? take(4 * M * HC) : 0;
  const int64_t widest = std::max<int64_t>({(int64_t)D.H * D.dk, (int64_t)D.dm, (int64_t)D.d});
  P.o_ones = take(4 * (int64_t)colsum_scratch_floats(widest));   // column-sum partials of the bias gradients
  // the largest operand / partial scratch over the backward's GEMMs
  const int64_t NR = (int64_t)D.H * D.dk, d = D.d, dm = D.dm, n = D.n;
  const int64_t shapes[][3] = {{M, NR, dm}, {M, d, dm}, {M, d, dm}, {dm, NR, M}, {dm, d, M}, {d, dm, M},
                               {M, dm, NR}, {M, dm, d}, {M, n, half}, {M, half, n}, {n, half, M}};
  size_t g = 0;
  for (const auto& sh : shapes) {
    if ((!balance || P.bal_tc) && (sh[1] == n || sh[2] == n || sh[0] == n) && (sh[1] == half || sh[2] == half))
      continue;
    const size_t f = gemm_any_scratch_floats(sh[0], sh[1], sh[2]);
    g = f > g ? f : g;
  }
  P.gemm_floats = g;
  P.o_gemm = take(4 * (int64_t)g);
  P.bytes = o;
  return P;
}

int check_bwd(const memlayer_config* cfg, Dims* D) {
  int st = check_config(cfg, D, true);
  if (st) return st;
  if (D->half % 4 || D->half > 128) return MEMLAYER_ERR_UNSUPPORTED;
  if ((int64_t)D->H * 2 * D->n >= (1LL << 31) || D->M * D->H * 2 * D->k >= (1LL << 31)) return MEMLAYER_ERR_BAD_SHAPE;
  return MEMLAYER_OK;
}

}  // namespace

int32_t memlayer_layer_backward_workspace_size(const memlayer_config* cfg, int32_t balance, size_t* bytes) {
  Dims D;
  int st = check_bwd(cfg, &D);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  *bytes = (size_t)bwd_plan(D, balance != 0).bytes;
  return MEMLAYER_OK;
}

// The layer backward, single GPU (comm == nullptr: every step) or on a
// row-sharded table after memlayer_layer_forward_sharded, in phases:
// ROUTE = recomputed projections, d (mem * gate), probe rows published;
// GATHER = this rank's dots for every source's reads of its rows;
// REDUCE = routing backward from the owners' dots, then the local rest.
static int layer_bwd_impl(const memlayer_config* cfg, const memlayer_layer_args* a, const memlayer_layer_grads* g,
                          void* workspace, size_t workspace_bytes, cudaStream_t s, memlayer_shard_comm* comm,
                          int phases) {
  Dims D;
  int st = check_bwd(cfg, &D);
  if (st) return st;
  if (!a || !g) return MEMLAYER_ERR_BAD_POINTER;
  const memlayer_pool_args* pa = &a->pool;
  if (!pa->sub_keys || !pa->log_temperature || !pa->values) return MEMLAYER_ERR_BAD_POINTER;
  if (D.M > 0 && (!a->h || !a->w_router || !a->w_gate || !a->w_out || !pa->slots || !pa->weights || !g->dy))
    return MEMLAYER_ERR_BAD_POINTER;
  if (!aligned16(pa->values) && D.vdtype != MEMLAYER_F32) return MEMLAYER_ERR_BAD_POINTER;
  const float* fwd_mem = a->mem ? a->mem : pa->out;   // sharded: the forward's read output
  if (comm) {
    if ((st = check_shard(cfg, pa->values, comm))) return st;
    if (D.M > 0 && !fwd_mem) return MEMLAYER_ERR_BAD_POINTER;
  }
  const bool balance = g->balance_coef != 0.f;
  if (balance && (!g->forward_workspace || !pa->balance_loss)) return MEMLAYER_ERR_BAD_POINTER;
  resolve_noise(&D, cfg, pa);
  const BwdPlan P = bwd_plan(D, balance);
  if (!workspace || workspace_bytes < (size_t)P.bytes || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  const bool route = !comm || (phases & MEMLAYER_PHASE_ROUTE);
  const bool gather = comm && (phases & MEMLAYER_PHASE_GATHER);
  const bool reduce = !comm || (phases & MEMLAYER_PHASE_REDUCE);
  if (comm && route) {
    // one backward per forward: the owners' inboxes hold that forward's reads
    // (claimed by the caller once this call's launches are enqueued)
    if (comm->epoch == 0 || comm->bwd_epoch == comm->epoch) return MEMLAYER_ERR_BAD_SHAPE;
  }
  char* ws = (char*)workspace;
  auto F32p = [&](int64_t off) { return reinterpret_cast<float*>(ws + off); };
  int* small = reinterpret_cast<int*>(ws);
  const GemmScratch GS{F32p(P.o_gemm), P.gemm_floats};   // the GEMMs' operand halves and partials
  int* gerr = small + 64;                                  // the status word (offset 256)
  if (route) ML_TRY(cudaMemsetAsync(ws, 0, 512, s));
  const int64_t M = D.M, H = D.H, HC = H * 2, half = D.half, n = D.n, d = D.d, dm = D.dm, NR = H * D.dk;
  const ShardK SK = comm ? shard_k(comm, D) : ShardK{};
  float* probe = g->probe ? g->probe : F32p(P.o_dmemg);   // in place when the caller keeps no probe
  if (comm && M == 0) {
    // no tokens here: publish the empty probe, serve the other ranks' reads
    if (route) ML_TRY(launch_shard_probe(SK, 0, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, s));
    if (gather) ML_TRY(launch_shard_dots(D, SK, pa->values, small + 64, s));
    if (!reduce) return MEMLAYER_OK;
  }
  if (M == 0) {
    // no tokens: every parameter gradient is zero (dh and probe are empty)
    const struct { float* p; int64_t n; } zero[] = {
        {g->dw_router, dm * NR}, {g->db_router, NR}, {g->dsub_keys, HC * n * half}, {g->dlog_temperature, 1},
        {g->dw_gate, dm * d},    {g->db_gate, d},    {g->dw_out, d * dm},           {g->db_out, dm}};
    for (const auto& z : zero)
      if (z.p) ML_TRY(cudaMemsetAsync(z.p, 0, sizeof(float) * z.n, s));
    return MEMLAYER_OK;
  }
  float* qn = F32p(P.o_qn);
  float* qlen = F32p(P.o_qlen);
  float* keys_n = F32p(P.o_keys);
  float* scal = F32p(P.o_scal);
  LayerBwd B{pa->slots, pa->weights, F32p(P.o_dmemg), F32p(P.o_zg), qn, qlen, keys_n, scal, probe, F32p(P.o_memg),
             F32p(P.o_dzg), F32p(P.o_dqhat), F32p(P.o_dqlen), F32p(P.o_dT),
             reinterpret_cast<int*>(ws + P.o_ent_s), F32p(P.o_ent_w)};
  if (route) {
    // forward activations: unit keys and temperature (memory.py:139-146), q (model.py:110), gate input (:118)
    // (+ the tf32 halves of the unit keys and queries for the balance term's MMAs)
    ML_TRY(launch_prep_keys(D, pa->sub_keys, pa->log_temperature, cfg->min_temperature, cfg->max_temperature, keys_n,
                            P.bal_tc ? F32p(P.o_khi) : nullptr, P.bal_tc ? F32p(P.o_klo) : nullptr, scal, small + 64,
                            small + 65, s));
    ML_TRY(launch_gemm_any(a->h, dm, 1, a->w_router, NR, 1, F32p(P.o_qraw), NR, M, NR, dm, false, GS, gerr, s,
                           a->b_router));
    ML_TRY(launch_normalize_queries(D, F32p(P.o_qraw), qn, qlen, P.bal_tc ? F32p(P.o_qhi) : nullptr,
                                    P.bal_tc ? F32p(P.o_qlo) : nullptr, s));
    ML_TRY(launch_gemm_any(a->h, dm, 1, a->w_gate, d, 1, F32p(P.o_zg), d, M, d, dm, false, GS, gerr, s, a->b_gate));
    // d (mem * gate) = dy W_out^T (model.py:119)
    ML_TRY(launch_gemm_any(g->dy, dm, 1, a->w_out, 1, dm, F32p(P.o_dmemg), d, M, d, dm, false, GS, gerr, s));
    if (comm) ML_TRY(launch_shard_probe(SK, M, B.dmemg, B.zg, fwd_mem, probe, B.memg, B.dzg, s));
  }
  if (gather) ML_TRY(launch_shard_dots(D, SK, pa->values, small + 64, s));
  if (!reduce) return MEMLAYER_OK;
  if (comm) {
    const char* mine = comm->peer[comm->rank];
    const BwdShard X{reinterpret_cast<const float*>(mine + comm->off.dots),
                     reinterpret_cast<const int*>(mine + comm->off.flags_dots), SK.mcap, comm->world, comm->epoch,
                     small + 64, comm->wait_ns};
    ML_TRY(launch_route_bwd_sharded(D, B, X, s));
  } else {
    B.mem_fwd = a->mem;   // the forward's read output when the caller kept it
    ML_TRY(launch_route_bwd(D, pa->values, B, s));
  }
  float* dkhat = F32p(P.o_dkhat);
  if (balance) {
    // memory.py:205-214: the softmax over every sub-key, from the recomputed cosines
    Flags ff;
    ff.layer = true;
    ff.balance = true;
    Work FW;
    layout(D, ff, (char*)g->forward_workspace, &FW);
    if (P.bal_tc) {
      const BalBwdBufs BB{qn, F32p(P.o_qhi), F32p(P.o_qlo), keys_n, F32p(P.o_khi), F32p(P.o_klo),
                          F32p(P.o_kthi), F32p(P.o_ktlo), F32p(P.o_dct), F32p(P.o_bpart), FW.clean_cnt, qlen,
                          scal, F32p(P.o_dqbal), dkhat,
                          F32p(P.o_dTrow), F32p(P.o_dqlrow), gerr,
                          reinterpret_cast<const int*>(ws + P.o_ent_s), F32p(P.o_ent_w)};
      ML_TRY(launch_bal_bwd_tc(D, P.bp, BB, g->balance_coef, s));
    }
    float* C = P.bal_tc ? nullptr : F32p(P.o_cbal);
    for (int hc = 0; C && hc < HC; ++hc)   // cos[hc] = Q_hat[hc] K_hat[hc]^T
      ML_TRY(launch_gemm_any(qn + hc * half, HC * half, 1, keys_n + (int64_t)hc * n * half, 1, half,
                             C + (int64_t)hc * M * n, n, M, n, half, false, GS, gerr, s));
    if (C)
      ML_TRY(launch_bal_rows(D, C, FW.clean_cnt, qlen, scal, g->balance_coef, F32p(P.o_dTrow), F32p(P.o_dqlrow),
                             s));
    for (int hc = 0; C && hc < HC; ++hc) {
      // d q_hat[hc] += d cos[hc] K_hat[hc];  d k_hat[hc] = d cos[hc]^T Q_hat[hc]
      ML_TRY(launch_gemm_any(C + (int64_t)hc * M * n, n, 1, keys_n + (int64_t)hc * n * half, half, 1,
                             F32p(P.o_dqhat) + hc * half, HC * half, M, half, n, true, GS, gerr, s));
      ML_TRY(launch_gemm_any(C + (int64_t)hc * M * n, 1, n, qn + hc * half, HC * half, 1,
                             dkhat + (int64_t)hc * n * half, half, n, half, M, false, GS, gerr, s));
    }
  } else {
    ML_TRY(cudaMemsetAsync(dkhat, 0, sizeof(float) * HC * n * half, s));
  }
  // the sparse sub-key gradient: sum over entries of d cos * q_hat row, per
  // sub-key (with the balance term on the tensor cores the entries were
  // added into its d cos matrix: its GEMM gave the whole sub-key gradient)
  if (!P.bal_tc) {
    RowGradK R{};
    R.n_reads = 1;
    R.slots[0] = reinterpret_cast<const int*>(ws + P.o_ent_s);
    R.weights[0] = F32p(P.o_ent_w);
    R.grad[0] = qn;
    R.off[0] = 0;
    R.off[1] = P.F;
    R.F = P.F;
    R.N = HC * n;
    R.Nslot = HC * n;
    R.hk = D.k;
    R.d = (int)half;
    ML_TRY(launch_rowgrad(R, P.L, ws + P.o_rg, reinterpret_cast<int*>(ws + P.o_uniq), F32p(P.o_rows), nullptr,
                          nullptr, nullptr, s));
    ML_TRY(launch_scatter_rows(reinterpret_cast<const int*>(ws + P.o_uniq), F32p(P.o_rows), P.cap, HC * n,
                               (int)half, dkhat, s));
  }
  if (g->dsub_keys)
    ML_TRY(launch_norm_bwd(keys_n, dkhat, nullptr, HC * n, (int)half, pa->sub_keys, nullptr, nullptr, g->dsub_keys,
                           s));
  // d q (memory.py:136-138)
  float* dq = F32p(P.o_dq);
  ML_TRY(launch_norm_bwd(qn, F32p(P.o_dqhat), qlen, M * HC, (int)half, nullptr, D.qscale ? F32p(P.o_dqlen) : nullptr,
                         (balance && D.btgrad && D.qscale) ? F32p(P.o_dqlrow) : nullptr, dq, s,
                         P.bal_tc ? F32p(P.o_dqbal) : nullptr));
  if (g->dlog_temperature)
    ML_TRY(launch_dlogt(F32p(P.o_dT), M * H, (balance && D.btgrad) ? F32p(P.o_dTrow) : nullptr,
                        (balance && D.btgrad) ? HC * M : 0, scal, g->dlog_temperature, s));
  // Dense-layer gradients (model.py:110, 118, 119)
  float* cpart = F32p(P.o_ones);   // column-sum partials
  if (g->dw_router)
    ML_TRY(launch_gemm_any(a->h, 1, dm, dq, NR, 1, g->dw_router, NR, dm, NR, M, false, GS, gerr, s));
  if (g->db_router) ML_TRY(launch_colsum_det(dq, M, NR, NR, cpart, g->db_router, s));
  if (g->dw_gate)
    ML_TRY(launch_gemm_any(a->h, 1, dm, F32p(P.o_dzg), d, 1, g->dw_gate, d, dm, d, M, false, GS, gerr, s));
  if (g->db_gate) ML_TRY(launch_colsum_det(F32p(P.o_dzg), M, d, d, cpart, g->db_gate, s));
  if (g->dw_out)
    ML_TRY(launch_gemm_any(F32p(P.o_memg), 1, d, g->dy, dm, 1, g->dw_out, dm, d, dm, M, false, GS, gerr, s));
  if (g->db_out) ML_TRY(launch_colsum_det(g->dy, M, dm, dm, cpart, g->db_out, s));
  if (g->dh) {
    ML_TRY(launch_gemm_any(dq, NR, 1, a->w_router, 1, NR, g->dh, dm, M, dm, NR, false, GS, gerr, s));
    if (!g->route_through_pool)
      ML_TRY(launch_gemm_any(F32p(P.o_dzg), d, 1, a->w_gate, 1, d, g->dh, dm, M, dm, d, true, GS, gerr, s));
  }
  return MEMLAYER_OK;
}

int32_t memlayer_layer_backward(const memlayer_config* cfg, const memlayer_layer_args* a, const memlayer_layer_grads* g,
                                void* workspace, size_t workspace_bytes, void* stream) {
  return layer_bwd_impl(cfg, a, g, workspace, workspace_bytes, (cudaStream_t)stream, nullptr, MEMLAYER_PHASE_ALL);
}

int32_t memlayer_layer_backward_sharded(const memlayer_config* cfg, const memlayer_layer_args* a,
                                        const memlayer_layer_grads* g, memlayer_shard_comm* comm, int32_t phases,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!comm) return MEMLAYER_ERR_BAD_POINTER;
  if (!phase_mask_ok(phases, false)) return MEMLAYER_ERR_BAD_SHAPE;
  const int st = layer_bwd_impl(cfg, a, g, workspace, workspace_bytes, (cudaStream_t)stream, comm, phases);
  // the forward's inboxes are spent only once a ROUTE has been enqueued: a
  // call refused or failed before that can be retried
  if (st == MEMLAYER_OK && (phases & MEMLAYER_PHASE_ROUTE)) comm->bwd_epoch = comm->epoch;
  return st;
}

// ---- staged exchange (the caller runs the collectives between phases) ----

int32_t memlayer_layer_forward_staged(const memlayer_config* cfg, const memlayer_layer_args* a,
                                      const memlayer_staged_args* x, int32_t phases, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  Dims D;
  int st = check_config(cfg, &D, true);
  if (st) return st;
  if (!a || !x) return MEMLAYER_ERR_BAD_POINTER;
  if ((phases & MEMLAYER_PHASE_ALL) == 0 || (phases & ~MEMLAYER_PHASE_ALL)) return MEMLAYER_ERR_BAD_SHAPE;
  if (x->world < 1 || x->world > MEMLAYER_MAX_SHARDS || x->rank < 0 || x->rank >= x->world)
    return MEMLAYER_ERR_BAD_SHAPE;
  if (x->route_stride < 0 || (x->route_stride > 0 && x->route_stride < cfg->tokens * cfg->heads * cfg->top_k))
    return MEMLAYER_ERR_BAD_SHAPE;
  if (D.d % 4) return MEMLAYER_ERR_UNSUPPORTED;
  if ((st = check_pool_args(D, &a->pool, true))) return st;
  if (!aligned16(a->pool.values) || !aligned16(x->partials) || !aligned16(x->mem) || !aligned16(a->mem))
    return MEMLAYER_ERR_BAD_POINTER;
  const bool route = phases & MEMLAYER_PHASE_ROUTE, gather = phases & MEMLAYER_PHASE_GATHER,
             reduce = phases & MEMLAYER_PHASE_REDUCE;
  if (D.M > 0) {
    if (route && (!a->pool.slots || !a->pool.weights)) return MEMLAYER_ERR_BAD_POINTER;
    if (gather && (!x->all_slots || !x->all_weights || !x->partials)) return MEMLAYER_ERR_BAD_POINTER;
    if (reduce && (!x->mem || !a->w_out || !a->y)) return MEMLAYER_ERR_BAD_POINTER;
  }
  Flags f;
  f.layer = true;
  f.balance = a->pool.balance_loss != nullptr;
  const size_t need = layout(D, f, nullptr, nullptr);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  Work W;
  layout(D, f, (char*)workspace, &W);
  const cudaStream_t s = (cudaStream_t)stream;
  resolve_noise(&D, cfg, &a->pool);
  if (route) {
    if (D.M == 0) return MEMLAYER_OK;
    if ((st = layer_impl(cfg, a, workspace, workspace_bytes, s, nullptr, MEMLAYER_PHASE_ALL, false, nullptr, true)))
      return st;
  }
  if (gather)
    ML_TRY(launch_staged_gather(D, x->all_slots, x->all_weights,
                                x->route_stride > 0 ? x->route_stride : D.M * D.H * D.k, x->rank, x->world,
                                shard_rows(D.N, x->rank, x->world), a->pool.values, x->partials, W.err, s));
  if (reduce && D.M > 0) {
    if (W.h_hi) {                                                                    // model.py:119
      ML_TRY(launch_staged_gate(x->mem, W.gate, D.M * D.d, nullptr, W.memg_hi, W.memg_lo, s));
      ML_TRY(launch_out_tc(D, W, a->b_out, a->y, s));
    } else {
      ML_TRY(launch_staged_gate(x->mem, W.gate, D.M * D.d, W.memg, nullptr, nullptr, s));
      ML_TRY(launch_gemm(W.memg, a->w_out, a->b_out, a->y, D.M, D.dm, D.d, false, s));
    }
    float* mem_out = a->mem ? a->mem : a->pool.out;
    if (mem_out && mem_out != x->mem)
      ML_TRY(cudaMemcpyAsync(mem_out, x->mem, sizeof(float) * D.M * D.d, cudaMemcpyDeviceToDevice, s));
  }
  return MEMLAYER_OK;
}

// ---- layer forward reusing the previous call's preparation ----

int32_t memlayer_layer_forward_prepared(const memlayer_config* cfg, const memlayer_layer_args* a, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  Dims D;
  int st = check_config(cfg, &D, true);
  if (st) return st;
  if (!a) return MEMLAYER_ERR_BAD_POINTER;
  Flags f;
  f.layer = true;
  f.balance = a->pool.balance_loss != nullptr;
  const size_t need = layout(D, f, nullptr, nullptr);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  if (!is_prepared(workspace, cfg, a)) return MEMLAYER_ERR_WORKSPACE;   // not prepared for these arguments
  Work W;
  layout(D, f, (char*)workspace, &W);
  ML_TRY(cudaMemsetAsync(W.err, 0, sizeof(int), (cudaStream_t)stream));   // this call's status word
  return layer_impl(cfg, a, workspace, workspace_bytes, (cudaStream_t)stream, nullptr, MEMLAYER_PHASE_ALL, true);
}

// ---- host-buffer layer forward ----

int32_t memlayer_layer_host_workspace_size(const memlayer_config* cfg, int32_t chunks, size_t* bytes) {
  Dims D;
  int st = check_config(cfg, &D, true);
  if (st) return st;
  if (!bytes) return MEMLAYER_ERR_BAD_POINTER;
  *bytes = host_plan(D, chunks).bytes;
  return MEMLAYER_OK;
}

int32_t memlayer_layer_forward_host(const memlayer_config* cfg, const memlayer_layer_args* a, int32_t chunks,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  Dims D;
  int st = check_config(cfg, &D, true);
  if (st) return st;
  if (!a) return MEMLAYER_ERR_BAD_POINTER;
  const memlayer_pool_args* pa = &a->pool;
  if (pa->subkey_counts || pa->slot_counts || pa->balance_loss || pa->top1_weight) return MEMLAYER_ERR_UNSUPPORTED;
  if (D.M > 0 && (!a->h || !a->y)) return MEMLAYER_ERR_BAD_POINTER;
  const HostPlan P = host_plan(D, chunks);
  if (!workspace || workspace_bytes < P.bytes || (reinterpret_cast<uintptr_t>(workspace) % ALIGN))
    return MEMLAYER_ERR_WORKSPACE;
  if (D.M == 0) return layer_impl(cfg, a, workspace, P.work_bytes, (cudaStream_t)stream, nullptr,
                                  MEMLAYER_PHASE_ALL);
  cudaStream_t s = (cudaStream_t)stream, cin = nullptr, cout = nullptr;
  if ((st = copy_streams(&cin, &cout))) return st;
  float* stage_h = reinterpret_cast<float*>((char*)workspace + P.work_bytes);
  float* stage_y = reinterpret_cast<float*>((char*)workspace + P.stage_off_y);
  // the chunks share one chunk-sized workspace layout
  memlayer_config cc = *cfg;
  cc.tokens = P.mc;
  Dims Dc;
  if ((st = check_config(&cc, &Dc, true))) return st;
  Flags f;
  f.layer = true;
  Work W;
  layout(Dc, f, (char*)workspace, &W);
  const int n = P.chunks;
  cudaEvent_t ev[2 * MEMLAYER_HOST_MAX_CHUNKS + 2];
  const int nev = 2 * n + 2;
  if (n > MEMLAYER_HOST_MAX_CHUNKS) return MEMLAYER_ERR_BAD_SHAPE;
  for (int i = 0; i < nev; ++i)
    if (cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaEventDestroy(ev[j]);
      return MEMLAYER_ERR_CUDA;
    }
  auto run = [&]() -> int {
    // copies start after the caller's earlier work on `stream` (staging reuse)
    ML_TRY(cudaEventRecord(ev[2 * n], s));
    ML_TRY(cudaStreamWaitEvent(cin, ev[2 * n], 0));
    ML_TRY(cudaStreamWaitEvent(cout, ev[2 * n], 0));
    for (int c = 0; c < n; ++c) {
      const int64_t t0 = c * P.mc, tn = (c + 1 == n) ? D.M - t0 : P.mc;
      ML_TRY(cudaMemcpyAsync(stage_h + t0 * D.dm, a->h + t0 * D.dm, sizeof(float) * tn * D.dm,
                             cudaMemcpyHostToDevice, cin));
      ML_TRY(cudaEventRecord(ev[c], cin));
    }
    for (int c = 0; c < n; ++c) {
      const int64_t t0 = c * P.mc, tn = (c + 1 == n) ? D.M - t0 : P.mc;
      memlayer_config ck = *cfg;
      ck.tokens = tn;
      memlayer_layer_args ak = *a;
      memlayer_pool_args& pk = ak.pool;
      ak.h = stage_h + t0 * D.dm;
      ak.y = stage_y + t0 * D.dm;
      if (a->mem) ak.mem = a->mem + t0 * D.d;
      if (pa->out) pk.out = pa->out + t0 * D.d;
      if (pa->slots) pk.slots = pa->slots + t0 * D.H * D.k;
      if (pa->weights) pk.weights = pa->weights + t0 * D.H * D.k;
      if (pa->gumbel) pk.gumbel = pa->gumbel + t0 * D.H * 2 * D.n;
      if (pa->queries_unit) pk.queries_unit = pa->queries_unit + t0 * D.H * D.dk;
      pk.temperature = (c + 1 == n) ? pa->temperature : nullptr;
      pk.stage_events = nullptr;
      ML_TRY(cudaStreamWaitEvent(s, ev[c], 0));
      int r = layer_impl(&ck, &ak, workspace, P.work_bytes, s, nullptr, MEMLAYER_PHASE_ALL, c > 0, &W);
      if (r) return r;
      ML_TRY(cudaEventRecord(ev[n + c], s));
      ML_TRY(cudaStreamWaitEvent(cout, ev[n + c], 0));
      ML_TRY(cudaMemcpyAsync(a->y + t0 * D.dm, stage_y + t0 * D.dm, sizeof(float) * tn * D.dm,
                             cudaMemcpyDeviceToHost, cout));
    }
    ML_TRY(cudaEventRecord(ev[2 * n + 1], cout));
    ML_TRY(cudaStreamWaitEvent(s, ev[2 * n + 1], 0));   // the caller's stream covers the whole call
    return MEMLAYER_OK;
  };
  st = run();
  for (int i = 0; i < nev; ++i) cudaEventDestroy(ev[i]);   // released once the recorded work completes
  return st;
}

}  // extern "C"
