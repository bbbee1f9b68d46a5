// Row-sharded pool over the GPUs of one node: internal types shared by the
// communicator / launch code (shard.cu) and the C ABI (capi.cu).
#pragma once

#include "common.cuh"

namespace ml {

// Byte offsets inside a communicator buffer.  Every rank's buffer has the
// same layout, so a rank addresses a peer's region with the peer's base.
struct ShardOff {
  int64_t flags_in;    // [2 halves][MAX] int: epoch of the inbox each source rank has filled
  int64_t flags_part;  // [2][MAX] int: epoch of the partials each owner rank has stored
  int64_t meta;        // [2][MAX][2] int: token range [lo, hi) of each source rank's half
  int64_t tickets;     // [2][2] int: CTA completion counters of push / gather (local use);
                       // [4], [5]: probe / dots kernels of the backward;
                       // [16 + 8 * half + source]: the gather's unit counters (local use)
  int64_t flags_probe; // [MAX] int (backward): epoch of the probe rows each source rank has stored
  int64_t flags_dots;  // [MAX] int (backward): epoch of the dots each owner rank has stored
  int64_t bmeta;       // [MAX] int (backward): token count of each source rank's call
  int64_t cnt;         // [world][mcap] int: entries from source rank per token
  int64_t inbox;       // [world][mcap][hk] int2: (local row, weight bits) per entry
  int64_t part;        // [world][mcap][d] float: partial sum of owner rank per token
  int64_t probe;       // [mcap][d] float (backward): this rank's d loss / d read output
  int64_t dots;        // [world][mcap][hk] float (backward): probe . row per inbox entry, from each owner
  int64_t bytes;       // total
};

// What a kernel needs to reach every rank's buffer.
struct ShardK {
  char* peer[MEMLAYER_MAX_SHARDS];  // base of each rank's buffer, device-visible from this GPU
  ShardOff off;
  int rank, world;
  int64_t mcap;    // per-rank token capacity
  int hk;          // heads * top_k: entries per token
  int d;           // d_value
  int64_t rows;    // value rows held by this rank
  int epoch;       // current call
  long long wait_ns;  // budget of each wait on another rank (communicator setting)
  // token half of this launch: flags / tickets / meta slots `hf`, this rank's
  // tokens [t0, t1), gather grid over `span` tokens per source rank
  int hf;
  int64_t t0, t1, span;
};

// ---- hand-off between ranks through flags in peer memory ----
constexpr long long kPeerWaitNs = 2000000000LL;   // default wait budget: 2 s

__device__ __forceinline__ long long global_ns() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Wait until *flag has reached epoch (wrap-safe).  Gives up after `budget_ns`
// of the global timer, or at once when another wait of this call already gave up.
// The polls back off (64 ns doubling to 2 us): many waiting CTAs would
// otherwise flood the L2 slice that holds the flag, which is also where the
// peers' stores for this call land.
__device__ inline bool wait_epoch(const int* flag, int epoch, int* err, int code, long long budget_ns) {
  if (ld_acquire_sys(flag) - epoch >= 0) return true;
  const long long t0 = global_ns();
  unsigned backoff = 64;
  while (true) {
    if (*(volatile int*)err != 0) return false;
    __nanosleep(backoff);
    backoff = backoff < 2048 ? backoff * 2 : 2048;
    if (ld_acquire_sys(flag) - epoch >= 0) return true;
    if (global_ns() - t0 > budget_ns) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
}

ShardOff shard_layout(int world, int64_t mcap, int hk, int d);

// ---- owner-sharded row update (training) ----
// Byte offsets inside a row-update communicator buffer (same on every rank).
struct RowShardOff {
  int64_t flags_in;   // [MAX] int: epoch of the row list each source rank has pushed
  int64_t flags_sq;   // [MAX] int: epoch of the squared-norm partial each owner rank has stored
  int64_t tickets;    // [4] int: CTA completion counter of the push (local use)
  int64_t cnt;        // [MAX] int: rows pushed by each source rank
  int64_t sq;         // [MAX] double: each owner rank's sum of its merged rows^2
  int64_t lin;        // [world][cap] int: local row of each pushed row (ascending per source)
  int64_t rin;        // [world][cap][d] float: the pushed row gradients
  int64_t bytes;
};

struct RowShardK {
  char* peer[MEMLAYER_MAX_SHARDS];
  RowShardOff off;
  int rank, world;
  int64_t cap;      // rows per (source, owner) inbox
  int64_t stride;   // ceil(pool rows / world): owner-grouped key = owner * stride + local row
  int64_t rows;     // value rows held by this rank
  int d;
  int epoch;
  long long wait_ns;  // budget of each wait on another rank
};

RowShardOff row_shard_layout(int world, int64_t cap, int d);

// Pointers of the merge region of a sharded row-update workspace.
struct RowMerge {
  int* small;      // [0] merged entries T, [1] touched local rows
  int* mkey;       // [world * cap] local row of each merged entry (stable by source rank)
  int* mref;       // [world * cap] inbox entry (source * cap + index) of each merged entry
  int* head;       // [world * cap] 1 at the first entry of each local row
  float* rowsq;    // [world * cap] squared norm of each merged row (at its head)
  float* mrow;     // [world * cap][d] merged row gradient (at its head)
};

// ROUTE: push this rank's merged rows (owner-grouped keys, ascending) to the owners.
cudaError_t launch_rows_push(const RowShardK& K, const int* uniq, const float* rows, const int* n_seg, int64_t ucap,
                             int* err, cudaStream_t s);
// GATHER: merge the sources' row lists in rank order, publish this owner's squared norm.
cudaError_t launch_rows_merge(const RowShardK& K, const RowMerge& G, int* err, cudaStream_t s);
// REDUCE: global-norm clip over every owner's partial, row-wise Adagrad on this rank's rows.
cudaError_t launch_rows_apply(const RowShardK& K, const RowMerge& G, float* values, float* accum, float lr,
                              float clip, const float* rest_sq, float* scale_out, int* n_unique_out, int* err,
                              cudaStream_t s);

// After stage 2 (routing only) of tokens [S.t0, S.t1): store every (local
// row, weight) entry into its owner rank's inbox and publish the inbox.
cudaError_t launch_shard_scatter(const Dims& D, const ShardK& S, const int* slots, const float* weights,
                                 int* own_cnt, int* err, cudaStream_t s);
// Owner side: gather local rows for every source rank's tokens and store the
// partial sums into the token owners' buffers.
cudaError_t launch_shard_gather(const Dims& D, const ShardK& S, const void* values_local, int* err,
                                cudaStream_t s);
// Token-owner side: sum the owners' partials in rank order, apply the gate.
cudaError_t launch_shard_reduce(const Dims& D, const ShardK& S, const int* own_cnt, const float* gate, float* out,
                                float* memg, float* memg_hi, float* memg_lo, int* err, cudaStream_t s);

// ---- staged exchange: the caller's collectives run between the phases ----
// For every token of every rank (world * D.M, rank-major; rank o's entries
// start at o * stride), the sum of w * V[local row] over the entries this
// rank owns -> partials [world * D.M][d].
cudaError_t launch_staged_gather(const Dims& D, const int* slots, const float* weights, int64_t stride, int rank,
                                 int world, int64_t rows, const void* values, float* partials, int* err,
                                 cudaStream_t s);
// mem * gate for the output projection (float32 product or tf32 halves).
cudaError_t launch_staged_gate(const float* mem, const float* gate, int64_t n, float* memg, float* memg_hi,
                               float* memg_lo, cudaStream_t s);

// ---- backward of the sharded layer (after its forward, on the same communicator) ----
// Reader side: probe = dmemg * silu(zg) (model.py:118-119) for this rank's
// M tokens, stored into the caller's probe and this rank's buffer, with
// memg = mem * gate and dzg; then publishes the probe rows and M to every rank.
cudaError_t launch_shard_probe(const ShardK& S, int64_t M, const float* dmemg, const float* zg, const float* mem,
                               float* probe, float* memg, float* dzg, cudaStream_t s);
// Owner side: for every inbox entry of the forward, probe . V[local row]
// (lanes over d, then a warp sum: the single-GPU backward's order), stored
// into the source rank's dots.
cudaError_t launch_shard_dots(const Dims& D, const ShardK& S, const void* values_local, int* err, cudaStream_t s);

}  // namespace ml

// The communicator behind the C ABI's opaque memlayer_shard_comm.
struct memlayer_shard_comm {
  int rank = 0, world = 1, device = 0;
  memlayer_config cfg{};                      // shapes the buffers were sized for (tokens = capacity)
  ml::ShardOff off{};
  char* base = nullptr;                       // this rank's buffer (cudaMalloc at create)
  char* peer[MEMLAYER_MAX_SHARDS] = {};       // every rank's buffer as seen from this GPU
  bool opened[MEMLAYER_MAX_SHARDS] = {};      // mapped through cudaIpcOpenMemHandle
  int epoch = 0;                              // last call started by the route phase
  int bwd_epoch = 0;                          // forward epoch whose backward has started
  long long wait_ns = ml::kPeerWaitNs;        // budget of each wait on another rank
  // kind 1: row-update communicator (memlayer_shard_comm_create_rowgrad)
  int kind = 0;
  int n_reads = 0;                            // reads (memory layers) per call it was sized for
  int64_t rcap = 0;                           // rows per (source, owner) inbox
  ml::RowShardOff roff{};
};
