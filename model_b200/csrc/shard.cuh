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
  int64_t tickets;     // [2][2] int: CTA completion counters of push / gather (local use)
  int64_t cnt;         // [world][mcap] int: entries from source rank per token
  int64_t inbox;       // [world][mcap][hk] int2: (local row, weight bits) per entry
  int64_t part;        // [world][mcap][d] float: partial sum of owner rank per token
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
  // token half of this launch: flags / tickets / meta slots `hf`, this rank's
  // tokens [t0, t1), gather grid over `span` tokens per source rank
  int hf;
  int64_t t0, t1, span;
};

ShardOff shard_layout(int world, int64_t mcap, int hk, int d);

// Stage 2 + push of (local row, weight) entries to the owner ranks
// (replaces launch_combine_gather in the sharded forward).
cudaError_t launch_shard_push(const Dims& D, const Work& W, const ShardK& S, int* slots, float* weights,
                              float* slot_counts, float* subkey_counts, int* own_cnt, cudaStream_t s);
// Owner side: gather local rows for every source rank's tokens and store the
// partial sums into the token owners' buffers.
cudaError_t launch_shard_gather(const Dims& D, const ShardK& S, const void* values_local, int* err,
                                cudaStream_t s);
// Token-owner side: sum the owners' partials in rank order, apply the gate.
cudaError_t launch_shard_reduce(const Dims& D, const ShardK& S, const int* own_cnt, const float* gate, float* out,
                                float* memg, float* memg_hi, float* memg_lo, int* err, cudaStream_t s);

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
};
