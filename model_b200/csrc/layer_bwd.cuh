// Backward of one memory layer: internal launchers (layer_bwd.cu).
#pragma once

#include "common.cuh"

namespace ml {

// Buffers of the routing backward kernel (one CTA per token).
struct LayerBwd {
  const int* slots;        // [M, H, k] the forward's slots
  const float* weights;    // [M, H, k] the forward's weights
  const float* dmemg;      // [M, d] d loss / d (mem * gate)
  const float* zg;         // [M, d] gate pre-activation h W_gate + b_gate
  const float* qn;         // [M, H, 2, half] unit query halves
  const float* qlen;       // [M, H, 2]
  const float* keys_n;     // [H * 2, n, half] unit sub-keys
  const float* scal;       // [1] temperature
  float* probe;            // [M, d] d loss / d read output
  float* memg;             // [M, d] mem * gate
  float* dzg;              // [M, d]
  float* dqhat;            // [M, H, 2, half]
  float* dqlen;            // [M, H, 2]
  float* dT_part;          // [M * H]
  int* ent_slot;           // [M, H, 2, k] (codebook * n + sub-key) of each slot-score gradient entry
  float* ent_w;            // [M, H, 2, k] its d cos
  const float* mem_fwd = nullptr;   // [M, d] the forward's read output, or nullptr: recomputed from the rows
};

// Row-sharded table: where the routing backward finds the per-read dots
// probe . V[read slot] that the owner ranks stored (shard.cu), and the flags
// (one per owner, in this rank's buffer) that say they are complete.
struct BwdShard {
  const float* dots;   // [world][mcap][H * k] in each owner's inbox order
  const int* flags;    // [world] epoch of each owner's dots
  int64_t mcap;
  int world, epoch;
  int* err;            // status word (36: an owner's dots did not arrive in time)
  long long wait_ns;   // budget of the wait
};

cudaError_t launch_fill(float* x, int64_t n, float v, cudaStream_t s);
cudaError_t launch_route_bwd(const Dims& D, const void* values, const LayerBwd& B, cudaStream_t s);
// The routing backward of the row-sharded layer: dw from the owners' dots
// (values are not read; probe / memg / dzg already written by the probe kernel).
cudaError_t launch_route_bwd_sharded(const Dims& D, const LayerBwd& B, const BwdShard& X, cudaStream_t s);
// C: [H * 2][M][n] cosines in, d cos out (balance term)
cudaError_t launch_bal_rows(const Dims& D, float* C, const float* cnt, const float* qlen, const float* scal, float coef,
                            float* dT_row, float* dql_row, cudaStream_t s);
// dx from d x_hat (+ dxhat2, a second share of it, when given)
cudaError_t launch_norm_bwd(const float* xhat, const float* dxhat, const float* len, int64_t rows, int half,
                            const float* raw, const float* dlen, const float* dlen2, float* dx, cudaStream_t s,
                            const float* dxhat2 = nullptr);
cudaError_t launch_scatter_rows(const int* uniq, const float* rows, int64_t cap, int64_t N, int half, float* dst,
                                cudaStream_t s);
cudaError_t launch_dlogt(const float* a, int64_t na, const float* b, int64_t nb, const float* scal, float* out,
                         cudaStream_t s);

}  // namespace ml
