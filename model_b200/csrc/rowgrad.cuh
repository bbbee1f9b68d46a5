// Fetched-row gradients / row-wise Adagrad: internal launch descriptors.
#pragma once

#include "common.cuh"

namespace ml {

// The reads whose fetches are merged (memory layers sharing one pool).
struct RowGradK {
  const int* slots[MEMLAYER_MAX_READS];
  const float* weights[MEMLAYER_MAX_READS];
  const float* grad[MEMLAYER_MAX_READS];
  int64_t off[MEMLAYER_MAX_READS + 1];   // first fetch of each read; off[n_reads] = F
  int n_reads;
  int64_t F;    // fetches in all reads
  int64_t N;    // key space: pool rows, or world * kstride with owner-grouped keys
  int64_t Nslot;    // pool rows (slot ids must lie in [0, Nslot))
  int kworld;       // > 1: sort key of slot s = (s % kworld) * kstride + s / kworld
  int64_t kstride;
  int64_t kadd;     // > 0: sort key of slot s = (s + kadd) % Nslot (the read slot under shuffle_reads)
  int hk;       // heads * top_k
  int d;        // d_value
};

// Byte offsets of the workspace regions (all 256-byte aligned).
struct RowGradLayout {
  int passes, rbits;
  int64_t nblk, nseg_blk, chunks, groups, cap;
  int64_t o_small, o_err, o_keys_a, o_vals_a, o_keys_b, o_vals_b, o_hist, o_dtot, o_segtot, o_seg_id, o_seg_start, o_uniq,
      o_rows, o_rowsq, o_spill, o_grp, o_part, o_sq, bytes;
};

struct RowAdagrad {
  float* values;
  float* accum;
  float lr;
  float clip;
  const float* rest_sq;
  float* scale_out;
  int* n_unique_out;
};

RowGradLayout rowgrad_layout(int64_t F, int64_t N, int d);
cudaError_t launch_rowgrad(const RowGradK& R, const RowGradLayout& L, char* ws, int* uniq_out, float* rows_out,
                           int* n_unique_out, float* sq_out, const RowAdagrad* ada, cudaStream_t s);

// Sort + segments only: the distinct keys in ascending order at L.o_uniq,
// their count at small[1] (L.o_small), and for every fetch f its segment:
// inv[f] = index of its key in uniq (out-of-range slots: -1).
cudaError_t launch_sort_unique(const RowGradK& R, const RowGradLayout& L, char* ws, int* inv, cudaStream_t s);

}  // namespace ml
