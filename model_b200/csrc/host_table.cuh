// Value table in page-locked host memory: fetch of the distinct rows into
// an HBM staging buffer, and the weighted mix from it.
#pragma once

#include "common.cuh"

namespace ml {

int64_t table_elem_bytes(int vdtype);

// Calls with at most this many fetches dedup their read slots in one CTA.
constexpr int TABLE_SMALL_F = 4096;

// uniq / *n_seg / inv of F <= TABLE_SMALL_F fetches (read slot = (s + kadd) % N when kadd > 0).
cudaError_t launch_table_unique_small(const int* slots, int F, int64_t N, int64_t kadd, int* uniq, int* n_seg,
                                      int* inv, cudaStream_t s);

// staging[u] = table[uniq[u]] for u < *n_seg (cap rows of staging).
cudaError_t launch_table_fetch(const Dims& D, const void* table, const int* uniq, const int* n_seg, int64_t cap,
                               void* staging, int* err, cudaStream_t s);

// out[m] = sum over heads and ranks of weights * staging[inv].
cudaError_t launch_table_mix(const Dims& D, const void* staging, const int* inv, const float* weights, float* out,
                             cudaStream_t s);

}  // namespace ml
