// Value table in page-locked host memory: fetch of the distinct rows into
// an HBM staging buffer, and the weighted mix from it.
#pragma once

#include "common.cuh"

namespace ml {

int64_t table_elem_bytes(int vdtype);

// staging[u] = table[uniq[u]] for u < *n_seg (cap rows of staging).
cudaError_t launch_table_fetch(const Dims& D, const void* table, const int* uniq, const int* n_seg, int64_t cap,
                               void* staging, int* err, cudaStream_t s);

// out[m] = sum over heads and ranks of weights * staging[inv].
cudaError_t launch_table_mix(const Dims& D, const void* staging, const int* inv, const float* weights, float* out,
                             cudaStream_t s);

}  // namespace ml
