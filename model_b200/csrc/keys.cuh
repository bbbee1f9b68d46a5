// Sub-key maintenance kernels (key_diversity_loss, revive_dead_keys).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ml {

struct KeyDivLayout {
  int64_t o_Mpart, o_M, o_lpart, o_sqpart, bytes;
};

KeyDivLayout key_div_layout(int HC, int n, int d);

// loss (1 float) and/or grad ([HC, n, d], scaled by `scale`) may be null.
cudaError_t launch_key_diversity(const float* sub_keys, int HC, int n, int d, char* ws, float* loss, float* grad,
                                 float scale, cudaStream_t s);

// In place on keys [HC, n, d] and usage [HC, n]; dead [HC, n], m0 and m1
// ([HC, n, d], zeroed on revived rows) may be null.
cudaError_t launch_revive(float* keys, float* usage, const float* queries, int64_t tokens, const int* pick,
                          const float* noise, int HC, int n, int d, float threshold, float noise_scale, int* dead,
                          float* m0, float* m1, cudaStream_t s);

}  // namespace ml
