// Tensor-core path of conv1d_relu_mse_b (conv_tc.cu).
#pragma once

#include "common.cuh"

namespace stade {

struct ConvShape {
  int64_t n_b, n_c, n_l, n_o, n_k;
};

// Whether the tcgen05 path takes these sizes (TMA needs 16-byte row pitches:
// n_c and n_o multiples of 4).
bool conv_tc_supported(const ConvShape& sh);
size_t conv_tc_workspace(const ConvShape& sh);
stade_status conv_tc_run(const ConvShape& sh, float* loss, const float* lossb, const float* x,
                         float* xb, const float* w, float* wb, const float* t, float* tb, float* z,
                         float* zb, float* r, float* rb, void* ws, cudaStream_t s);
// Reads and clears the kernel's error word (-1 when it cannot be read).
int conv_tc_take_error();

}  // namespace stade
