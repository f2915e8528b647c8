// Tensor-core (tcgen05) Float32 contractions of the mlp2_ce adjoint.
// Declarations; the kernels live in tc_gemm.cu.
#pragma once

#include "common.cuh"

namespace stade {

// Whether the tcgen05 path handles these sizes (otherwise the SIMT path runs).
bool tc_mlp_supported(int64_t n_s, int64_t n_i, int64_t n_h);
size_t tc_mlp_workspace(int64_t n_s, int64_t n_i, int64_t n_h);

// h = tanh(x W1 + b1); x: S x I, W1: I x H.
stade_status tc_forward_tanh(const float* x, const float* w1, const float* b1, float* h, int S,
                             int I, int H, void* ws, cudaStream_t s);
// w1b += x^T s1b, b1b += colsum(s1b).
stade_status tc_weight_grad(const float* x, const float* s1b, float* w1b, float* b1b, int S, int I,
                            int H, void* ws, cudaStream_t s);
// xb += s1b W1^T.
stade_status tc_input_grad(const float* s1b, const float* w1, float* xb, int S, int I, int H,
                           void* ws, cudaStream_t s);

}  // namespace stade
