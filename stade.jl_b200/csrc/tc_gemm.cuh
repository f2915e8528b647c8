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
// h = tanh(x W1 + b1) and the logits' partial sums zpart[part][s][c] over
// disjoint sets of hidden units (tc_logit_parts(H) parts; n_o = O <= 32).
int tc_logit_parts(int64_t n_h);
stade_status tc_forward_tanh_logits(const float* x, const float* w1, const float* b1,
                                    const float* w2, float* h, float* zpart, int S, int I, int H,
                                    int O, cudaStream_t s);
// w1b += x^T s1b, b1b += colsum(s1b).
stade_status tc_weight_grad(const float* x, const float* s1b, float* w1b, float* b1b, int S, int I,
                            int H, void* ws, cudaStream_t s);
// xb += s1b W1^T.
stade_status tc_input_grad(const float* s1b, const float* w1, float* xb, int S, int I, int H,
                           void* ws, cudaStream_t s);

// ---- TMA-fed path (tc_tma.cu): operands as TF32 hi / lo planes --------------
stade_status tma_split(const float* a, float* hi, float* lo, int64_t n, cudaStream_t s);
// lo plane only (the array is its own hi plane for kind::tf32)
stade_status tma_split_lo(const float* a, float* lo, int64_t n, cudaStream_t s);
size_t tma_w1b_part_floats(int64_t n_s, int64_t n_i, int64_t n_h);
stade_status tma_forward_tanh_logits(const float* x_hi, const float* x_lo, const float* w1_hi,
                                     const float* w1_lo, const float* b1, const float* w2,
                                     float* h, float* zpart, int S, int I, int H, int O,
                                     cudaStream_t s);
stade_status tma_weight_grad(const float* x_hi, const float* x_lo, const float* s1b_hi,
                             const float* s1b_lo, float* w1b, float* part, int S, int I, int H,
                             cudaStream_t s);
stade_status tma_input_grad(const float* s1b_hi, const float* s1b_lo, const float* w1_hi,
                            const float* w1_lo, float* xb, int S, int I, int H, cudaStream_t s);

}  // namespace stade
