// TMA-fed tensor-core (tcgen05) Float32 contractions of the mlp2_ce adjoint
// (3xTF32 on hi / lo operand planes). Declarations; the kernels live in
// tc_tma.cu.
#pragma once

#include "common.cuh"

namespace stade {

// Whether the tensor-core path handles these sizes (TMA needs 16-byte row
// pitches; otherwise the CUDA-core path runs).
bool tma_mlp_supported(int64_t n_s, int64_t n_i, int64_t n_h);
// Partial sums of the logits the forward GEMM's epilogue writes when w2 does
// not fit in shared memory: zpart[part][s][c] over disjoint sets of hidden
// units.
int tma_logit_parts(int64_t n_h);

// x's and W1's TF32 lo planes in one launch (each array is its own hi plane
// for kind::tf32; n0, n1 > 0)
stade_status tma_split_lo2(const float* a0, float* lo0, int64_t n0, const float* a1, float* lo1,
                           int64_t n1, cudaStream_t s);
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
