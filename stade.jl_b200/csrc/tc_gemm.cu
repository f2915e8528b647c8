// Tensor-core (tcgen05) Float32 contractions of the mlp2_ce adjoint.
#include "tc_gemm.cuh"

namespace stade {

bool tc_mlp_supported(int64_t, int64_t, int64_t) { return false; }
size_t tc_mlp_workspace(int64_t, int64_t, int64_t) { return 0; }

stade_status tc_forward_tanh(const float*, const float*, const float*, float*, int, int, int, void*,
                             cudaStream_t) {
  return fail(STADE_ENOTSUP, "tcgen05 path not built");
}
stade_status tc_weight_grad(const float*, const float*, float*, float*, int, int, int, void*,
                            cudaStream_t) {
  return fail(STADE_ENOTSUP, "tcgen05 path not built");
}
stade_status tc_input_grad(const float*, const float*, float*, int, int, int, void*, cudaStream_t) {
  return fail(STADE_ENOTSUP, "tcgen05 path not built");
}

}  // namespace stade
