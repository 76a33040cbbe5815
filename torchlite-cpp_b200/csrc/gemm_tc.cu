// Tensor-core GEMM (TF32 / 3xTF32) on tcgen05: placeholder until the kernel lands.
#include "common.cuh"

namespace tlc {
int gemm_tc(const Gemm&, int, cudaStream_t) {
    return set_error(TLC_ERR_UNSUPPORTED, "tensor-core modes are not built yet");
}
}  // namespace tlc
