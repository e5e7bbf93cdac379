// Tensor-core projection kernels for one codebook family (sx_gemm_impl.cuh).
#include "sx_gemm_launch.cuh"

namespace sx {
template cudaError_t gemm_dispatch<K_MUL1>(const CUtensorMap&, const GemmArgs&, int, int, int, int, cudaStream_t, bool, int);
}  // namespace sx
