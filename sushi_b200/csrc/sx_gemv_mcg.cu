// GEMV instantiations for the MCG codebook family.
#include "sx_gemv_impl.cuh"

namespace sx {
template cudaError_t dispatch_n<K_MCG, 1>(const GemvArgs&, int, int, int, cudaStream_t);
template cudaError_t dispatch_n<K_MCG, 2>(const GemvArgs&, int, int, int, cudaStream_t);
}  // namespace sx
