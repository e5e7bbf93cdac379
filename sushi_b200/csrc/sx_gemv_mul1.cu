// GEMV instantiations for the MUL1 codebook family.
#include "sx_gemv_impl.cuh"

namespace sx {
template cudaError_t dispatch_n<K_MUL1, 1>(const GemvArgs&, int, int, int, cudaStream_t);
template cudaError_t dispatch_n<K_MUL1, 2>(const GemvArgs&, int, int, int, cudaStream_t);
}  // namespace sx
