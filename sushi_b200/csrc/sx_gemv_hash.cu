// GEMV instantiations for the HASH codebook family.
#include "sx_gemv_impl.cuh"

namespace sx {
template cudaError_t dispatch_n<K_HASH, 1>(const GemvArgs&, int, int, int, cudaStream_t);
template cudaError_t dispatch_n<K_HASH, 2>(const GemvArgs&, int, int, int, cudaStream_t);
}  // namespace sx
