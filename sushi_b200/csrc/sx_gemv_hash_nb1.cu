// GEMV instantiations: HASH codebook family, 1 row group(s).
#include "sx_gemv_impl.cuh"

namespace sx {
template cudaError_t dispatch_n<K_HASH, 1, true>(const GemvArgs&, int, int, cudaStream_t);
template cudaError_t dispatch_n<K_HASH, 1, false>(const GemvArgs&, int, int, cudaStream_t);
}  // namespace sx
