// GEMV instantiations: MCG codebook family, 2 row group(s).
#include "sx_gemv_impl.cuh"

namespace sx {
template cudaError_t dispatch_n<K_MCG, 2, true>(const GemvArgs&, int, int, cudaStream_t);
template cudaError_t dispatch_n<K_MCG, 2, false>(const GemvArgs&, int, int, cudaStream_t);
}  // namespace sx
