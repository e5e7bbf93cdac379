// GEMV instantiations: MUL1 codebook family, 2 row group(s).
#include "sx_gemv_impl.cuh"

namespace sx {
template cudaError_t dispatch_n<K_MUL1, 2, true>(const GemvArgs&, int, int, cudaStream_t);
template cudaError_t dispatch_n<K_MUL1, 2, false>(const GemvArgs&, int, int, cudaStream_t);
}  // namespace sx
