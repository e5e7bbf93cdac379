// MoE decode-chain instantiations for the HASH codebook family.
#include "sx_moe_launch.cuh"

namespace sx {
template cudaError_t moe_launch_kind<K_HASH>(const MoeArgs&, int, int, int, int, int, cudaStream_t);
template cudaError_t moe_launch_kind_direct<K_HASH>(const MoeArgs&, int, int, int, int, cudaStream_t);
}  // namespace sx
