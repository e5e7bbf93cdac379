// MoE decode-chain instantiations for the MUL1 codebook family.
#include "sx_moe_launch.cuh"

namespace sx {
template cudaError_t moe_launch_kind<K_MUL1>(const MoeArgs&, int, int, int, int, int, cudaStream_t);
template cudaError_t moe_launch_kind_direct<K_MUL1>(const MoeArgs&, int, int, int, int, cudaStream_t);
}  // namespace sx
