// Fused EXL3 projection: host dispatch over codebook and row count (kernels in sx_gemv_impl.cuh,
// instantiated per codebook in sx_gemv_{mcg,mul1,hash,pair1}.cu).
#include "sx_kernels.h"
#include "sx_decode.cuh"

namespace sx {

template <int KIND, int NB>
cudaError_t dispatch_n(const GemvArgs& a, int n, int groups, int S, cudaStream_t stream);

// Shared memory of one GEMV CTA (sx_core.cuh core_layout with NP = 1), computed at run time.
size_t gemv_smem_bytes(int n, int nb, int in, int S) {
    const int KB = in / 128;
    const int kbl_max = (KB + S - 1) / S;
    const int stage = 64 * n * 2;
    const int nst = stage <= 5120 ? 8 : (stage <= 10240 ? 6 : 4);
    return (size_t)nst * stage + (size_t)kbl_max * 8 * nb * 32 * 16 + (size_t)nb * 8 * 128 * 4 + 2 * nst * 8;
}

cudaError_t launch_gemv(const GemvArgs& a, int kind, int n, int groups, int S, cudaStream_t stream) {
    const int nb = (a.rows + 7) / 8;
    switch (kind * 4 + nb) {
        case K_MUL1 * 4 + 1: return dispatch_n<K_MUL1, 1>(a, n, groups, S, stream);
        case K_MUL1 * 4 + 2: return dispatch_n<K_MUL1, 2>(a, n, groups, S, stream);
        case K_MCG * 4 + 1: return dispatch_n<K_MCG, 1>(a, n, groups, S, stream);
        case K_MCG * 4 + 2: return dispatch_n<K_MCG, 2>(a, n, groups, S, stream);
        case K_HASH * 4 + 1: return dispatch_n<K_HASH, 1>(a, n, groups, S, stream);
        case K_HASH * 4 + 2: return dispatch_n<K_HASH, 2>(a, n, groups, S, stream);
        case K_PAIR1 * 4 + 1: return dispatch_n<K_PAIR1, 1>(a, n, groups, S, stream);
        case K_PAIR1 * 4 + 2: return dispatch_n<K_PAIR1, 2>(a, n, groups, S, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace sx
