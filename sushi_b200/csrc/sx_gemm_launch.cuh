// Launch of the tensor-core projection (sx_gemm_impl.cuh) over the admitted rates, per codebook
// (included by sx_gemm_{mcg,mul1,hash,pair1}.cu).
#pragma once

#include "sx_gemm_impl.cuh"
#include "sx_kernels.h"

namespace sx {

// The largest split <= S whose clusters (`clusters` of them, S CTAs each) are all co-resident, so
// no cluster waits for another to drain (cached per kernel, cluster count and split); 1 if none.
int gemm_coresident_split(const void* kern, int smem, int threads, dim3 grid_xy, int S);

template <int KIND, int N, int RT, bool PAIR = false, int NT = kGemmRows>
static cudaError_t launch_gemm_t(const CUtensorMap& pmap, const GemmArgs& a, int items, int S, cudaStream_t stream) {
    if (PAIR && (S != 1 || (a.out / 128) % 2)) return cudaErrorInvalidValue;  // pairs: no split, even blocks
    auto kern = gemm_kernel<KIND, N, NT, RT, false, PAIR>;
    const int smem = GemmLayout<N, NT, RT, PAIR>::ALLOC;
    cudaError_t e = func_attrs((const void*)kern, smem, S > 8);
    if (e != cudaSuccess) return e;
    if (!PAIR && S > 1) S = gemm_coresident_split((const void*)kern, smem, kGemmThreads, dim3(a.out / 128, items), S);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.out / 128, items, S);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = PAIR ? 2 : 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = S;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, pmap, a);
}

#define SX_GEMM_N_LIST(X) \
    X(16) X(18) X(20) X(22) X(24) X(26) X(28) X(30) X(32) X(34) X(36) X(38) X(40) X(42) X(44) X(46) X(48) X(50) X(52) \
    X(54) X(56) X(58) X(60) X(62) X(64) X(66) X(68) X(70) X(72) X(74) X(76) X(78) X(80) X(82) X(84) X(86) X(88) X(90) \
    X(92) X(94) X(96) X(98) X(100) X(102) X(104) X(106) X(108) X(110) X(112) X(114) X(116) X(118) X(120) X(122) X(124) \
    X(126) X(128)

#define SX_GEMM_N_LIST_PAIR1(X) \
    X(24) X(26) X(28) X(30) X(32) X(34) X(36) X(38) X(40) X(42) X(44) X(46) X(48) X(50) X(52) X(54) X(56) X(58) X(60) \
    X(62) X(64)

// Rates with a four-row-tile (RT = 4) kernel: the configs' K1..K4 and PAIR1's common rows; other
// rates run one row tile per CTA.
#define SX_GEMM_N_LIST_RT(X) X(16) X(24) X(32) X(40) X(48) X(64)

template <int KIND>
cudaError_t gemm_dispatch(const CUtensorMap& pmap, const GemmArgs& a, int n, int rt, int items, int S,
                          cudaStream_t stream, bool pair, int nt) {
    const bool narrow = nt == kGemmRowsNarrow;
    if (nt != kGemmRows && (!narrow || rt != 1 || pair)) return cudaErrorInvalidValue;
#define SX_CASE(NN) \
    case NN: return narrow ? launch_gemm_t<KIND, NN, 1, false, kGemmRowsNarrow>(pmap, a, items, S, stream) \
                           : launch_gemm_t<KIND, NN, 1>(pmap, a, items, S, stream);
#define SX_CASE4(NN) \
    case NN: return pair ? launch_gemm_t<KIND, NN, 4, true>(pmap, a, items, S, stream) \
                         : launch_gemm_t<KIND, NN, 4>(pmap, a, items, S, stream);
    if (rt == 4) {
        switch (n) {
            SX_GEMM_N_LIST_RT(SX_CASE4)
            default: return cudaErrorInvalidValue;
        }
    }
    if constexpr (KIND == K_PAIR1) {
        switch (n) {
            SX_GEMM_N_LIST_PAIR1(SX_CASE)
            default: return cudaErrorInvalidValue;
        }
    } else {
        switch (n) {
            SX_GEMM_N_LIST(SX_CASE)
            default: return cudaErrorInvalidValue;
        }
    }
#undef SX_CASE
#undef SX_CASE4
}

}  // namespace sx
