// Bit-exact dequantisation: the inner f16 matrix of one bank, as the reference's host
// `reconstructInner` writes it (src/exl3/expert_exl3.zig:416-438).  One warp per 16x16 tile; lane L
// decodes stream positions 8L..8L+7 through the same funnel the GEMV uses, with the reference's
// per-codeword f16 arithmetic (sx_decode.cuh exact_decode), and stores each weight at its
// tensorCorePerm place.  Used by the bit-exact parity tests and by callers that want the dense
// inner matrix (the reference's trunk_gemm decode-once arm, src/exl3/trunk_gemm.zig).
#include "sx_decode.cuh"
#include "sx_internal.h"
#include "sx_kernels.h"

namespace sx {

__device__ int g_device_error = 0;

__constant__ uint32_t c_pow2_16[17] = {65536u, 32768u, 16384u, 8192u, 4096u, 2048u, 1024u, 512u, 256u,
                                       128u,   64u,    32u,    16u,   8u,    4u,    2u,    1u};

template <int KIND, int N>
__global__ void __launch_bounds__(256) dequant_kernel(DequantArgs a) {
    const int OT = a.out_f / 16;
    const int IT = a.in_f / 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long tile = (long long)blockIdx.x * 8 + warp;
    if (tile >= (long long)IT * OT) return;
    const int tk = (int)(tile / OT), tn = (int)(tile % OT);
    const uint32_t* words = reinterpret_cast<const uint32_t*>(a.trellis + (size_t)tile * N);
    LaneFunnel<N> lf;
    lf.init(lane);
    uint32_t r[Funnel<N>::NR];
    lane_stream<N>(words, lf, r);
    uint32_t cw[8];
    cw[0] = codeword<N, 0, false>(r, a.wmask);
    cw[1] = codeword<N, 1, false>(r, a.wmask);
    cw[2] = codeword<N, 2, false>(r, a.wmask);
    cw[3] = codeword<N, 3, false>(r, a.wmask);
    cw[4] = codeword<N, 4, false>(r, a.wmask);
    cw[5] = codeword<N, 5, false>(r, a.wmask);
    cw[6] = codeword<N, 6, false>(r, a.wmask);
    cw[7] = codeword<N, 7, false>(r, a.wmask);
    const DecParams dp{a.wmask, a.mult, a.mask0, a.mask1, a.rot};
    const int gq = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int v = 0; v < 8; v++) {
        uint16_t w;
        exact_decode<KIND>(cw[v], cw[v | 1], dp, v & 1, w);
        const int rowsel = v & 3;
        const int i = 2 * cq + (rowsel & 1) + ((rowsel >> 1) << 3);
        const int o = gq + ((v >> 2) << 3);
        a.dst[((size_t)tk * 16 + i) * a.out_f + (size_t)tn * 16 + o] = w;
    }
}

template <int KIND>
__global__ void codewords_kernel(uint32_t* out32, DecParams dp) {
    const uint32_t cw = blockIdx.x * blockDim.x + threadIdx.x;
    if (cw >= 65536u) return;
    const uint32_t m = cw & dp.wmask;
    uint16_t w0, w1 = 0;
    if constexpr (KIND == K_PAIR1) {
        exact_decode<KIND>(m, m, dp, 0, w0);
        exact_decode<KIND>(m, m, dp, 1, w1);
    } else {
        exact_decode<KIND>(m, m, dp, 0, w0);
    }
    out32[cw] = (uint32_t)w0 | ((uint32_t)w1 << 16);
}

#define SX_DQ_N_LIST(X) \
    X(16) X(18) X(20) X(22) X(24) X(26) X(28) X(30) X(32) X(34) X(36) X(38) X(40) X(42) X(44) X(46) X(48) X(50) X(52) \
    X(54) X(56) X(58) X(60) X(62) X(64) X(66) X(68) X(70) X(72) X(74) X(76) X(78) X(80) X(82) X(84) X(86) X(88) X(90) \
    X(92) X(94) X(96) X(98) X(100) X(102) X(104) X(106) X(108) X(110) X(112) X(114) X(116) X(118) X(120) X(122) X(124) \
    X(126) X(128)

template <int KIND>
static cudaError_t dequant_n(const DequantArgs& a, cudaStream_t stream) {
    const long long tiles = (long long)(a.in_f / 16) * (a.out_f / 16);
    const dim3 grid((unsigned)((tiles + 7) / 8));
    switch (a.n) {
#define SX_CASE(NN)                                                  \
    case NN:                                                         \
        dequant_kernel<KIND, NN><<<grid, 256, 0, stream>>>(a);       \
        return cudaGetLastError();
        SX_DQ_N_LIST(SX_CASE)
#undef SX_CASE
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_dequant(const DequantArgs& a, int kind, cudaStream_t stream) {
    switch (kind) {
        case K_MUL1: return dequant_n<K_MUL1>(a, stream);
        case K_MCG: return dequant_n<K_MCG>(a, stream);
        case K_HASH: return dequant_n<K_HASH>(a, stream);
        case K_PAIR1: return dequant_n<K_PAIR1>(a, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_decode_codewords(int kind, int n, uint32_t wmask, uint32_t mult, uint32_t mask0, uint32_t mask1,
                                    uint32_t rot, uint32_t* out32, cudaStream_t stream) {
    (void)n;
    const DecParams dp{wmask, mult, mask0, mask1, rot};
    switch (kind) {
        case K_MUL1: codewords_kernel<K_MUL1><<<256, 256, 0, stream>>>(out32, dp); break;
        case K_MCG: codewords_kernel<K_MCG><<<256, 256, 0, stream>>>(out32, dp); break;
        case K_HASH: codewords_kernel<K_HASH><<<256, 256, 0, stream>>>(out32, dp); break;
        case K_PAIR1: codewords_kernel<K_PAIR1><<<256, 256, 0, stream>>>(out32, dp); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace sx

namespace sx {
namespace {

// A wait nothing will satisfy: one thread waits on a fresh mbarrier (expected arrivals 1, none
// made) through the same bounded wait every kernel uses, gives up after limit_ns and latches
// DEV_TIMEOUT_SELFTEST.
__global__ void wait_selftest_kernel(uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_wait(&bar, 0, DEV_TIMEOUT_SELFTEST, limit_ns);
    }
}

}  // namespace
}  // namespace sx

extern "C" sx_status sx_selftest_wait_timeout(sx_stream stream, int32_t limit_ms) {
    if (limit_ms < 1 || limit_ms > 2000) return SX_ERR_BAD_SHAPE;
    sx::wait_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>((uint64_t)limit_ms * 1000000ull);
    return sx::cuda_status(cudaGetLastError(), "selftest launch");
}
