// Per-codebook launch of the MoE pair and down kernels over the admitted rates (included by
// sx_moe_{mcg,mul1,hash,pair1}.cu).
#pragma once

#include "sx_moe_impl.cuh"

namespace sx {

template <typename Kern>
static cudaError_t launch_clustered(Kern kern, dim3 grid, int S, size_t smem, cudaStream_t stream, const MoeArgs& a) {
    const cudaError_t e = func_attrs((const void*)kern, (int)smem, S > 8);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = S;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

// Shared memory that lets two CTAs share an SM (per-SM capacity / 2 less the per-block reserve).
int two_per_sm_smem();
// The same for three CTAs per SM.
int three_per_sm_smem();

// The split-K cluster size of a chain kernel: the smallest S >= S_min whose CTAs fit two per SM.
// S_min asks for enough CTAs to cover the SMs when few experts are active; then (S_min > 1) the
// smallest S >= S_min that fits three per SM is taken if any (the chain kernels' registers allow
// three).  The kernels are compiled for three CTAs per SM (72 registers) either way.  Measured on
// B200 against two per SM everywhere at 94 registers: the 2048/512 layer 3.5% / 2% / 3% faster
// at 1 / 8 / 64 tokens, the 16-layer 7168/2048 stack within 1% at 1 token, 6% faster at 8 and 1%
// at 64; taking three per SM also where S_min = 1 was no faster there and 3% slower on the stack
// at 64 tokens.  More splits than needed pay the cluster reduce and per-CTA start-up more often.
// Static shared memory of the chain kernels (slot ids, the pair finish's weights), counted against
// the per-SM budget next to the dynamic carve-up.
constexpr size_t kChainStaticSmem = 2048;

template <int N, int NP>
static int fit_split(int S, int KB, int mg) {
    S = S < KB ? S : KB;
    const size_t three = (size_t)three_per_sm_smem() - kChainStaticSmem, two = (size_t)two_per_sm_smem() - kChainStaticSmem;
    if (S > 1)
        for (int c = S; c <= 16 && c <= KB; c++)
            if (core_layout<N, NP, 1>((KB + c - 1) / c, mg).total <= three) return c;
    while (S < 16 && S < KB && core_layout<N, NP, 1>((KB + S - 1) / S, mg).total > two) S++;
    return S;
}

template <int KIND, int N>
static cudaError_t launch_pair_t(const MoeArgs& a, int S, int W_max, cudaStream_t stream) {
    const int KB = a.D / 128;
    S = fit_split<N, 2>(S, KB, a.split_chunk ? a.split_chunk : a.chunk);
    const CoreLayout L = core_layout<N, 2, 1>((KB + S - 1) / S, a.chunk);
    return launch_clustered(moe_pair_kernel<KIND, N>, dim3(W_max, a.I / 128, S), S, L.total, stream, a);
}

template <int KIND, int N>
static cudaError_t launch_down_t(const MoeArgs& a, int S, int W_max, cudaStream_t stream) {
    const int KB = a.I / 128;
    S = fit_split<N, 1>(S, KB, a.split_chunk ? a.split_chunk : a.chunk);
    const CoreLayout L = core_layout<N, 1, 1>((KB + S - 1) / S, a.chunk);
    return launch_clustered(moe_down_kernel<KIND, N>, dim3(W_max, a.D / 128, S), S, L.total, stream, a);
}

// The one-token down + reduce (moe_down1): grid (D/128, W) in clusters of the W items.
template <int KIND, int N>
static cudaError_t launch_down1_t(const MoeArgs& a, int W, cudaStream_t stream) {
    const CoreLayout L = core_layout<N, 1, 1>(a.I / 128, 1);
    auto kern = moe_down1_kernel<KIND, N>;
    const cudaError_t e = func_attrs((const void*)kern, (int)L.total, W > 8);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.D / 128, W, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = W;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

#define SX_MOE_N_LIST(X) \
    X(16) X(18) X(20) X(22) X(24) X(26) X(28) X(30) X(32) X(34) X(36) X(38) X(40) X(42) X(44) X(46) X(48) X(50) X(52) \
    X(54) X(56) X(58) X(60) X(62) X(64) X(66) X(68) X(70) X(72) X(74) X(76) X(78) X(80) X(82) X(84) X(86) X(88) X(90) \
    X(92) X(94) X(96) X(98) X(100) X(102) X(104) X(106) X(108) X(110) X(112) X(114) X(116) X(118) X(120) X(122) X(124) \
    X(126) X(128)

#define SX_MOE_N_LIST_PAIR1(X) \
    X(24) X(26) X(28) X(30) X(32) X(34) X(36) X(38) X(40) X(42) X(44) X(46) X(48) X(50) X(52) X(54) X(56) X(58) X(60) \
    X(62) X(64)

template <int KIND>
cudaError_t moe_launch_kind(const MoeArgs& a, int n_gu, int n_d, int S_gu, int S_d, int W_max, cudaStream_t stream) {
    cudaError_t e = cudaErrorInvalidValue;
#define SX_PAIR_CASE(NN) \
    case NN: e = launch_pair_t<KIND, NN>(a, S_gu, W_max, stream); break;
#define SX_DOWN_CASE(NN) \
    case NN: e = launch_down_t<KIND, NN>(a, S_d, W_max, stream); break;
    if constexpr (KIND == K_PAIR1) {
        switch (n_gu) { SX_MOE_N_LIST_PAIR1(SX_PAIR_CASE) default: return cudaErrorInvalidValue; }
        if (e != cudaSuccess) return e;
        switch (n_d) { SX_MOE_N_LIST_PAIR1(SX_DOWN_CASE) default: return cudaErrorInvalidValue; }
    } else {
        switch (n_gu) { SX_MOE_N_LIST(SX_PAIR_CASE) default: return cudaErrorInvalidValue; }
        if (e != cudaSuccess) return e;
        switch (n_d) { SX_MOE_N_LIST(SX_DOWN_CASE) default: return cudaErrorInvalidValue; }
    }
#undef SX_PAIR_CASE
#undef SX_DOWN_CASE
    return e;
}

// The one-token chain: moe_pair over the W direct items, then moe_down1.
template <int KIND>
cudaError_t moe_launch_kind_direct(const MoeArgs& a, int n_gu, int n_d, int S_gu, int W, cudaStream_t stream) {
    cudaError_t e = cudaErrorInvalidValue;
#define SX_PAIR_CASE(NN) \
    case NN: e = launch_pair_t<KIND, NN>(a, S_gu, W, stream); break;
#define SX_DOWN1_CASE(NN) \
    case NN: e = launch_down1_t<KIND, NN>(a, W, stream); break;
    if constexpr (KIND == K_PAIR1) {
        switch (n_gu) { SX_MOE_N_LIST_PAIR1(SX_PAIR_CASE) default: return cudaErrorInvalidValue; }
        if (e != cudaSuccess) return e;
        switch (n_d) { SX_MOE_N_LIST_PAIR1(SX_DOWN1_CASE) default: return cudaErrorInvalidValue; }
    } else {
        switch (n_gu) { SX_MOE_N_LIST(SX_PAIR_CASE) default: return cudaErrorInvalidValue; }
        if (e != cudaSuccess) return e;
        switch (n_d) { SX_MOE_N_LIST(SX_DOWN1_CASE) default: return cudaErrorInvalidValue; }
    }
#undef SX_PAIR_CASE
#undef SX_DOWN1_CASE
    return e;
}

}  // namespace sx
