// Fused EXL3 projection for 1..16 rows: y = svh * H128( W_inner . H128(suh * x) )
// (kernel template; instantiated per codebook in sx_gemv_{mcg,mul1,hash,pair1}.cu).
//
// One launch does the reference's three host stages (src/exl3/expert_exl3.zig:490-544,
// prepareInput -> innerGemv -> finishOutput; on the GPU, project_rows.zig:759's rows kernel plus
// its finish dispatch):
//   * A CTA owns one 128-wide output block and a contiguous range of input blocks (sx_core.cuh);
//     the CTAs that split one output block's k range form a thread-block cluster (<= 16 CTAs).
//   * While the producer warp fills the tile ring, the consumer warps prepare the CTA's input
//     slice (f16(x) * suh, Hadamard-128 by warp butterflies, rounded to f16 as prepareInput does)
//     straight into MMA B-fragment order.
//   * The cluster's rank-0 CTA sums its peers' partials over distributed shared memory (DSMEM),
//     applies Hadamard-128, svh and the codebook scale, and writes y once in the input's dtype.
//     No global scratch.
#pragma once

#include <algorithm>

#include "sx_core.cuh"
#include "sx_kernels.h"

namespace sx {

template <int KIND, int NB, bool W16>
cudaError_t dispatch_n(const GemvArgs& a, int n, int groups, cudaStream_t stream);

// Consumer warps of the GEMV: 8, each owning one output tile across a stage's 8 input-tile rows,
// compiled for three CTAs per SM up to 8 rows (measured on B200: faster than 16 warps at two CTAs
// per SM on every sweep shape, and no slower than the same kernel given two CTAs' registers).
constexpr int kGemvCW = 8;
constexpr int kGemvThreads = (kGemvCW + 1) * 32;

// The RMS norm of the first linear of a stacked launch (project_rows.zig:394-456's finish, MLX's
// rms_norm on the finished row): called by every thread of each rank-0 CTA of linear 0 once its
// rows and sums of squares are written and fenced.  The block that counts itself last reads the
// whole segment's sums (fixed order), and rewrites the segment's rows as
// w[c] * T(o[c] * rsqrt(sum / cols + eps)).  No block waits on another.
// `flag` is a word of the CTA's shared memory that nothing reads any more.
__device__ __forceinline__ void gemv_norm_last(const GemvArgs& a, int lane, int warp, int* flag) {
    const int blocks = a.seg_end[0];
    if (threadIdx.x == 0) *flag = atomicAdd(a.norm_count, 1u) == (unsigned)(blocks - 1);
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    const int cols = blocks * 128;
    const int nw = blockDim.x >> 5;
    for (int m = warp; m < a.rows; m += nw) {
        float ss = 0.0f;
        for (int b = lane; b < blocks; b += 32) ss += __ldcg(a.norm_ssq + m * blocks + b);
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
        const float inv = __frsqrt_rn(ss / (float)cols + a.norm_eps);
        void* yr = static_cast<uint8_t*>(a.ys[0]) + (size_t)m * cols * (a.xdt == 0 ? 4 : 2);
        for (int c = lane; c < cols; c += 32) {
            const float t = round_act(load_act_cg(yr, c, a.xdt) * inv, a.xdt);
            store_act(yr, c, a.xdt, load_act(a.norm_w, c, a.xdt) * t);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *a.norm_count = 0u;  // ready for the next launch on the stream
}

template <int KIND, int N, int NB, bool W16>
__global__ void __launch_bounds__(kGemvThreads, NB == 1 ? 3 : 2) gemv_kernel(GemvArgs a) {
    constexpr int CW = kGemvCW;
    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int ob = blockIdx.x;     // output block (128 outputs)
    const int split = blockIdx.y;  // k-split index == cluster rank
    const int g = blockIdx.z;      // bank (grouped linears)
    const int S = gridDim.y;
    const int KB = a.in / 128;
    const int kb0 = (int)(((long long)split * KB) / S);
    const int kbl = (int)(((long long)(split + 1) * KB) / S) - kb0;
    const int kbl_max = (KB + S - 1) / S;
    const int mg = a.rows < 8 ? a.rows : 8;
    const CoreSmem s = core_smem<N, 1, NB>(smem, kbl_max, mg);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int OT = a.out / 16;
    int seg = 0;  // the stacked linear this output block belongs to
    while (seg + 1 < a.nseg && ob >= a.seg_end[seg]) seg++;
    const uint16_t* suh = a.suh + (size_t)(g + seg) * a.in;
    const uint16_t* svh = a.svh + (size_t)g * a.out;

    core_init_barriers<N, 1, CW>(s);
    __syncthreads();
    grid_launch_dependents();

    uint16_t svh0[4] = {0, 0, 0, 0};  // the finish's svh values of this lane (rank 0)
    if (warp == CW) {
        // The weights are read-only to the grids around this one, so they stream before the
        // dependency wait (launches with programmatic serialisation only).
        if (lane == 0) {
            const uint16_t* const tr[1] = {a.trellis + (size_t)g * ((size_t)KB * 8 * OT * N)};
            core_produce<N, 1>(s, tr, OT, ob, kb0, kbl);
        }
    } else {
        // Prepare (prepareInput): warp w takes the CTA's input blocks w, w + CW, ...; per block and
        // 8-row group the lane's four x values of every stored row are loaded together (one round
        // of loads per block and group, not one per row), then each row is prepared: f16(x) *
        // suh, Hadamard-128, f16, into its B fragments.  suh and svh are weights: the first
        // block's suh and, in rank 0, the lane's four svh values of the finish are read before the
        // dependency wait.
        const bool vec = a.vec != 0;
        float su[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (warp < kbl) load_half4(suh, (size_t)(kb0 + warp) * 128 + lane * 4, vec, su);
        if (split == 0) {
#pragma unroll
            for (int i = 0; i < 4; i++) svh0[i] = svh[ob * 128 + lane * 4 + i];
        }
        grid_dependency_wait();  // x may come from the previous grid
        for (int kbi = warp; kbi < kbl; kbi += CW) {
            const int base = (kb0 + kbi) * 128 + lane * 4;
            if (kbi != warp) load_half4(suh, base, vec, su);
#pragma unroll
            for (int nb = 0; nb < NB; nb++) {
                float v[8][4];
#pragma unroll
                for (int gg = 0; gg < 8; gg++) {
                    const int m = nb * 8 + gg;
                    if (gg < mg && m < a.rows)
                        load_act4v(a.x, (size_t)g * a.x_group_stride + (size_t)m * a.in + base, a.xdt, vec, v[gg]);
                }
#pragma unroll
                for (int gg = 0; gg < 8; gg++) {
                    const int m = nb * 8 + gg;
                    if (gg >= mg) continue;  // rows of later lanes read row mg-1's fragments
                    float (&vr)[4] = v[gg];
                    if (m < a.rows) {
#pragma unroll
                        for (int i = 0; i < 4; i++) vr[i] = round_f16(vr[i]) * su[i];
                        warp_hadamard128(vr);
                    } else {
                        vr[0] = vr[1] = vr[2] = vr[3] = 0.0f;
                    }
                    const uint16_t h[4] = {f2h(vr[0]), f2h(vr[1]), f2h(vr[2]), f2h(vr[3])};
                    bfrag_put4<NB>(s.bfrag, mg, kbi, m, lane, h);
                }
            }
        }
        consumers_sync<CW>();

        const DecParams dp[1] = {{a.wmask, a.mult, a.mask0, a.mask1, a.rot}};
        float acc[1][NB][4];
        core_consume<KIND, N, 1, NB, W16, CW>(s, kbl, dp, acc);
        core_reduce<1, NB, CW>(s.red, acc);
    }

    // rank 0 sums the cluster's partials over DSMEM and finishes
    const bool normed = a.norm_w != nullptr && seg == 0;
    cluster.sync();
    if (split == 0 && warp < CW) {
        for (int m = warp; m < a.rows; m += CW) {
            const float4 t = cluster_sum4(cluster, s.red, S, m * 128);
            float v[4] = {t.x, t.y, t.z, t.w};
            warp_hadamard128(v);
            void* yp = a.y;
            size_t yoff = (size_t)g * a.y_group_stride + (size_t)m * a.out + (size_t)ob * 128 + lane * 4;
            if (a.nseg > 0) {
                const int first = seg ? a.seg_end[seg - 1] : 0;
                yp = a.ys[seg];
                yoff = (size_t)m * a.ywidth[seg] + (size_t)(ob - first) * 128 + lane * 4;
            }
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float f = v[i] * a.out_scale * h2f(svh0[i]);
                if (normed) {
                    const float r = round_act(f, a.xdt);
                    ss = fmaf(r, r, ss);
                }
                store_act(yp, yoff + i, a.xdt, f);
            }
            if (normed) {
#pragma unroll
                for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
                if (lane == 0) a.norm_ssq[m * a.seg_end[0] + ob] = ss;
            }
        }
        if (normed) __threadfence();  // this block's rows and sums before its count below
    }
    cluster.sync();
    // After that sync no peer reads this CTA's shared memory: its first word serves as a flag.
    if (normed && split == 0) gemv_norm_last(a, lane, warp, reinterpret_cast<int*>(smem));
}

// The split-K cluster size for a launch: the largest S <= 16 (and <= the input blocks) whose
// clusters are all co-resident in one wave, so no cluster waits for another to drain; S = 1 when
// even unsplit output blocks exceed a wave.  Cached per kernel and geometry.
struct SplitKey {
    const void* kern;
    int out, in, groups, mg;
    bool operator==(const SplitKey& o) const {
        return kern == o.kern && out == o.out && in == o.in && groups == o.groups && mg == o.mg;
    }
};

int cached_split(const SplitKey& k);
void remember_split(const SplitKey& k, int S);
int sm_count();

// Dynamic shared memory that holds the GEMV to two CTAs per SM.
constexpr int kGemvTwoPerSmSmem = 80 * 1024;

template <int KIND, int N, int NB, bool W16>
static cudaError_t launch_gemv_t(const GemvArgs& a, int groups, cudaStream_t stream) {
    const int KB = a.in / 128;
    const int OB = a.out / 128;
    const int mg = a.rows < 8 ? a.rows : 8;
    auto kern = gemv_kernel<KIND, N, NB, W16>;
    const SplitKey key{(const void*)kern, a.out, a.in, groups, mg};
    int S = cached_split(key);  // split | (two-per-SM floor << 8)
    cudaError_t e;
    if (S <= 0) {
        // The split and occupancy: among co-resident splits (no cluster waits for another to
        // drain), at the kernel's natural occupancy and with a shared-memory floor of two CTAs per
        // SM, the least estimated time of the busiest SM: its CTAs times each CTA's input blocks.
        // Clusters pack within GPCs, so past one CTA per SM the busiest SM is taken to hold one
        // CTA more than the even share, up to the occupancy; an SM decodes at about the same rate
        // with two or three CTAs and at ~0.55 of it with one (measured on B200); of equal estimates
        // the one with fewer CTAs (fewer partial sums to gather, less per-CTA set-up).  Without any
        // co-resident split: the largest one (the most CTAs, the least shared memory per CTA),
        // which then runs in several waves.  The kernel's attributes only ever grow (func_attrs),
        // so a launch of another geometry never meets a shared-memory limit this search lowered.
        const int s_max = KB < 16 ? KB : 16;
        const long long sms = sm_count();
        long long best_cost = -1, best_ctas = 0;
        int best = s_max;
        for (int floor2 = 0; floor2 < 2; floor2++) {
            for (int cand = s_max; cand >= 1; cand--) {
                const CoreLayout L = core_layout<N, 1, NB>((KB + cand - 1) / cand, mg);
                if (L.total > 200 * 1024) break;  // smaller splits only need more
                const int natural = (int)L.total;
                const int smem = floor2 && natural < kGemvTwoPerSmSmem ? kGemvTwoPerSmSmem : natural;
                e = func_attrs((const void*)kern, smem, true);
                if (e != cudaSuccess) return e;
                int occ = 0;
                if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kGemvThreads, smem) != cudaSuccess ||
                    occ < 1) {
                    cudaGetLastError();
                    continue;
                }
                if (floor2 && natural >= kGemvTwoPerSmSmem) continue;  // the same launch as without the floor
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3(OB, cand, groups);
                cfg.blockDim = dim3(kGemvThreads, 1, 1);
                cfg.dynamicSmemBytes = smem;
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeClusterDimension;
                attr[0].val.clusterDim.x = 1;
                attr[0].val.clusterDim.y = cand;
                attr[0].val.clusterDim.z = 1;
                cfg.attrs = attr;
                cfg.numAttrs = 1;
                int clusters = 0;
                if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < OB * groups) {
                    cudaGetLastError();
                    continue;
                }
                const long long ctas = (long long)OB * cand * groups;
                const long long even = (ctas + sms - 1) / sms;
                const long long busiest = ctas <= sms ? 1 : std::min<long long>(occ, even + 1);
                const long long blocks = (KB + cand - 1) / cand;
                const long long cost = busiest == 1 ? blocks * 36 : busiest * blocks * 20;
                if (best_cost < 0 || cost < best_cost || (cost == best_cost && ctas < best_ctas)) {
                    best_cost = cost;
                    best_ctas = ctas;
                    best = cand | (floor2 << 8);
                }
            }
        }
        S = best;
        remember_split(key, S);
    }
    const bool floor2 = (S >> 8) != 0;
    S &= 0xFF;
    const CoreLayout L = core_layout<N, 1, NB>((KB + S - 1) / S, mg);
    const int smem = floor2 && (int)L.total < kGemvTwoPerSmSmem ? kGemvTwoPerSmSmem : (int)L.total;
    e = func_attrs((const void*)kern, smem, S > 8);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(OB, S, groups);
    cfg.blockDim = dim3(kGemvThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = S;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

#define SX_N_LIST(X) \
    X(16) X(18) X(20) X(22) X(24) X(26) X(28) X(30) X(32) X(34) X(36) X(38) X(40) X(42) X(44) X(46) X(48) X(50) X(52) \
    X(54) X(56) X(58) X(60) X(62) X(64) X(66) X(68) X(70) X(72) X(74) X(76) X(78) X(80) X(82) X(84) X(86) X(88) X(90) \
    X(92) X(94) X(96) X(98) X(100) X(102) X(104) X(106) X(108) X(110) X(112) X(114) X(116) X(118) X(120) X(122) X(124) \
    X(126) X(128)

#define SX_N_LIST_PAIR1(X) \
    X(24) X(26) X(28) X(30) X(32) X(34) X(36) X(38) X(40) X(42) X(44) X(46) X(48) X(50) X(52) X(54) X(56) X(58) X(60) \
    X(62) X(64)

// PAIR1 has rows at n = 24..64 only (src/exl3/expert_exl3.zig:49-52); the others span 16..128.
template <int KIND, int NB, bool W16>
cudaError_t dispatch_n(const GemvArgs& a, int n, int groups, cudaStream_t stream) {
#define SX_CASE(NN) \
    case NN: return launch_gemv_t<KIND, NN, NB, W16>(a, groups, stream);
    if constexpr (KIND == K_PAIR1) {
        switch (n) {
            SX_N_LIST_PAIR1(SX_CASE)
            default: return cudaErrorInvalidValue;
        }
    } else {
        switch (n) {
            SX_N_LIST(SX_CASE)
            default: return cudaErrorInvalidValue;
        }
    }
#undef SX_CASE
}

}  // namespace sx
