// Fused MoE router: moeRouterTopK (src/moe_router.zig:442, kernel text :112-290).
//
// One CTA per row.  Phase 1 writes every expert's selection key (softmax: the logit; sigmoid
// modes: sigmoid(logit) + bias, with the raw sigmoid kept as the weight) to shared memory.  The
// grouped mode scores each of n_group equal groups by the sum of its two best keys and pushes the
// experts of every group outside the best topk_group to -1e4 (the composed chain's finite
// penalty).  Warp 0 then runs k rounds of "max, then mask" whose ties go to the LOWEST expert id,
// so the pick is a pure function of the keys, and normalises the picked weights: softmax
// probabilities renormalised over the picks; sigmoid scores divided by their sum (+1e-20) when
// `renorm` and k > 1, times `scale`.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "../../include/sushi_exl3.h"
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

constexpr int kRouterMaxExperts = 2048;
constexpr int kRouterThreads = 256;

__device__ __forceinline__ void warp_argmax_lowest(float& v, int& idx) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, m);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, m);
        if (ov > v || (ov == v && oi < idx)) {
            v = ov;
            idx = oi;
        }
    }
}

__global__ void __launch_bounds__(kRouterThreads) router_kernel(const float* __restrict__ logits,
                                                                const float* __restrict__ bias, int E, int K, int mode,
                                                                int renorm, float scale, int n_group, int topk_group,
                                                                uint32_t* __restrict__ inds, float* __restrict__ scores) {
    extern __shared__ float sm[];
    float* key = sm;        // [E]
    float* wraw = sm + E;   // [E] (sigmoid modes)
    __shared__ float red_max[kRouterThreads / 32], red_sum[kRouterThreads / 32];
    __shared__ int sel[32];
    __shared__ float gscore[32];
    const int row = blockIdx.x;
    const float* lg = logits + (size_t)row * E;
    const bool sigmoid = mode != SX_ROUTER_SOFTMAX;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    float lmax = -CUDART_INF_F;
    for (int e = tid; e < E; e += blockDim.x) {
        const float l = lg[e];
        if (sigmoid) {
            // The two-sided form of MLX's Sigmoid the reference mirrors (src/moe_router.zig:214-219).
            const float sy = 1.0f / (1.0f + expf(fabsf(l)));
            const float sg = l < 0.0f ? sy : 1.0f - sy;
            key[e] = sg + bias[e];
            wraw[e] = sg;
        } else {
            key[e] = l;
            lmax = fmaxf(lmax, l);
        }
    }
    float snorm = 0.0f, smax = 0.0f;
    if (!sigmoid) {
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, m));
        if (lane == 0) red_max[warp] = lmax;
        __syncthreads();
        smax = red_max[0];
        for (int w = 1; w < (int)(blockDim.x / 32); w++) smax = fmaxf(smax, red_max[w]);
        float acc = 0.0f;
        for (int e = tid; e < E; e += blockDim.x) acc += expf(key[e] - smax);
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
        if (lane == 0) red_sum[warp] = acc;
    }
    __syncthreads();
    if (!sigmoid) {
        float tot = 0.0f;
        for (int w = 0; w < (int)(blockDim.x / 32); w++) tot += red_sum[w];
        snorm = 1.0f / tot;
    }
    if (warp != 0) return;

    if (mode == SX_ROUTER_SIGMOID_BIAS_GROUPED) {
        const int gsz = E / n_group;
        for (int g = lane; g < n_group; g += 32) {
            float m1 = -CUDART_INF_F, m2 = -CUDART_INF_F;
            for (int j = 0; j < gsz; j++) {
                const float v = key[g * gsz + j];
                if (v > m1) {
                    m2 = m1;
                    m1 = v;
                } else if (v > m2) {
                    m2 = v;
                }
            }
            gscore[g] = m1 + m2;
        }
        __syncwarp();
        uint32_t keep = 0;
        for (int r = 0; r < topk_group; r++) {
            float v = lane < n_group ? gscore[lane] : -CUDART_INF_F;
            int idx = lane < n_group ? lane : 0x7fffffff;
            warp_argmax_lowest(v, idx);
            keep |= 1u << idx;
            if (lane == 0) gscore[idx] = -CUDART_INF_F;
            __syncwarp();
        }
        for (int e = lane; e < E; e += 32)
            if (!((keep >> (e / gsz)) & 1u)) key[e] = -1.0e4f;
        __syncwarp();
    }

    for (int r = 0; r < K; r++) {
        float best = -CUDART_INF_F;
        int bidx = 0x7fffffff;
        for (int e = lane; e < E; e += 32) {
            const float v = key[e];
            if (v > best) {
                best = v;
                bidx = e;
            }
        }
        warp_argmax_lowest(best, bidx);
        if (bidx >= E) bidx = E - 1;
        if (lane == 0) {
            sel[r] = bidx;
            key[bidx] = -CUDART_INF_F;
        }
        __syncwarp();
    }

    float w = 0.0f;
    int myidx = 0;
    if (lane < K) {
        myidx = sel[lane];
        w = sigmoid ? wraw[myidx] : expf(lg[myidx] - smax) * snorm;
    }
    float tot = 0.0f;
    for (int j = 0; j < K; j++) tot += __shfl_sync(0xffffffffu, w, j);
    if (sigmoid) {
        if (renorm && K > 1) w = w / (tot + 1e-20f);
        w = w * scale;
    } else {
        w = w / tot;
    }
    if (lane < K) {
        inds[(size_t)row * K + lane] = (uint32_t)myidx;
        scores[(size_t)row * K + lane] = w;
    }
}

}  // namespace sx

using namespace sx;

extern "C" sx_status sx_router_topk(sx_stream stream, const float* logits, const float* bias, int32_t rows,
                                    int32_t experts, int32_t k, int32_t mode, int32_t renorm, float scale,
                                    int32_t n_group, int32_t topk_group, uint32_t* inds, float* scores) {
    if (!logits || !inds || !scores) return SX_ERR_NULL_POINTER;
    if (rows < 1) return SX_ERR_BAD_SHAPE;
    if (mode < SX_ROUTER_SOFTMAX || mode > SX_ROUTER_SIGMOID_BIAS_GROUPED) return SX_ERR_ROUTER_DECLINED;
    // The reference kernel's admission (src/moe_router.zig:466-490): it declines, the caller keeps its chain.
    if (experts < k || experts > kRouterMaxExperts || k < 1 || k > 32) return SX_ERR_ROUTER_DECLINED;
    if (mode != SX_ROUTER_SOFTMAX && !bias) return SX_ERR_ROUTER_DECLINED;
    if (mode == SX_ROUTER_SIGMOID_BIAS_GROUPED) {
        if (n_group <= 1 || n_group > 32 || topk_group <= 0 || topk_group > n_group || experts % n_group != 0 ||
            experts / n_group < 2)
            return SX_ERR_ROUTER_DECLINED;
    }
    const size_t smem = (size_t)2 * experts * sizeof(float);
    router_kernel<<<rows, kRouterThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
        logits, bias, experts, k, mode, renorm, scale, n_group, topk_group, inds, scores);
    return cuda_status(cudaGetLastError(), "router launch");
}
