// Fused MoE router: moeRouterTopK / moeRouterTopKGate (src/moe_router.zig:442, :457; kernel text
// :112-336).
//
// One CTA per row.  Phase 1 writes every expert's selection key (softmax: the logit; sigmoid
// modes: sigmoid(logit) + bias, with the raw sigmoid kept as the weight) to shared memory.  The
// grouped mode scores each of n_group equal groups by the sum of its two best keys and pushes the
// experts of every group outside the best topk_group to -1e4 (the composed chain's finite
// penalty).  Warp 0 then runs k rounds of "max, then mask" whose ties go to the LOWEST expert id,
// so the pick is a pure function of the keys, and normalises the picked weights: softmax
// probabilities renormalised over the picks; sigmoid scores divided by their sum (+1e-20) when
// `renorm` and k > 1, times `scale`.  Logits are F32, F16 or BF16.  The softmax_gate mode adds the
// shared-expert gate's logit, the dot of the row's x with a flat weight vector: warps 1..7 compute
// it while warp 0 selects.
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

// The shared-expert gate's logit (moeRouterTopKGate's `gate`): x . w over gk elements (x and w of
// dtype dt, F16 or BF16) in the order of MLX's dot_product as the reference kernel restates it
// (src/moe_router.zig:200-218, :328-332): virtual group vs owns elements [1024 vs, 1024 vs + 1024);
// lane l accumulates a float4 c over its four 8-element chunks at 1024 vs + 8 l + 256 i (chunks that
// run past gk are skipped), c[q] += x * w element by element; then c0 + c1 + c2 + c3, a warp sum,
// and a sum of the groups' partials over 16 lanes (zeros past the last group).  Products and sums
// are rounded separately (no fused multiply-add).  Called by warps 1..7 (warp w takes groups
// w-1, w+6, ...); partials land in gp[16].
__device__ __forceinline__ void router_gate_partials(const void* gx, const void* gw, int gk, int dt, float* gp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int groups = (gk + 1023) / 1024;
    // The four chunks' x and w are loaded before any product (16-byte loads when both vectors
    // start 16-byte aligned: a chunk is 8 elements at a multiple of 8), one round of loads.
    const bool vec = ((reinterpret_cast<uintptr_t>(gx) | reinterpret_cast<uintptr_t>(gw)) & 15) == 0;
    for (int vs = warp - 1; vs < groups; vs += kRouterThreads / 32 - 1) {
        float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        float xv[4][8], wv[4][8];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int idx = vs * 1024 + lane * 8 + q * 256;
            if (idx + 8 <= gk) {
                if (vec) {
                    const uint4 ux = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(gx) + idx);
                    const uint4 uw = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(gw) + idx);
                    const uint32_t px[4] = {ux.x, ux.y, ux.z, ux.w}, pw[4] = {uw.x, uw.y, uw.z, uw.w};
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const uint16_t hx = (uint16_t)(px[j >> 1] >> (16 * (j & 1)));
                        const uint16_t hw = (uint16_t)(pw[j >> 1] >> (16 * (j & 1)));
                        xv[q][j] = dt == 1 ? __half2float(__ushort_as_half(hx)) : __bfloat162float(__ushort_as_bfloat16(hx));
                        wv[q][j] = dt == 1 ? __half2float(__ushort_as_half(hw)) : __bfloat162float(__ushort_as_bfloat16(hw));
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        xv[q][j] = load_act(gx, idx + j, dt);
                        wv[q][j] = load_act(gw, idx + j, dt);
                    }
                }
            }
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int idx = vs * 1024 + lane * 8 + q * 256;
            if (idx + 8 <= gk) {
#pragma unroll
                for (int j = 0; j < 8; j++) c[j & 3] = __fadd_rn(c[j & 3], __fmul_rn(xv[q][j], wv[q][j]));
            }
        }
        float ga = __fadd_rn(__fadd_rn(__fadd_rn(c[0], c[1]), c[2]), c[3]);
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) ga = __fadd_rn(ga, __shfl_xor_sync(0xffffffffu, ga, m));
        if (lane == 0) gp[vs] = ga;
    }
}

// Every thread of the block, from warp 0's selection path and the other warps' gate path: a named
// barrier over the whole block (the two paths reach it from different code).
__device__ __forceinline__ void router_join() { asm volatile("bar.sync 2, %0;" ::"n"(kRouterThreads) : "memory"); }

__global__ void __launch_bounds__(kRouterThreads) router_kernel(const void* __restrict__ logits, int ldt,
                                                                const float* __restrict__ bias, int E, int K, int mode,
                                                                int renorm, float scale, int n_group, int topk_group,
                                                                uint32_t* __restrict__ inds, float* __restrict__ scores,
                                                                const void* gx, const void* gw, int gk, int gdt,
                                                                void* glogit) {
    extern __shared__ float sm[];
    float* key = sm;        // [E]
    float* wraw = sm + E;   // [E] (sigmoid modes)
    __shared__ float red_max[kRouterThreads / 32], red_sum[kRouterThreads / 32];
    __shared__ int sel[32];
    __shared__ float gscore[32];
    __shared__ float gp[16];
    const int row = blockIdx.x;
    const size_t lbase = (size_t)row * E;
    const bool sigmoid = mode != SX_ROUTER_SOFTMAX;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // Programmatic dependent launch: the next grid (a routed layer's first kernel, which waits for
    // this grid before reading the picks) may start launching now; this grid waits for the one
    // that wrote the logits before reading them.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    float lmax = -CUDART_INF_F;
    for (int e = tid; e < E; e += blockDim.x) {
        const float l = load_act(logits, lbase + e, ldt);
        if (sigmoid) {
            // The two-sided form of MLX's Sigmoid the reference mirrors (src/moe_router.zig:214-219).
            const float sy = 1.0f / (1.0f + expf(fabsf(l)));
            const float sg = l < 0.0f ? sy : 1.0f - sy;
            key[e] = sg + bias[e];
            wraw[e] = sg;
        } else {
            key[e] = l;
            wraw[e] = l;  // the picked logits' weights read it back (the key is masked when picked)
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
    if (warp != 0) {
        if (gk > 0) router_gate_partials(gx, gw, gk, gdt, gp);
        router_join();  // the gate's partials, for warp 0's final sum
        return;
    }

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

    // k rounds of "max, then mask", ties to the lowest id.  Each key becomes an order-preserving
    // integer (-inf and NaN: 0, never picked, as they lose every strict comparison; -0 as +0); a
    // round is a warp max over the lanes' best keys and a warp min over the ids holding it (one
    // redux each), and only the lane that held the pick rescans its keys.  With no key left the
    // pick is the last expert, as the comparison form gives.  Up to 512 experts a lane holds its
    // keys (e = lane + 32 i) in registers, so a rescan is a run of compares with no loads.
    auto ordered = [](float v) -> uint32_t {
        if (!(v > -CUDART_INF_F)) return 0u;  // -inf, NaN
        const uint32_t u = v == 0.0f ? 0u : __float_as_uint(v);
        return (u >> 31) ? ~u : (u | 0x80000000u);
    };
    uint32_t bk;
    int bi;
    if (E <= 512) {
        uint32_t kv[16];
#pragma unroll
        for (int i = 0; i < 16; i++) kv[i] = lane + 32 * i < E ? ordered(key[lane + 32 * i]) : 0u;
        auto rescan = [&]() {
            bk = 0u;
            bi = 0x7fffffff;
#pragma unroll
            for (int i = 0; i < 16; i++) {
                if (kv[i] > bk) {
                    bk = kv[i];
                    bi = lane + 32 * i;
                }
            }
        };
        rescan();
        for (int r = 0; r < K; r++) {
            const uint32_t top = __reduce_max_sync(0xffffffffu, bk);
            int pick = (int)__reduce_min_sync(0xffffffffu, (top != 0u && bk == top) ? (uint32_t)bi : 0xffffffffu);
            if (top == 0u) pick = E - 1;
            if (lane == 0) sel[r] = pick;
            if (lane == (pick & 31)) {
#pragma unroll
                for (int i = 0; i < 16; i++)
                    if (lane + 32 * i == pick) kv[i] = 0u;
                rescan();
            }
        }
    } else {
        auto lane_best = [&]() {
            bk = 0u;
            bi = 0x7fffffff;
            for (int e = lane; e < E; e += 32) {
                const uint32_t k = ordered(key[e]);
                if (k > bk) {
                    bk = k;
                    bi = e;
                }
            }
        };
        lane_best();
        for (int r = 0; r < K; r++) {
            const uint32_t top = __reduce_max_sync(0xffffffffu, bk);
            int pick = (int)__reduce_min_sync(0xffffffffu, (top != 0u && bk == top) ? (uint32_t)bi : 0xffffffffu);
            if (top == 0u) pick = E - 1;
            if (lane == 0) sel[r] = pick;
            if (lane == (pick & 31)) {
                key[pick] = -CUDART_INF_F;
                lane_best();
            }
            __syncwarp();
        }
    }
    __syncwarp();

    float w = 0.0f;
    int myidx = 0;
    if (lane < K) {
        myidx = sel[lane];
        w = sigmoid ? wraw[myidx] : expf(wraw[myidx] - smax) * snorm;
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
    router_join();
    if (gk > 0) {
        float gt = lane < 16 && lane < (gk + 1023) / 1024 ? gp[lane] : 0.0f;
#pragma unroll
        for (int m = 8; m > 0; m >>= 1) gt = __fadd_rn(gt, __shfl_xor_sync(0xffffffffu, gt, m));
        if (lane == 0) store_act(glogit, row, gdt, gt);
    }
}

}  // namespace sx

using namespace sx;

namespace {

sx_status router_launch(sx_stream stream, const void* logits, sx_dtype ldt, const float* bias, int32_t rows,
                        int32_t experts, int32_t k, int32_t mode, int32_t renorm, float scale, int32_t n_group,
                        int32_t topk_group, uint32_t* inds, float* scores, const void* gx, const void* gw, int32_t gk,
                        sx_dtype gdt, void* glogit) {
    if (!logits || !inds || !scores) return SX_ERR_NULL_POINTER;
    if (rows < 1) return SX_ERR_BAD_SHAPE;
    if (ldt != SX_DT_F32 && ldt != SX_DT_F16 && ldt != SX_DT_BF16) return SX_ERR_ROUTER_DECLINED;
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
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows, 1, 1);
    cfg.blockDim = dim3(kRouterThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, router_kernel, logits, (int)ldt, bias, (int)experts, (int)k, (int)mode,
                                          (int)renorm, scale, (int)n_group, (int)topk_group, inds, scores, gx, gw,
                                          (int)gk, (int)gdt, glogit),
                       "router launch");
}

}  // namespace

extern "C" sx_status sx_router_topk(sx_stream stream, const float* logits, const float* bias, int32_t rows,
                                    int32_t experts, int32_t k, int32_t mode, int32_t renorm, float scale,
                                    int32_t n_group, int32_t topk_group, uint32_t* inds, float* scores) {
    return router_launch(stream, logits, SX_DT_F32, bias, rows, experts, k, mode, renorm, scale, n_group, topk_group,
                         inds, scores, nullptr, nullptr, 0, SX_DT_BF16, nullptr);
}

extern "C" sx_status sx_router_topk_gate(sx_stream stream, const void* logits, sx_dtype logits_dtype, const float* bias,
                                         int32_t rows, int32_t experts, int32_t k, int32_t mode, int32_t renorm,
                                         float scale, int32_t n_group, int32_t topk_group, const void* gate_x,
                                         const void* gate_w, int32_t gate_k, sx_dtype gate_dtype, void* gate_logit,
                                         uint32_t* inds, float* scores) {
    // The gate rides the softmax mode only (src/moe_router.zig:471); the reference's admission of
    // it (:499-506): one row, 1..16384 elements in whole 8-element chunks, F16 or BF16.
    const bool gate = mode == SX_ROUTER_SOFTMAX && (gate_x || gate_w || gate_logit);
    if (gate) {
        if (!gate_x || !gate_w || !gate_logit) return SX_ERR_NULL_POINTER;
        if (rows != 1 || gate_k <= 0 || gate_k > 16384 || gate_k % 8 != 0) return SX_ERR_ROUTER_DECLINED;
        if (gate_dtype != SX_DT_F16 && gate_dtype != SX_DT_BF16) return SX_ERR_ROUTER_DECLINED;
    }
    return router_launch(stream, logits, logits_dtype, bias, rows, experts, k, mode, renorm, scale, n_group,
                         topk_group, inds, scores, gate ? gate_x : nullptr, gate ? gate_w : nullptr, gate ? gate_k : 0,
                         gate_dtype, gate ? gate_logit : nullptr);
}
