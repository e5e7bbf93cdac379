// Routed SwiGLU experts, decode chain (kernel templates; instantiated per codebook in
// sx_moe_{mcg,mul1,hash,pair1}.cu).  The reference runs four dispatches per MoE layer
// (src/exl3/expert_exl3_kernels.zig:2683 moeSwigluFused: pair prepare, split-K pair GEMV, fused
// mid+down GEMV, finish reduce); this chain is:
//   1. route_prep (one CTA): histogram of the slots' experts, scan, scatter -> slots sorted by
//      expert, the active experts, and a work list of (active expert, 8-row chunk), one record
//      and the slot ids per item.
// The four launch with programmatic dependent launch: each starts its prologue (barriers, shared
// memory) while its predecessor drains and waits for it before its first global access.
//   2. moe_pair: per work item and 128-wide block of the intermediate, gate AND up of the expert
//      for the chunk's rows (NP = 2 core, split-K cluster).  Its rank-0 epilogue does the
//      reference's mid (:2243 MID_SOURCE): H128, svh, SwiGLU in f32 (gate upper-clamped and up
//      clipped when a limit is set), times the down projection's suh, H128 over the same block,
//      rounded to f16: the down projection's prepared input.
//   3. moe_down: per work item and 128-wide output block, the down GEMV over the prepared rows,
//      H128, svh, times the slot's score, into a per-slot f32 plane.
//   4. moe_reduce: per token, the slots' planes summed in k order, rounded to the output dtype,
//      plus the shared expert (optionally sigmoid-gated), as moeWithShared/moeWithGatedShared do.
#pragma once

#include <cooperative_groups.h>

#include "sx_core.cuh"

namespace cg = cooperative_groups;

namespace sx {

struct MoeArgs {
    const void* x;          // [R][D]
    int xdt;
    int R, K, D, I, E;
    int e_lo;               // the group's first expert id: slot ids in [e_lo, e_lo + E) are this launch's
    const uint32_t* inds;   // [R*K]
    const float* scores;    // [R*K]
    const uint16_t* gate_tr; const uint16_t* gate_suh; const uint16_t* gate_svh;
    const uint16_t* up_tr;   const uint16_t* up_suh;   const uint16_t* up_svh;
    const uint16_t* down_tr; const uint16_t* down_suh; const uint16_t* down_svh;
    DecParams dp_gu, dp_down;
    float scale_gu, scale_down;
    float clamp;            // 0 = none
    // workspace
    int* meta;              // [0] = number of work items
    int* act_expert;        // [A_max]
    int* act_start;         // [A_max]
    int* act_count;         // [A_max]
    int* work_act;          // [W_max]
    int* work_chunk;        // [W_max]
    int* order;             // [R*K] slots sorted by expert
    uint16_t* hprep;        // [R*K][I] f16: the down projection's prepared input
    float* yslot;           // [R*K][D] f32: score * expert output
    // output
    const void* shared;     // [R][D] x dtype, or null
    const void* shared_gate;// [R] x dtype logits, or null
    void* y;                // [R][D] x dtype
    float* partial;         // [R][D] f32: when set, the k-order sum lands here unrounded (no shared)
    int chunk;              // rows per work item: 2 or 8 (decode chain) or kGemmRows (tensor-core path)
    int split_chunk;        // when set, the chunk the k splits are fitted for (direct items taking the routed chain's splits)
    int big_min;            // experts with this many rows or more go to the second list (INT_MAX: none)
    int big_chunk;          // rows per work item of the second list (4 row tiles per CTA)
    int* work_act4;         // second list: [W4_max]
    int* work_chunk4;
    int* sorted_e;          // [R*K] the expert of each sorted position
    int4* work_rec;         // [W_max] list-1 items: expert, first sorted position, rows
    int* work_slots;        // [W_max][8] decode chain (chunk 8): the slot id of each row of an item
    // A shared expert in the decode chain (sh_items > 0): work items w >= w_routed of the pair and
    // down launches are its 8-row chunks of all R rows, read from the sh_* bank (one expert), with
    // slot ids sh_slot0 + row (past the routed slots) and score 1.  w_routed = 0: a launch of the
    // shared expert alone (no routing metadata read).
    int w_routed, sh_items, sh_slot0;
    const void* sh_x;       // the shared expert's rows: x, or an expert-parallel rank's own rows
    int sh_rows;
    const uint16_t* sh_gate_tr; const uint16_t* sh_gate_suh; const uint16_t* sh_gate_svh;
    const uint16_t* sh_up_tr;   const uint16_t* sh_up_suh;   const uint16_t* sh_up_svh;
    const uint16_t* sh_down_tr; const uint16_t* sh_down_suh; const uint16_t* sh_down_svh;
    int sh_plane;           // reduce: the shared term is the plane of slots sh_slot0 + row, rounded
    // tensor-core path (sorted positions p): prepared gate/up inputs, gate/up outputs
    uint16_t* tg;           // [R*K][D] f16
    uint16_t* tu;           // [R*K][D] f16
    float* gf;              // [R*K][I] f32
    float* uf;              // [R*K][I] f32
    // An expert-parallel rank's received rows (seg_cnt set): R = nseg * seg_cap places, segment g
    // (the rows source rank g sent) live in its first min(seg_cnt[g], seg_cap) places; route_prep
    // reads the counts after its dependency wait and skips every other place.
    const int* seg_cnt;
    int seg_cap, nseg;
    const uint32_t* seg_wait;  // route_prep waits for seg_wait[g] >= *seg_seq, g < nseg, when set
    const uint32_t* seg_seq;
    // Direct items (direct != 0): no routing metadata; work item w < w_routed is slot w (its expert
    // inds[w] - e_lo, one row: w / K, slot id w), later items the folded shared expert's rows.  One
    // token: the down projection and the reduce run as moe_down1 (a cluster over the items per
    // output block).  An expert-parallel rank's small call: item w lives once its source's flag is
    // up and its place is within the rows that source sent; moe_down writes the per-slot planes.
    int direct;
    // The reduce folded into moe_down (a one-group decode-chain layer, rounded output): rcount
    // [R][D/128] arrival counters, zeroed by route_prep; the last of a (token, output block)'s
    // planes to land (its live routed slots, plus the shared plane when sh_plane) makes that
    // block of the token's output, as moe_reduce would.
    int* rcount;
};

// A token's routed sum `acc` (f32) made into its output value: rounded to the output dtype, then
// the shared expert added (optionally sigmoid-gated by the logit gl, with MLX's bf16/f16 rounding
// steps), as moeWithShared / moeWithGatedShared do (src/exl3/root.zig:56-92;
// moe_shared_fold.folded, src/moe_shared_fold.zig:24).  has_sh: a shared term sh (already in the
// output dtype's values) is added.
__device__ __forceinline__ float routed_finish_g(float acc, int xdt, bool has_sh, float sh, bool gated, float gl) {
    float y = acc;
    if (xdt != 0) y = xdt == 1 ? __half2float(__float2half_rn(y)) : __bfloat162float(__float2bfloat16_rn(y));
    if (has_sh) {
        if (gated) {
            float sg = 1.0f / (1.0f + expf(-gl));
            if (xdt == 2) {
                sg = __bfloat162float(__float2bfloat16_rn(sg));
                sh = __bfloat162float(__float2bfloat16_rn(sg * sh));
            } else if (xdt == 1) {
                sg = __half2float(__float2half_rn(sg));
                sh = __half2float(__float2half_rn(sg * sh));
            } else {
                sh = sg * sh;
            }
        }
        y = y + sh;
    }
    return y;
}

// routed_finish_g with token r's gate logit read from shared_gate [R] (null: no gate).
__device__ __forceinline__ float routed_finish(float acc, int xdt, bool has_sh, float sh, const void* shared_gate, int r) {
    const bool gated = has_sh && shared_gate;
    return routed_finish_g(acc, xdt, has_sh, sh, gated, gated ? load_act(shared_gate, r, xdt) : 0.0f);
}

// moe_reduce's arithmetic for four outputs d..d+3 of token r: the live slots' planes in k order,
// rounded, plus the shared term (the shared plane rounded, or the caller's shared row), gated.
// Plane reads bypass L1: other CTAs wrote them during this grid.
__device__ __forceinline__ void reduce_outputs4(const MoeArgs& a, int r, int d) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int k = 0; k < a.K; k++) {
        if (a.inds[r * a.K + k] >= (uint32_t)a.E) continue;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(a.yslot + (size_t)(r * a.K + k) * a.D + d));
        acc[0] += v.x;
        acc[1] += v.y;
        acc[2] += v.z;
        acc[3] += v.w;
    }
    float sh[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (a.sh_plane) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(a.yslot + (size_t)(a.sh_slot0 + r) * a.D + d));
        sh[0] = round_act(v.x, a.xdt), sh[1] = round_act(v.y, a.xdt), sh[2] = round_act(v.z, a.xdt);
        sh[3] = round_act(v.w, a.xdt);
    } else if (a.shared) {
#pragma unroll
        for (int i = 0; i < 4; i++) sh[i] = load_act(a.shared, (size_t)r * a.D + d + i, a.xdt);
    }
    const bool has_sh = a.sh_plane || a.shared;
#pragma unroll
    for (int i = 0; i < 4; i++)
        store_act(a.y, (size_t)r * a.D + d + i, a.xdt, routed_finish(acc[i], a.xdt, has_sh, sh[i], a.shared_gate, r));
}

// Work item -> (expert, first sorted slot, rows of the chunk); shx: a chunk of the shared expert
// (first = its first row).
struct WorkItem {
    int e, first, rows;
    bool shx;
};

// The item count and the item's record are loaded together (one round of global loads; a record
// past the count is never used).
__device__ __forceinline__ bool work_item(const MoeArgs& a, int w, WorkItem& it) {
    if (a.direct && w < a.w_routed) {
        if (a.seg_cnt) {  // an expert-parallel rank's received place w / K: live once its source's rows arrived
            const int place = w / a.K, g = place / a.seg_cap, i = place % a.seg_cap;
            if (a.seg_wait) wait_flag(a.seg_wait + g, *a.seg_seq);
            if (i >= min(max(a.seg_cnt[g], 0), a.seg_cap)) return false;
        }
        const uint32_t e = a.inds[w] - (uint32_t)a.e_lo;
        if (e >= (uint32_t)a.E) return false;  // the slot's expert is in no expert of this launch
        it.e = (int)e;
        it.first = w;
        it.rows = 1;
        it.shx = false;
        return true;
    }
    if (w >= a.w_routed) {
        const int c = w - a.w_routed;
        if (c >= a.sh_items) return false;
        it.e = 0;
        it.first = c * a.chunk;
        it.rows = min(a.chunk, a.sh_rows - c * a.chunk);
        it.shx = true;
        return true;
    }
    const int count = a.meta[0];
    const int4 rec = a.work_rec[w];
    if (w >= count) return false;
    it.e = rec.x;
    it.first = rec.y;
    it.rows = rec.z;
    it.shx = false;
    return true;
}

// work_item for the one-token down kernel (direct items, no expert-parallel segments).
__device__ __forceinline__ bool work_item_token(const MoeArgs& a, int w, WorkItem& it) {
    if (w < a.K) {
        const uint32_t e = a.inds[w] - (uint32_t)a.e_lo;
        if (e >= (uint32_t)a.E) return false;
        it.e = (int)e;
        it.first = w;
        it.rows = 1;
        it.shx = false;
        return true;
    }
    if (w - a.K >= a.sh_items) return false;
    it.e = 0;
    it.first = 0;
    it.rows = 1;
    it.shx = true;
    return true;
}

// The slot id of row t of a work item.
__device__ __forceinline__ int work_slot(const MoeArgs& a, int w, const WorkItem& it, int t) {
    return it.shx ? a.sh_slot0 + it.first + t : a.direct ? it.first : a.work_slots[w * 8 + t];  // (chunk <= 8)
}

// ------------------------------------------------------------------ 2. gate + up + mid
template <int KIND, int N>
__global__ void __launch_bounds__(kThreads, 3) moe_pair_kernel(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int slot_of[8];
    __shared__ __align__(16) uint16_t mid_h[3][128];  // rank 0's finish: gate svh, up svh, down suh
    cg::cluster_group cluster = cg::this_cluster();
    const int ob = blockIdx.y;
    const int S = cluster.dim_blocks().z;
    const int split = blockIdx.z % S;
    const int KB = a.D / 128;
    const int kb0 = (int)(((long long)split * KB) / S);
    const int kbl = (int)(((long long)(split + 1) * KB) / S) - kb0;
    const int kbl_max = (KB + S - 1) / S;
    const int mg = a.chunk;  // rows per work item: the B fragments hold this many rows
    const CoreSmem s = core_smem<N, 2, 1>(smem, kbl_max, mg);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int OT = a.I / 16;
    const size_t per = (size_t)(a.D / 16) * OT * N;
    core_init_barriers<N, 2, kConsumerWarps>(s);
    grid_dependency_wait();  // the routing comes from route_prep
    // Dependents may launch only now: every grid before this one has completed, so moe_down
    // may read the routing (and stream its weights) before its own dependency wait.
    grid_launch_dependents();
    WorkItem it;
    if (!work_item(a, blockIdx.x, it)) return;  // every CTA of the cluster shares blockIdx.x
    if (threadIdx.x < 8) slot_of[threadIdx.x] = threadIdx.x < it.rows ? work_slot(a, blockIdx.x, it, threadIdx.x) : 0;
    __syncthreads();

    if (warp == kConsumerWarps) {
        if (lane == 0) {
            const uint16_t* const tr[2] = {it.shx ? a.sh_gate_tr : a.gate_tr + (size_t)it.e * per,
                                           it.shx ? a.sh_up_tr : a.up_tr + (size_t)it.e * per};
            core_produce<N, 2>(s, tr, OT, ob, kb0, kbl);
        }
    } else {
        const uint16_t* suh_p[2] = {it.shx ? a.sh_gate_suh : a.gate_suh + (size_t)it.e * a.D,
                                    it.shx ? a.sh_up_suh : a.up_suh + (size_t)it.e * a.D};
        // Prepare: warp w takes units w, w + 8, ... of the (projection, input block) units; per unit
        // the lane's four suh values and the four x values of every row of the item are loaded
        // together (one round of loads), then each row is prepared: f16(x) * suh, Hadamard-128,
        // f16, into its B fragments.
        const void* xs = it.shx ? a.sh_x : a.x;
        const bool xvec = (reinterpret_cast<uintptr_t>(xs) & 15) == 0;
        // rank 0's finish weights of this block (gate and up svh, down suh): read by the last
        // consumer warp together with its prepare loads, kept in shared memory for the finish
        const bool mid_loader = split == 0 && warp == kConsumerWarps - 1;
        // (asynchronous copies straight into shared memory: no registers held across the prepare)
        if (mid_loader) {
            const uint16_t* mp[3] = {it.shx ? a.sh_gate_svh : a.gate_svh + (size_t)it.e * a.I,
                                     it.shx ? a.sh_up_svh : a.up_svh + (size_t)it.e * a.I,
                                     it.shx ? a.sh_down_suh : a.down_suh + (size_t)it.e * a.I};
#pragma unroll
            for (int q = 0; q < 3; q++) {
                const uint16_t* src = mp[q] + (size_t)ob * 128 + lane * 4;
                if ((reinterpret_cast<uintptr_t>(mp[q]) & 7) == 0) {
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(&mid_h[q][lane * 4])), "l"(src)
                                 : "memory");
                } else {
#pragma unroll
                    for (int i = 0; i < 4; i++) mid_h[q][lane * 4 + i] = src[i];
                }
            }
        }
        for (int u = warp; u < 2 * kbl; u += kConsumerWarps) {
            const int p = u / kbl, kbi = u % kbl;
            const int base = (kb0 + kbi) * 128 + lane * 4;
            float su[4];
            load_half4(suh_p[p], base, (reinterpret_cast<uintptr_t>(suh_p[p]) & 7) == 0, su);
            float v[8][4];
#pragma unroll
            for (int m = 0; m < 8; m++) {
                if (m < mg && m < it.rows) {
                    const int row = it.shx ? slot_of[m] - a.sh_slot0 : slot_of[m] / a.K;
                    load_act4v(xs, (size_t)row * a.D + base, a.xdt, xvec, v[m]);
                }
            }
#pragma unroll
            for (int m = 0; m < 8; m++) {
                if (m >= mg) continue;
                float (&vr)[4] = v[m];
                if (m < it.rows) {
#pragma unroll
                    for (int i = 0; i < 4; i++) vr[i] = round_f16(vr[i]) * su[i];
                    warp_hadamard128(vr);
                } else {
                    vr[0] = vr[1] = vr[2] = vr[3] = 0.0f;
                }
                const uint16_t h[4] = {f2h(vr[0]), f2h(vr[1]), f2h(vr[2]), f2h(vr[3])};
                bfrag_put4<1>(s.bfrag + p * s.bfrag_proj_stride, mg, kbi, m, lane, h);
            }
        }
        if (mid_loader) asm volatile("cp.async.wait_all;" ::: "memory");
        consumers_sync<kConsumerWarps>();
        const DecParams dp[2] = {a.dp_gu, a.dp_gu};
        float acc[2][1][4];
        core_consume<KIND, N, 2, 1, false, kConsumerWarps>(s, kbl, dp, acc);
        core_reduce<2, 1, kConsumerWarps>(s.red, acc);
    }

    cluster.sync();
    if (split == 0 && warp < it.rows) {
        const int m = warp;
        const float4 gs = cluster_sum4(cluster, s.red, S, m * 128);
        const float4 us = cluster_sum4(cluster, s.red, S, 8 * 128 + m * 128);
        float g[4] = {gs.x, gs.y, gs.z, gs.w}, u[4] = {us.x, us.y, us.z, us.w};
        warp_hadamard128(g);
        warp_hadamard128(u);
        float h[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int o = lane * 4 + i;
            float gv = g[i] * a.scale_gu * h2f(mid_h[0][o]);
            float uv = u[i] * a.scale_gu * h2f(mid_h[1][o]);
            if (a.clamp > 0.0f) {
                gv = fminf(gv, a.clamp);
                uv = fminf(fmaxf(uv, -a.clamp), a.clamp);
            }
            h[i] = gv / (1.0f + expf(-gv)) * uv * h2f(mid_h[2][o]);
        }
        warp_hadamard128(h);
        uint16_t* dst = a.hprep + (size_t)slot_of[m] * a.I + ob * 128 + lane * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) dst[i] = f2h(h[i]);
    }
    cluster.sync();
}

// ------------------------------------------------------------------ 3. down
template <int KIND, int N>
__global__ void __launch_bounds__(kThreads, 3) moe_down_kernel(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int slot_of[8];
    cg::cluster_group cluster = cg::this_cluster();
    const int ob = blockIdx.y;
    const int S = cluster.dim_blocks().z;
    const int split = blockIdx.z % S;
    const int KB = a.I / 128;
    const int kb0 = (int)(((long long)split * KB) / S);
    const int kbl = (int)(((long long)(split + 1) * KB) / S) - kb0;
    const int kbl_max = (KB + S - 1) / S;
    const int mg = a.chunk;  // rows per work item: the B fragments hold this many rows
    const CoreSmem s = core_smem<N, 1, 1>(smem, kbl_max, mg);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int OT = a.D / 16;
    const size_t per = (size_t)(a.I / 16) * OT * N;
    core_init_barriers<N, 1, kConsumerWarps>(s);
    grid_launch_dependents();
    // moe_pair (this grid's predecessor) lets it launch only after its own dependency wait, so the
    // routing (route_prep's, from before moe_pair) is complete here: the work record is read and
    // the expert's weights stream before this grid's wait, which guards only the prepared rows
    // (moe_pair's output).  A CTA without work still waits, so this grid completes after moe_pair.
    WorkItem it;
    if (!work_item(a, blockIdx.x, it)) {
        grid_dependency_wait();
        return;
    }
    if (threadIdx.x < 8) slot_of[threadIdx.x] = threadIdx.x < it.rows ? work_slot(a, blockIdx.x, it, threadIdx.x) : 0;
    __syncthreads();

    if (warp == kConsumerWarps) {
        if (lane == 0) {
            const uint16_t* const tr[1] = {it.shx ? a.sh_down_tr : a.down_tr + (size_t)it.e * per};
            core_produce<N, 1>(s, tr, OT, ob, kb0, kbl);
        }
    } else {
        grid_dependency_wait();  // the prepared rows come from moe_pair
        const bool hvec = (reinterpret_cast<uintptr_t>(a.hprep) & 7) == 0;
        for (int item = warp; item < kbl * mg; item += kConsumerWarps) {
            const int kbi = item / mg, m = item % mg;
            const uint16_t* src = a.hprep + (size_t)slot_of[m] * a.I + (kb0 + kbi) * 128 + lane * 4;
            uint16_t h[4] = {0, 0, 0, 0};
            if (m < it.rows) {
                if (hvec) {
                    const uint2 u = *reinterpret_cast<const uint2*>(src);
                    h[0] = (uint16_t)u.x, h[1] = (uint16_t)(u.x >> 16), h[2] = (uint16_t)u.y, h[3] = (uint16_t)(u.y >> 16);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; i++) h[i] = src[i];
                }
            }
            bfrag_put4<1>(s.bfrag, mg, kbi, m, lane, h);
        }
        consumers_sync<kConsumerWarps>();
        const DecParams dp[1] = {a.dp_down};
        float acc[1][1][4];
        core_consume<KIND, N, 1, 1, false, kConsumerWarps>(s, kbl, dp, acc);
        core_reduce<1, 1, kConsumerWarps>(s.red, acc);
    }

    cluster.sync();
    if (split == 0 && warp < it.rows) {
        const int m = warp;
        const float4 ds = cluster_sum4(cluster, s.red, S, m * 128);
        float d[4] = {ds.x, ds.y, ds.z, ds.w};
        warp_hadamard128(d);
        const int slot = slot_of[m];
        const float sc = (it.shx ? 1.0f : a.scores[slot]) * a.scale_down;
        const uint16_t* dsv = it.shx ? a.sh_down_svh : a.down_svh + (size_t)it.e * a.D;
        float* dst = a.yslot + (size_t)slot * a.D + ob * 128 + lane * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) dst[i] = d[i] * h2f(dsv[ob * 128 + lane * 4 + i]) * sc;
        if (a.rcount) {
            // the folded reduce: the last plane of (token, output block) to land makes the block
            const int r = it.shx ? it.first + m : slot / a.K;
            __threadfence();
            __syncwarp();
            const bool live = lane < a.K && a.inds[r * a.K + lane] < (uint32_t)a.E;
            const int need = __popc(__ballot_sync(0xffffffffu, live)) + (a.sh_plane ? 1 : 0);
            int last = 0;
            if (lane == 0) last = atomicAdd(&a.rcount[r * (a.D / 128) + ob], 1) == need - 1;
            if (__shfl_sync(0xffffffffu, last, 0)) {
                __threadfence();
                reduce_outputs4(a, r, ob * 128 + lane * 4);
            }
        }
    }
    cluster.sync();
}

// ------------------------------------------------------------------ 3'. one token: down + reduce
// A one-token layer (direct work items): grid (D/128 output blocks, W items), clusters of the W
// items of one output block.  Rank w runs item w's down GEMV over the whole intermediate (its
// expert's weights stream before the dependency wait, as in moe_down), finishes it as moe_down
// does (H128 of its sum, svh, the slot's score) into its own shared memory; rank 0 then adds the
// live slots' blocks in k order over distributed shared memory, rounds and adds the shared term
// (the shared item's block rounded, or the caller's shared row, gated): moe_reduce's arithmetic
// with no per-slot planes and no arrival counters.  (The codebooks other than MCG, and MCG above
// 6 bits per weight, need the registers of two CTAs per SM here.)
template <int KIND, int N>
__global__ void __launch_bounds__(kThreads, KIND == K_MCG && N <= 96 ? 3 : 2) moe_down1_kernel(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int ob = blockIdx.x;
    const int w = blockIdx.y;  // the item, and the rank in the cluster
    const int KB = a.I / 128;
    const CoreSmem s = core_smem<N, 1, 1>(smem, KB, 1);
    float* fin = s.red + 128;  // the finished block (row 1 of the reduction area: one row here)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int OT = a.D / 16;
    const size_t per = (size_t)(a.I / 16) * OT * N;
    core_init_barriers<N, 1, kConsumerWarps>(s);
    grid_launch_dependents();
    // Routing is complete here (moe_pair lets this grid launch after its own dependency wait):
    // the item, its finish's svh values and score are read before this grid's wait.
    // (kept in shared memory across the main loop, not in registers)
    __shared__ __align__(16) float fin_sv[128];
    __shared__ float fin_sc;
    WorkItem it;
    const bool has = work_item_token(a, w, it);
    __syncthreads();

    if (warp == kConsumerWarps) {
        if (lane == 0 && has) {
            const uint16_t* const tr[1] = {it.shx ? a.sh_down_tr : a.down_tr + (size_t)it.e * per};
            core_produce<N, 1>(s, tr, OT, ob, 0, KB);
        }
    } else {
        if (has && warp == 0) {
            const uint16_t* dsv = it.shx ? a.sh_down_svh : a.down_svh + (size_t)it.e * a.D;
            float sv[4];
            load_half4(dsv, (size_t)ob * 128 + lane * 4, (reinterpret_cast<uintptr_t>(dsv) & 7) == 0, sv);
            *reinterpret_cast<float4*>(fin_sv + lane * 4) = make_float4(sv[0], sv[1], sv[2], sv[3]);
            if (lane == 0) fin_sc = (it.shx ? 1.0f : a.scores[w]) * a.scale_down;
        }
        const int hrow = has ? work_slot(a, w, it, 0) : 0;
        grid_dependency_wait();  // the prepared rows come from moe_pair
        if (has) {
            const bool hvec = (reinterpret_cast<uintptr_t>(a.hprep) & 7) == 0;
            for (int kbi = warp; kbi < KB; kbi += kConsumerWarps) {
                const uint16_t* src = a.hprep + (size_t)hrow * a.I + kbi * 128 + lane * 4;
                uint16_t h[4];
                if (hvec) {
                    const uint2 u = *reinterpret_cast<const uint2*>(src);
                    h[0] = (uint16_t)u.x, h[1] = (uint16_t)(u.x >> 16), h[2] = (uint16_t)u.y, h[3] = (uint16_t)(u.y >> 16);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; i++) h[i] = src[i];
                }
                bfrag_put4<1>(s.bfrag, 1, kbi, 0, lane, h);
            }
            consumers_sync<kConsumerWarps>();
            const DecParams dp[1] = {a.dp_down};
            float acc[1][1][4];
            core_consume<KIND, N, 1, 1, false, kConsumerWarps>(s, KB, dp, acc);
            core_reduce<1, 1, kConsumerWarps>(s.red, acc);
            consumers_sync<kConsumerWarps>();
            if (warp == 0) {
                // moe_down's finish of an unsplit block (0 + partial, as its one-rank cluster sum)
                const float4 t = *reinterpret_cast<const float4*>(s.red + lane * 4);
                float d[4] = {0.0f + t.x, 0.0f + t.y, 0.0f + t.z, 0.0f + t.w};
                warp_hadamard128(d);
                const float4 sv = *reinterpret_cast<const float4*>(fin_sv + lane * 4);
                const float sc = fin_sc;
                float4 f;
                f.x = d[0] * sv.x * sc;
                f.y = d[1] * sv.y * sc;
                f.z = d[2] * sv.z * sc;
                f.w = d[3] * sv.w * sc;
                *reinterpret_cast<float4*>(fin + lane * 4) = f;
            }
        }
    }

    // Rank 0's sum: the live slots (a ballot over the slot ids, read before the barrier, as are
    // the caller's shared row and the gate) loaded from every rank at once, added in k order.
    const int d0 = ob * 128 + lane * 4;
    unsigned live = 0u;
    float sh[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float gate = 0.0f;
    if (w == 0 && warp == 0) {
        live = __ballot_sync(0xffffffffu, lane < a.K && a.inds[lane] - (uint32_t)a.e_lo < (uint32_t)a.E);
        if (!a.sh_plane && a.shared) {
#pragma unroll
            for (int i = 0; i < 4; i++) sh[i] = load_act(a.shared, d0 + i, a.xdt);
        }
        if (a.shared_gate) gate = load_act(a.shared_gate, 0, a.xdt);
    }
    cluster.sync();
    if (w == 0 && warp == 0) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int k0 = 0; k0 < 16; k0 += 8) {  // eight ranks' loads in flight at a time
            float4 v[8];
#pragma unroll
            for (int k = 0; k < 8; k++)
                if ((live >> (k0 + k)) & 1u)
                    v[k] = *reinterpret_cast<const float4*>(cluster.map_shared_rank(fin, k0 + k) + lane * 4);
#pragma unroll
            for (int k = 0; k < 8; k++) {
                if (!((live >> (k0 + k)) & 1u)) continue;
                acc[0] += v[k].x;
                acc[1] += v[k].y;
                acc[2] += v[k].z;
                acc[3] += v[k].w;
            }
        }
        if (a.sh_plane) {
            const float4 s4 = *reinterpret_cast<const float4*>(cluster.map_shared_rank(fin, a.K) + lane * 4);
            sh[0] = round_act(s4.x, a.xdt), sh[1] = round_act(s4.y, a.xdt), sh[2] = round_act(s4.z, a.xdt);
            sh[3] = round_act(s4.w, a.xdt);
        }
        const bool has_sh = a.sh_plane || a.shared;
#pragma unroll
        for (int i = 0; i < 4; i++) store_act(a.y, d0 + i, a.xdt, routed_finish_g(acc[i], a.xdt, has_sh, sh[i], a.shared_gate != nullptr, gate));
    }
    cluster.sync();
}

}  // namespace sx
