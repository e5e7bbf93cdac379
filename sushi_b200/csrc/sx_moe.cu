// Routed SwiGLU experts: sx_moe (root.moe / moeWithShared / moeWithGatedShared / moeClamped,
// src/exl3/root.zig:51-125) and its workspace query.  Kernels in sx_moe_impl.cuh.
#include <algorithm>
#include <cmath>

#include "sx_gemm_impl.cuh"
#include "sx_internal.h"
#include "sx_moe_impl.cuh"

namespace sx {

template <int KIND>
cudaError_t moe_launch_kind(const MoeArgs& a, int n_gu, int n_d, int S_gu, int S_d, int W_max, cudaStream_t stream);
template <int KIND>
cudaError_t moe_launch_kind_direct(const MoeArgs& a, int n_gu, int n_d, int S_gu, int W, cudaStream_t stream);

namespace {

// A plain (non-cluster) launch with programmatic dependent launch allowed.
template <typename Kern>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const MoeArgs& a) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

// ------------------------------------------------------------------ 1. routing metadata
// Exclusive block-wide scan of four counters (1024 threads); `tot` receives the block's sums.
// Every thread of the block calls it.
__device__ __forceinline__ int4 block_scan4(int4 v, int4* wsum, int4& tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int4 inc = v;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const int tx = __shfl_up_sync(0xffffffffu, inc.x, m), ty = __shfl_up_sync(0xffffffffu, inc.y, m);
        const int tz = __shfl_up_sync(0xffffffffu, inc.z, m), tw = __shfl_up_sync(0xffffffffu, inc.w, m);
        if (lane >= m) inc.x += tx, inc.y += ty, inc.z += tz, inc.w += tw;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int4 w = lane < nw ? wsum[lane] : make_int4(0, 0, 0, 0);
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) {
            const int tx = __shfl_up_sync(0xffffffffu, w.x, m), ty = __shfl_up_sync(0xffffffffu, w.y, m);
            const int tz = __shfl_up_sync(0xffffffffu, w.z, m), tw = __shfl_up_sync(0xffffffffu, w.w, m);
            if (lane >= m) w.x += tx, w.y += ty, w.z += tz, w.w += tw;
        }
        if (lane < nw) wsum[lane] = w;
    }
    __syncthreads();
    const int4 pre = warp > 0 ? wsum[warp - 1] : make_int4(0, 0, 0, 0);
    tot = wsum[nw - 1];
    __syncthreads();  // wsum is reused by the next call
    return make_int4(pre.x + inc.x - v.x, pre.y + inc.y - v.y, pre.z + inc.z - v.z, pre.w + inc.w - v.w);
}

// One CTA: the slots' expert histogram, a block-wide scan over the experts, and the scatter of
// slots into expert order.  Work items: experts with fewer than big_min rows are cut into chunks
// of `chunk` rows (list 1, meta[0] items, one record each: expert, first sorted position, rows);
// larger ones into chunks of big_chunk rows (list 2, meta[1] items), so that the tensor-core path
// can reuse each decoded weight chunk over four row tiles.  meta[2] = slots.  With chunk 8 (the
// decode chain) each list-1 item also lists its rows' slot ids.
__global__ void __launch_bounds__(1024) route_prep_kernel(MoeArgs a) {
    extern __shared__ int rp[];
    int* cnt = rp;             // [E]
    int* off = rp + a.E;       // [E] first sorted position
    int* wb = rp + 2 * a.E;    // [E] first list-1 item
    __shared__ int4 wsum[32];
    const int tid = threadIdx.x;
    const int RK = a.R * a.K;
    grid_launch_dependents();
    for (int e = tid; e < a.E; e += blockDim.x) cnt[e] = 0;
    grid_dependency_wait();  // the routing comes from the previous kernel
    if (a.seg_wait) {  // an expert-parallel rank's received rows: every source's flag of this call
        const uint32_t seq = *a.seg_seq;
        for (int g = tid; g < a.nseg; g += blockDim.x) wait_flag(a.seg_wait + g, seq);
    }
    __syncthreads();
    // The slots to sort, in warp-uniform strides: every slot, or an expert-parallel rank's live
    // places only (segment by segment).  body(s, in_range) runs on every lane of a warp at once.
    auto for_slots = [&](auto&& body) {
        if (!a.seg_cnt) {
            for (int s0 = tid - (tid & 31); s0 < RK; s0 += blockDim.x) body(s0 + (tid & 31), s0 + (tid & 31) < RK);
            return;
        }
        for (int g = 0; g < a.nseg; g++) {
            const int live = min(max(a.seg_cnt[g], 0), a.seg_cap) * a.K;
            const int base = g * a.seg_cap * a.K;
            for (int s0 = tid - (tid & 31); s0 < live; s0 += blockDim.x)
                body(base + s0 + (tid & 31), s0 + (tid & 31) < live);
        }
    };
    // Warp-aggregated counting: lanes holding the same expert add once (a hot expert would
    // otherwise serialise thousands of atomics on one shared-memory word).
    for_slots([&](int s, bool in_range) {
        const uint32_t e = in_range ? a.inds[s] - (uint32_t)a.e_lo : 0xFFFFFFFFu;  // ids below the group wrap past E
        const bool valid = e < (uint32_t)a.E;
        const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : 0xFFFFFFFFu);
        if (valid && (tid & 31) == __ffs(peers) - 1) atomicAdd(&cnt[e], __popc(peers));
    });
    __syncthreads();
    auto items1 = [&](int c) { return c >= a.big_min ? 0 : (c + a.chunk - 1) / a.chunk; };
    auto items2 = [&](int c) { return c >= a.big_min ? (c + a.big_chunk - 1) / a.big_chunk : 0; };
    int4 carry = make_int4(0, 0, 0, 0);  // slots, active experts, list-1 items, list-2 items
    for (int base = 0; base < a.E; base += blockDim.x) {
        const int e = base + tid;
        const int c = e < a.E ? cnt[e] : 0;
        int4 tot;
        const int4 ex = block_scan4(make_int4(c, c > 0, items1(c), items2(c)), wsum, tot);
        if (c > 0) {
            const int s0 = carry.x + ex.x, ai = carry.y + ex.y, w0 = carry.z + ex.z, v0 = carry.w + ex.w;
            off[e] = s0;
            wb[e] = w0;
            a.act_expert[ai] = e;
            a.act_start[ai] = s0;
            a.act_count[ai] = c;
            for (int ch = 0; ch < items1(c); ch++) {
                a.work_act[w0 + ch] = ai;
                a.work_chunk[w0 + ch] = ch;
                a.work_rec[w0 + ch] = make_int4(e, s0 + ch * a.chunk, min(a.chunk, c - ch * a.chunk), 0);
            }
            for (int ch = 0; ch < items2(c); ch++) {
                a.work_act4[v0 + ch] = ai;
                a.work_chunk4[v0 + ch] = ch;
            }
        }
        carry.x += tot.x, carry.y += tot.y, carry.z += tot.z, carry.w += tot.w;
    }
    if (tid == 0) {
        a.meta[0] = carry.z;
        a.meta[1] = carry.w;
        a.meta[2] = carry.x;
    }
    if (a.rcount)  // the folded reduce's arrival counters of this call (after the dependency wait)
        for (int i = tid; i < a.R * (a.D / 128); i += blockDim.x) a.rcount[i] = 0;
    __syncthreads();
    for (int e = tid; e < a.E; e += blockDim.x) cnt[e] = 0;  // reused as cursors
    __syncthreads();
    for_slots([&](int s, bool in_range) {
        const int lane = tid & 31;
        const uint32_t e = in_range ? a.inds[s] - (uint32_t)a.e_lo : 0xFFFFFFFFu;
        const bool valid = e < (uint32_t)a.E;
        const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : 0xFFFFFFFFu);
        const int leader = __ffs(peers) - 1;
        int base = 0;
        if (valid && lane == leader) base = atomicAdd(&cnt[e], __popc(peers));
        base = __shfl_sync(0xffffffffu, base, leader);
        if (valid) {
            const int pos = base + __popc(peers & ((1u << lane) - 1u));
            a.order[off[e] + pos] = s;
            a.sorted_e[off[e] + pos] = (int)e;
            if (a.chunk <= 8 && pos < a.big_min) a.work_slots[(wb[e] + pos / a.chunk) * 8 + pos % a.chunk] = s;
        }
    });
}

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

struct MoeWs {
    size_t meta, act_expert, act_start, act_count, work_act, work_chunk, work_act4, work_chunk4, order, sorted_e, hprep,
        yslot, tg, tu, gf, uf, work_rec, work_slots, rcount, total;
    int A_max, W_max, W4_max, chunk, big_min, big_chunk;
    bool gemm;
};

// Experts with at least this many routed rows take the four-row-tile kernel (chunks of 512).
constexpr int kBigRows = 3 * kGemmRows;

// The decode chain serves up to 16 rows (the reference's DECODE_ROWS_MAX,
// src/exl3/expert_exl3_kernels.zig:152); more rows go through the tensor-core path once the
// routed slots average at least 16 rows per active expert, so that a 128-row tile is not mostly
// empty (decode batches of 64 tokens spread over 512 experts stay on the decode chain).
// `slots` bounds the slots that can be valid (R*K for sx_moe; an expert-parallel rank's share).
constexpr int kDecodeRowsMax = 16;

bool use_gemm(int E, int R, int K, long long slots) {
    if (R <= kDecodeRowsMax) return false;
    if (slots <= 0) slots = (long long)R * K;
    return slots >= 16LL * std::min<long long>(E, slots);
}

// Rows per work item of the decode chain: kSmallChunk when the routed slots spread over about as
// many experts as there are slots (at most two rows per active expert expected for uniform
// routing), so a CTA's B fragments hold two rows and its shared memory fits fewer k splits; else 8.
#ifndef SX_CHAIN_SMALL_CHUNK
#define SX_CHAIN_SMALL_CHUNK 2
#endif
constexpr int kSmallChunk = SX_CHAIN_SMALL_CHUNK;

int chain_chunk(int E, int R, int K, long long slots) {
    const double v = slots > 0 ? (double)slots : (double)R * K;
    const double active = E * (1.0 - std::exp(-v / std::max(1, E)));
    return v <= 2.0 * active ? kSmallChunk : 8;
}

// extra_rows: prepared-input rows past the routed slots (a shared expert's rows riding the chain).
// bound: the routed slots known to be valid at most (-1: R*K); it sizes the work lists, the
// sorted positions and the launches that run over them (not the per-slot planes, indexed by slot).
MoeWs moe_ws_layout(int E, int R, int K, int D, int I, int n_gu, int n_d, long long slots = 0, bool with_yslot = true,
                    int extra_rows = 0, long long bound = -1) {
    MoeWs w;
    const int RK = bound >= 0 ? (int)std::min<long long>(bound, (long long)R * K) : R * K;
    w.gemm = use_gemm(E, R, K, slots);
    const bool big = w.gemm && gemm_rt_rate(n_gu) && gemm_rt_rate(n_d);
    w.chunk = w.gemm ? kGemmRows : chain_chunk(E, R, K, slots);
    w.big_min = big ? kBigRows : 0x7FFFFFFF;
    w.big_chunk = 4 * kGemmRows;
    w.A_max = std::min(E, RK);
    w.W_max = w.A_max + RK / w.chunk + 1;
    w.W4_max = big ? RK / w.big_chunk + RK / w.big_min + 1 : 0;
    size_t off = 0;
    w.meta = off; off = align_up(off + 16 * sizeof(int));
    w.act_expert = off; off = align_up(off + (size_t)w.A_max * sizeof(int));
    w.act_start = off; off = align_up(off + (size_t)w.A_max * sizeof(int));
    w.act_count = off; off = align_up(off + (size_t)w.A_max * sizeof(int));
    w.work_act = off; off = align_up(off + (size_t)w.W_max * sizeof(int));
    w.work_chunk = off; off = align_up(off + (size_t)w.W_max * sizeof(int));
    w.work_rec = off; off = align_up(off + (size_t)w.W_max * sizeof(int4));
    w.work_slots = off; off = align_up(off + (size_t)(w.gemm ? 1 : w.W_max * 8) * sizeof(int));
    w.rcount = off; off = align_up(off + (size_t)(w.gemm ? 1 : R * ((D + 127) / 128)) * sizeof(int));
    w.work_act4 = off; off = align_up(off + (size_t)std::max(1, w.W4_max) * sizeof(int));
    w.work_chunk4 = off; off = align_up(off + (size_t)std::max(1, w.W4_max) * sizeof(int));
    w.order = off; off = align_up(off + (size_t)RK * sizeof(int));
    w.sorted_e = off; off = align_up(off + (size_t)RK * sizeof(int));
    w.hprep = off; off = align_up(off + (size_t)(RK + extra_rows) * I * sizeof(uint16_t));
    w.yslot = off;
    if (with_yslot) off = align_up(off + (size_t)R * K * D * sizeof(float));
    w.tg = w.tu = w.gf = w.uf = 0;
    if (w.gemm) {
        w.tg = off; off = align_up(off + (size_t)RK * D * sizeof(uint16_t));
        w.tu = off; off = align_up(off + (size_t)RK * D * sizeof(uint16_t));
        w.gf = off; off = align_up(off + (size_t)RK * I * sizeof(float));
        w.uf = off; off = align_up(off + (size_t)RK * I * sizeof(float));
    }
    w.total = off;
    return w;
}

// Per token and 512-wide block of the output (128 threads, four outputs each): the token's slots
// in k order summed, rounded, plus the shared expert; or the unrounded f32 partial.
constexpr int kReduceCols = 512;

__global__ void __launch_bounds__(128) moe_reduce_kernel(MoeArgs a) {
    const int r = blockIdx.x;
    __shared__ int live[32];  // the row's slots with an expert of the layer, in k order
    __shared__ int nlive;
    grid_launch_dependents();
    grid_dependency_wait();  // the slots' planes come from the previous kernels
    if (threadIdx.x < 32) {
        const int k = threadIdx.x;
        const bool ok = k < a.K && a.inds[r * a.K + k] < (uint32_t)a.E;
        const unsigned m = __ballot_sync(0xffffffffu, ok);
        if (ok) live[__popc(m & ((1u << k) - 1u))] = r * a.K + k;
        if (k == 0) nlive = __popc(m);
    }
    __syncthreads();
    const int nl = nlive;
    const int d = blockIdx.y * kReduceCols + threadIdx.x * 4;
    if (d >= a.D) return;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int j = 0; j < nl; j++) {
        const float4 v = *reinterpret_cast<const float4*>(a.yslot + (size_t)live[j] * a.D + d);
        acc[0] += v.x;
        acc[1] += v.y;
        acc[2] += v.z;
        acc[3] += v.w;
    }
    if (a.partial) {  // an expert-parallel rank's share: combined and rounded by the token's owner
        *reinterpret_cast<float4*>(a.partial + (size_t)r * a.D + d) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        return;
    }
    // The routed sum is rounded to the output dtype before a shared expert is added
    // (docs/engine-exl3-experts.md "Streamed serial decode"; src/exl3/root.zig:56-92).
    float sh[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (a.sh_plane) {  // the shared expert's plane, rounded as its own layer output would be
        const float4 v = *reinterpret_cast<const float4*>(a.yslot + (size_t)(a.sh_slot0 + r) * a.D + d);
        sh[0] = round_act(v.x, a.xdt), sh[1] = round_act(v.y, a.xdt), sh[2] = round_act(v.z, a.xdt);
        sh[3] = round_act(v.w, a.xdt);
    } else if (a.shared) {
#pragma unroll
        for (int i = 0; i < 4; i++) sh[i] = load_act(a.shared, (size_t)r * a.D + d + i, a.xdt);
    }
    const bool has_sh = a.sh_plane || a.shared;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float y = routed_finish(acc[i], a.xdt, has_sh, sh[i], a.shared_gate, r);
        store_act(a.y, (size_t)r * a.D + d + i, a.xdt, y);
    }
}

// ------------------------------------------------------------------ tensor-core path
// The gate and up projections' prepared inputs of every sorted position p (slot order[p], token
// order[p] / K, expert sorted_e[p]): f16(H128(f16(x) * suh)) per 128-input block, as
// prepareInput does.  One warp per position and block; positions past meta[2] return.
__global__ void __launch_bounds__(256) moe_prep_kernel(MoeArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p = blockIdx.x * 8 + warp;
    if (p >= a.meta[2]) return;
    const int e = a.sorted_e[p];
    const int kb = blockIdx.y;
    const int base = kb * 128 + lane * 4;
    const uint16_t* sg = a.gate_suh + (size_t)e * a.D;
    const uint16_t* su = a.up_suh + (size_t)e * a.D;
    const int tok = a.order[p] / a.K;
    float xv[4];
    load_act4(a.x, (size_t)tok * a.D + base, a.xdt, xv);
    const uint2 sgv = *reinterpret_cast<const uint2*>(sg + base);
    const uint2 suv = *reinterpret_cast<const uint2*>(su + base);
    const uint16_t sgh[4] = {(uint16_t)sgv.x, (uint16_t)(sgv.x >> 16), (uint16_t)sgv.y, (uint16_t)(sgv.y >> 16)};
    const uint16_t suh4[4] = {(uint16_t)suv.x, (uint16_t)(suv.x >> 16), (uint16_t)suv.y, (uint16_t)(suv.y >> 16)};
    float g[4], u[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float v = round_f16(xv[i]);
        g[i] = v * h2f(sgh[i]);
        u[i] = v * h2f(suh4[i]);
    }
    warp_hadamard128(g);
    warp_hadamard128(u);
    uint2 hg, hu;
    hg.x = (uint32_t)f2h(g[0]) | ((uint32_t)f2h(g[1]) << 16);
    hg.y = (uint32_t)f2h(g[2]) | ((uint32_t)f2h(g[3]) << 16);
    hu.x = (uint32_t)f2h(u[0]) | ((uint32_t)f2h(u[1]) << 16);
    hu.y = (uint32_t)f2h(u[2]) | ((uint32_t)f2h(u[3]) << 16);
    *reinterpret_cast<uint2*>(a.tg + (size_t)p * a.D + base) = hg;
    *reinterpret_cast<uint2*>(a.tu + (size_t)p * a.D + base) = hu;
}

// The reference's mid (expert_exl3_kernels.zig:2243 MID_SOURCE) on the gate and up outputs of
// every sorted position: SwiGLU in f32 (gate upper-clamped, up clipped when a limit is set), times
// the down projection's suh, H128, rounded to f16: the down projection's prepared input.
__global__ void __launch_bounds__(256) moe_mid_kernel(MoeArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p = blockIdx.x * 8 + warp;
    if (p >= a.meta[2]) return;
    const int e = a.sorted_e[p];
    const int o0 = blockIdx.y * 128 + lane * 4;
    const uint16_t* dsu = a.down_suh + (size_t)e * a.I;
    const float4 g4 = *reinterpret_cast<const float4*>(a.gf + (size_t)p * a.I + o0);
    const float4 u4 = *reinterpret_cast<const float4*>(a.uf + (size_t)p * a.I + o0);
    const float gg[4] = {g4.x, g4.y, g4.z, g4.w}, uu[4] = {u4.x, u4.y, u4.z, u4.w};
    float h[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float gv = gg[i], uv = uu[i];
        if (a.clamp > 0.0f) {
            gv = fminf(gv, a.clamp);
            uv = fminf(fmaxf(uv, -a.clamp), a.clamp);
        }
        h[i] = gv / (1.0f + expf(-gv)) * uv * h2f(dsu[o0 + i]);
    }
    warp_hadamard128(h);
    uint2 hh;
    hh.x = (uint32_t)f2h(h[0]) | ((uint32_t)f2h(h[1]) << 16);
    hh.y = (uint32_t)f2h(h[2]) | ((uint32_t)f2h(h[3]) << 16);
    *reinterpret_cast<uint2*>(a.hprep + (size_t)p * a.I + o0) = hh;
}

void set_shared_ptrs(MoeArgs& a, const sx_bank& sh) {
    a.sh_gate_tr = sh.gate.trellis; a.sh_gate_suh = sh.gate.suh; a.sh_gate_svh = sh.gate.svh;
    a.sh_up_tr = sh.up.trellis;     a.sh_up_suh = sh.up.suh;     a.sh_up_svh = sh.up.svh;
    a.sh_down_tr = sh.down.trellis; a.sh_down_suh = sh.down.suh; a.sh_down_svh = sh.down.svh;
}

// Every row routed to expert 0 with score 1 (a shared expert through the tensor-core path).
__global__ void shared_route_kernel(uint32_t* inds, float* scores, int rows) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows) {
        inds[r] = 0u;
        scores[r] = 1.0f;
    }
}

}  // namespace

int three_per_sm_smem() {
    static int cached = 0;
    if (cached <= 0) {
        int dev = 0, per_sm = 0, reserve = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        cudaDeviceGetAttribute(&reserve, cudaDevAttrReservedSharedMemoryPerBlock, dev);
        cached = per_sm > 0 ? per_sm / 3 - reserve : 74 * 1024;
    }
    return cached;
}

int two_per_sm_smem() {
    static int cached = 0;
    if (cached <= 0) {
        int dev = 0, per_sm = 0, reserve = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        cudaDeviceGetAttribute(&reserve, cudaDevAttrReservedSharedMemoryPerBlock, dev);
        cached = per_sm > 0 ? per_sm / 2 - reserve : 112 * 1024;
    }
    return cached;
}

namespace {

// The least split-K cluster size of a chain kernel over `units` (work items x output blocks):
// enough CTAs to give every SM one; fit_split then grows it until two CTAs fit per SM.
#ifndef SX_CHAIN_CTAS_PER_SM
#define SX_CHAIN_CTAS_PER_SM 1
#endif
int min_split(long long units) {
    const long long want = (long long)sm_count() * SX_CHAIN_CTAS_PER_SM;
    const long long S = (want + std::max(1LL, units) - 1) / std::max(1LL, units);
    return (int)std::max(1LL, std::min(16LL, S));
}

// moe_pair's split over one row's items (the one-token chain, and an expert-parallel call whose
// places hold one row): the largest S <= 16 whose CTAs (units * S) all fit at three per SM and
// whose ranks all get input blocks (KB in chunks of ceil(KB / S)).  So few items still occupy
// every SM with two or three CTAs of short k ranges, and an SM that holds one CTA more carries
// less.  Measured on B200, 512 experts 2048/512, one token (11 items x 4 output blocks), the
// routed call in a loop of calls: S = 3 / 4 / 6 / 8 / 16 took 36.0 / 30.0 / 28.0 / 24.7 / 34.5 us
// (16: two waves).
int one_row_split(long long units, int KB) {
    const long long cap = (long long)sm_count() * 3;
    for (int S = 16; S > 1; S--) {
        const int chunk = (KB + S - 1) / S;
        if (units * S <= cap && (KB + chunk - 1) / chunk == S) return S;
    }
    return min_split(units);
}

// Direct items of an expert-parallel rank's call at most (a few tokens per rank: every received
// slot one item, most of them other ranks' sentinels that exit at once), and the down launch's
// items x output blocks at most: past that the dead items' CTAs cost more than the routing pass
// (measured at two GPUs: the 7168-wide DeepSeek layers at 8 tokens per rank, 7168 CTAs per
// group, took 20.7 ms per stack against 15.1 routed).
constexpr long long kDirectEpItems = 512;
constexpr long long kDirectEpCtas = 2048;

// The pair and down launches of the decode chain over `items` work items.
cudaError_t chain_launch(const MoeArgs& a, int kind, int n_gu, int n_d, int items, int active, cudaStream_t s,
                         bool one_row = false) {
    const int S_gu = one_row ? one_row_split((long long)active * (a.I / 128), a.D / 128)
                             : min_split((long long)active * (a.I / 128));
    const int S_d = min_split((long long)active * (a.D / 128));
    switch (kind) {
        case K_MCG: return moe_launch_kind<K_MCG>(a, n_gu, n_d, S_gu, S_d, items, s);
        case K_MUL1: return moe_launch_kind<K_MUL1>(a, n_gu, n_d, S_gu, S_d, items, s);
        case K_HASH: return moe_launch_kind<K_HASH>(a, n_gu, n_d, S_gu, S_d, items, s);
        case K_PAIR1: return moe_launch_kind<K_PAIR1>(a, n_gu, n_d, S_gu, S_d, items, s);
        default: return cudaErrorInvalidValue;
    }
}

// The one-token chain over W direct items (moe_pair, then moe_down1).
cudaError_t chain_launch_direct(const MoeArgs& a, int kind, int n_gu, int n_d, int W, cudaStream_t s) {
    const int S_gu = one_row_split((long long)W * (a.I / 128), a.D / 128);
    switch (kind) {
        case K_MCG: return moe_launch_kind_direct<K_MCG>(a, n_gu, n_d, S_gu, W, s);
        case K_MUL1: return moe_launch_kind_direct<K_MUL1>(a, n_gu, n_d, S_gu, W, s);
        case K_HASH: return moe_launch_kind_direct<K_HASH>(a, n_gu, n_d, S_gu, W, s);
        case K_PAIR1: return moe_launch_kind_direct<K_PAIR1>(a, n_gu, n_d, S_gu, W, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

}  // namespace sx

using namespace sx;

namespace sx {

// The valid slots a group can expect: its share of the layer's experts.
long long group_slots(long long slots, int rows, int topk, int Eg, int Etot) {
    const long long base = slots > 0 ? slots : (long long)rows * topk;
    return std::max(1LL, base * Eg / std::max(1, Etot));
}

size_t yslot_bytes(int rows, int topk, int D) { return align_up((size_t)rows * topk * D * sizeof(float)); }

bool same_decode(const sx_decode* a, const sx_decode* b) {
    return a == b || (a && b && a->codebook == b->codebook && a->window_bits == b->window_bits && a->table == b->table);
}

// How a layer's shared expert runs (moe_shared_fold.folded, src/moe_shared_fold.zig:24; fold_gated,
// src/exl3/fold_gated.zig:122-160, which serves one to eight rows): up to 16 rows, folded into the
// decode-chain launches of a routed group with its rates, decode and intermediate size (no launch
// of its own), else as its own pair and down launches of the chain (no routing pass); more rows
// through the tensor-core path with a routing of every row to it.  Each is the path a one-expert
// layer of those rows takes, so the arithmetic per row is the unfused composition's (its k split
// may differ).  Its output is the plane of slots rows*topk + row.
struct SharedPlan {
    int mode;   // 0 none, 1 folded into `group`, 2 chain launches of its own, 3 tensor-core path
    int group;
};

// sh_rows: the rows the shared expert runs over (the routed rows, or an expert-parallel rank's own
// rows when the routed ones are the rows it received).  any_decode: as if the decodes matched (the
// workspace query, which is asked without them).
SharedPlan shared_plan(const MoeGroup* g, int ng, int Etot, int rows, int topk, long long slots, const sx_bank* sh,
                       const sx_decode* dec, const sx_decode* sh_dec, int sh_rows, bool any_decode = false) {
    if (!sh) return {0, -1};
    const int D = g[0].bank.gate.in_features, I = g[0].bank.gate.out_features;
    for (int i = 0; i < ng; i++) {
        const sx_bank& b = g[i].bank;
        const MoeWs L = moe_ws_layout(b.gate.experts, rows, topk, D, I, b.gate.n, b.down.n,
                                      group_slots(slots, rows, topk, b.gate.experts, Etot), false);
        if (!L.gemm && sh_rows <= kDecodeRowsMax && sh->gate.n == b.gate.n && sh->down.n == b.down.n &&
            sh->gate.out_features == I && (any_decode || same_decode(dec, sh_dec)))
            return {1, i};
    }
    return {sh_rows <= kDecodeRowsMax ? 2 : 3, -1};
}

size_t shared_fill_bytes(int rows) { return align_up((size_t)rows * (sizeof(uint32_t) + sizeof(float))); }

// Workspace of a layer of groups: the per-slot planes first (every group writes its slots', and a
// shared expert its rows' past them), then the largest group's own scratch (the groups and the
// shared expert run one after another on the stream).
size_t moe_groups_ws(const MoeGroup* g, int ng, int Etot, int rows, int topk, long long slots, const sx_bank* sh,
                     const sx_decode* dec, const sx_decode* sh_dec, int sh_rows) {
    const int D = g[0].bank.gate.in_features, I = g[0].bank.gate.out_features;
    // The shared expert's scratch for the plan its rows and rates allow whichever decodes the call
    // brings: folded (the candidate group's extra prepared rows) and its own chain launches both.
    const SharedPlan plan = shared_plan(g, ng, Etot, rows, topk, slots, sh, dec, sh_dec, sh_rows, true);
    size_t most = 0;
    for (int i = 0; i < ng; i++) {
        const sx_bank& b = g[i].bank;
        const MoeWs L = moe_ws_layout(b.gate.experts, rows, topk, D, I, b.gate.n, b.down.n,
                                      group_slots(slots, rows, topk, b.gate.experts, Etot), false,
                                      plan.mode == 1 && plan.group == i ? sh_rows : 0);
        most = std::max(most, L.total);
    }
    if (plan.mode == 1 || plan.mode == 2)
        most = std::max(most, align_up((size_t)(rows * topk + sh_rows) * sh->gate.out_features * 2));
    if (plan.mode == 3) {
        const MoeWs L = moe_ws_layout(1, sh_rows, 1, D, sh->gate.out_features, sh->gate.n, sh->down.n, sh_rows, false);
        most = std::max(most, L.total + shared_fill_bytes(sh_rows));
    }
    return yslot_bytes(rows, topk, D) + (sh ? yslot_bytes(sh_rows, 1, D) : 0) + most;
}

size_t moe_groups_ws(const MoeGroup* g, int ng, int Etot, int rows, int topk, long long slots, const sx_bank* sh,
                     const sx_decode* dec, const sx_decode* sh_dec) {
    return moe_groups_ws(g, ng, Etot, rows, topk, slots, sh, dec, sh_dec, rows);
}

size_t moe_groups_ws(const MoeGroup* g, int ng, int Etot, int rows, int topk, long long slots) {
    return moe_groups_ws(g, ng, Etot, rows, topk, slots, nullptr, nullptr, nullptr, rows);
}

size_t moe_workspace_bytes(const sx_bank* bank, int32_t rows, int32_t topk, long long slots) {
    if (!bank || rows < 1 || topk < 1) return 0;
    const MoeGroup g{*bank, 0};
    return moe_groups_ws(&g, 1, bank->gate.experts, rows, topk, slots);
}

// Route metadata and the decode chain or the tensor-core path for one group's slots, into yslot.
// fold: a shared expert riding this group's decode-chain launches (shared_plan mode 1), or null.
sx_status moe_group(sx_stream stream, const sx_bank* bank, int e_lo, const sx_decode* dec, const void* x,
                    sx_dtype dtype, int32_t rows, const uint32_t* inds, const float* scores, int32_t topk,
                    int32_t clamp_limit, float* yslot, uint8_t* ws, long long slots, const sx_bank* fold = nullptr,
                    const MoeSegments* seg = nullptr, const MoeArgs* reduce = nullptr, bool* reduced = nullptr,
                    const SharedRows* fold_rows = nullptr) {
    const int E = bank->gate.experts;
    const int D = bank->gate.in_features, I = bank->gate.out_features;
    sx_status st;
    const int sh_rows = fold_rows ? fold_rows->rows : rows;
    const MoeWs L = moe_ws_layout(E, rows, topk, D, I, bank->gate.n, bank->down.n, slots, false, fold ? sh_rows : 0,
                                  seg ? seg->live_slots : -1);
    MoeArgs a{};
    int kind_gu, kind_d;
    if ((st = resolve_decode(dec, bank->gate.n, &kind_gu, &a.dp_gu))) return st;
    if ((st = resolve_decode(dec, bank->down.n, &kind_d, &a.dp_down))) return st;
    a.x = x;
    a.xdt = dtype;
    a.R = rows;
    a.K = topk;
    a.D = D;
    a.I = I;
    a.E = E;
    a.inds = inds;
    a.scores = scores;
    a.gate_tr = bank->gate.trellis; a.gate_suh = bank->gate.suh; a.gate_svh = bank->gate.svh;
    a.up_tr = bank->up.trellis;     a.up_suh = bank->up.suh;     a.up_svh = bank->up.svh;
    a.down_tr = bank->down.trellis; a.down_suh = bank->down.suh; a.down_svh = bank->down.svh;
    a.scale_gu = kind_scale(kind_gu);
    a.scale_down = kind_scale(kind_d);
    a.clamp = (float)clamp_limit;
    a.meta = reinterpret_cast<int*>(ws + L.meta);
    a.act_expert = reinterpret_cast<int*>(ws + L.act_expert);
    a.act_start = reinterpret_cast<int*>(ws + L.act_start);
    a.act_count = reinterpret_cast<int*>(ws + L.act_count);
    a.work_act = reinterpret_cast<int*>(ws + L.work_act);
    a.work_chunk = reinterpret_cast<int*>(ws + L.work_chunk);
    a.order = reinterpret_cast<int*>(ws + L.order);
    a.hprep = reinterpret_cast<uint16_t*>(ws + L.hprep);
    a.yslot = yslot;
    a.e_lo = e_lo;
    a.chunk = L.chunk;
    a.big_min = L.big_min;
    a.big_chunk = L.big_chunk;
    a.work_act4 = reinterpret_cast<int*>(ws + L.work_act4);
    a.work_chunk4 = reinterpret_cast<int*>(ws + L.work_chunk4);
    a.sorted_e = reinterpret_cast<int*>(ws + L.sorted_e);
    a.work_rec = reinterpret_cast<int4*>(ws + L.work_rec);
    a.work_slots = reinterpret_cast<int*>(ws + L.work_slots);
    a.w_routed = L.W_max;
    if (seg) {
        a.seg_cnt = seg->cnt;
        a.seg_cap = seg->cap;
        a.nseg = seg->n;
        a.seg_wait = seg->wait_flags;
        a.seg_seq = seg->seq;
    }
    a.sh_x = fold_rows ? fold_rows->x : x;
    a.sh_rows = sh_rows;
    if (fold) {
        a.sh_items = (sh_rows + L.chunk - 1) / L.chunk;
        a.sh_slot0 = rows * topk;
        set_shared_ptrs(a, *fold);
    }

    if (reduce && !L.gemm) {  // the layer's reduce rides moe_down (see MoeArgs::rcount)
        a.rcount = reinterpret_cast<int*>(ws + L.rcount);
        a.shared = reduce->shared;
        a.shared_gate = reduce->shared_gate;
        a.y = reduce->y;
        a.sh_plane = reduce->sh_plane;
        a.sh_slot0 = rows * topk;
        if (reduced) *reduced = true;
    }

    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    // One token on the decode chain with the reduce folded (one group, no expert-parallel
    // segments, at most 16 items): the token's slots are the work items, so no routing pass runs,
    // and moe_down1 reduces over a cluster of the items.
    // An expert-parallel rank's small call (launches sized for every place, no host-read counts):
    // every received slot is a direct item (dead ones exit at once), no routing pass; moe_down
    // writes the per-slot planes the rank's reduce reads.  The k splits are the ones the routed
    // chain would take (its active items and chunk), so the per-slot arithmetic is the same: a
    // world of one gives sx_moe's bits.
    const long long ep_items = (long long)rows * topk + (fold ? sh_rows : 0);
    if (seg && seg->wait_flags && !reduce && !L.gemm && ep_items <= kDirectEpItems &&
        ep_items * (D / 128) <= kDirectEpCtas) {
        const int routed_active = L.A_max + a.sh_items;
        a.split_chunk = a.chunk;
        a.direct = 1;
        a.chunk = 1;
        a.w_routed = rows * topk;
        a.sh_items = fold ? sh_rows : 0;
        a.sh_slot0 = rows * topk;
        e = chain_launch(a, kind_gu, bank->gate.n, bank->down.n, (int)ep_items, routed_active, s, rows == 1);
        return e == cudaSuccess ? SX_OK : cuda_status(e, "moe expert-parallel direct chain launch");
    }
    const int direct_items = topk + (fold ? 1 : 0);
    if (rows == 1 && a.rcount && !seg && !fold_rows && direct_items <= 16) {
        a.direct = 1;
        a.chunk = 1;
        a.w_routed = topk;
        a.sh_items = fold ? 1 : 0;
        a.sh_slot0 = topk;
        a.rcount = nullptr;
        e = chain_launch_direct(a, kind_gu, bank->gate.n, bank->down.n, direct_items, s);
        return e == cudaSuccess ? SX_OK : cuda_status(e, "moe one-token chain launch");
    }
    const size_t rp_smem = 3 * (size_t)E * sizeof(int);
    if (rp_smem > 48 * 1024) e = func_attrs((const void*)route_prep_kernel, (int)rp_smem, false);
    if (e == cudaSuccess) e = launch_pdl(route_prep_kernel, dim3(1), dim3(1024), rp_smem, s, a);
    if (e != cudaSuccess) return cuda_status(e, "route_prep launch");
    if (L.gemm) {
        // Tensor-core path (kernels.moePrefill, src/exl3/expert_exl3_kernels.zig:2861): prepared
        // gate/up inputs per sorted position, the gate and up GEMMs, the mid, the down GEMM into the
        // per-slot planes; the same k-order reduce as the decode chain.
        // the prep kernel reads x rows and the suh rows as vectors; TMA reads the workspace
        if (reinterpret_cast<uintptr_t>(ws) % 16 || reinterpret_cast<uintptr_t>(x) % 16 ||
            reinterpret_cast<uintptr_t>(bank->gate.suh) % 8 || reinterpret_cast<uintptr_t>(bank->up.suh) % 8)
            return SX_ERR_BAD_SHAPE;
        a.tg = reinterpret_cast<uint16_t*>(ws + L.tg);
        a.tu = reinterpret_cast<uint16_t*>(ws + L.tu);
        a.gf = reinterpret_cast<float*>(ws + L.gf);
        a.uf = reinterpret_cast<float*>(ws + L.uf);
        const int RK = seg && seg->live_slots >= 0 ? (int)std::min<long long>(seg->live_slots, (long long)rows * topk)
                                                   : rows * topk;  // sorted positions at most
        const dim3 pos_grid(std::max(1, (RK + 7) / 8), 1);  // positions past meta[2] return
        moe_prep_kernel<<<dim3(pos_grid.x, D / 128), 256, 0, s>>>(a);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "moe prep launch");
        CUtensorMap mg, mu, mh;
        if ((e = prep_map(&mg, a.tg, RK, D, kGemmRows)) != cudaSuccess ||
            (e = prep_map(&mu, a.tu, RK, D, kGemmRows)) != cudaSuccess ||
            (e = prep_map(&mh, a.hprep, RK, I, kGemmRows)) != cudaSuccess)
            return cuda_status(e, "cuTensorMapEncodeTiled");
        // two launches per projection: list 1 (chunks of 128 rows, one row tile per CTA) and list 2
        // (chunks of 512 rows of the experts with many rows, four row tiles per CTA)
        auto both = [&](GemmArgs g, int kind, const CUtensorMap& m, int n, int out_blocks, int chunks) -> cudaError_t {
            g.meta = a.meta;
            g.work_act = a.work_act;
            g.work_chunk = a.work_chunk;
            const int S = gemm_split((long long)L.A_max * out_blocks, chunks);
            cudaError_t r = gemm_launch(kind, m, g, n, 1, L.W_max, S, s);
            if (r != cudaSuccess || L.W4_max == 0) return r;
            g.meta = a.meta + 1;
            g.work_act = a.work_act4;
            g.work_chunk = a.work_chunk4;
            return gemm_launch(kind, m, g, n, 4, L.W4_max, 1, s, out_blocks % 2 == 0);
        };
        GemmArgs g{};
        g.rows = 0;
        g.act_expert = a.act_expert;
        g.act_start = a.act_start;
        g.act_count = a.act_count;
        g.mode = GEMM_OUT_F32;
        g.in = D;
        g.out = I;
        g.dp = a.dp_gu;
        g.scale = a.scale_gu;
        const struct { const sx_proj* p; float* out; const CUtensorMap* m; } gu[2] = {{&bank->gate, a.gf, &mg},
                                                                                        {&bank->up, a.uf, &mu}};
        for (const auto& q : gu) {
            g.trellis = q.p->trellis;
            g.tr_expert = (size_t)(D / 16) * (I / 16) * q.p->n;
            g.svh = q.p->svh;
            g.yf = q.out;
            if ((e = both(g, kind_gu, *q.m, q.p->n, I / 128, D / kGemmKC)) != cudaSuccess)
                return cuda_status(e, "moe gate/up gemm launch");
        }
        moe_mid_kernel<<<dim3(pos_grid.x, I / 128), 256, 0, s>>>(a);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "moe mid launch");
        g.mode = GEMM_OUT_SLOT;
        g.in = I;
        g.out = D;
        g.dp = a.dp_down;
        g.scale = a.scale_down;
        g.trellis = bank->down.trellis;
        g.tr_expert = (size_t)(I / 16) * (D / 16) * bank->down.n;
        g.svh = bank->down.svh;
        g.yf = a.yslot;
        g.order = a.order;
        g.scores = a.scores;
        if ((e = both(g, kind_d, mh, bank->down.n, D / 128, I / kGemmKC)) != cudaSuccess)
            return cuda_status(e, "moe down gemm launch");
        return SX_OK;
    }
    e = chain_launch(a, kind_gu, bank->gate.n, bank->down.n, L.W_max + a.sh_items, L.A_max + a.sh_items, s);
    if (e != cudaSuccess) return cuda_status(e, "moe pair/down launch");
    return SX_OK;
}

// A shared expert's own decode-chain launches (shared_plan mode 2): every work item is one of its
// 8-row chunks; no routing metadata.  hprep holds rows*topk + rows prepared rows.
sx_status shared_chain(sx_stream stream, const sx_bank* sh, const sx_decode* dec, const void* x, sx_dtype dtype,
                       int32_t rows, int32_t slot0, int32_t clamp_limit, float* yslot, uint8_t* ws) {
    MoeArgs a{};
    int kind_gu, kind_d;
    sx_status st;
    if ((st = resolve_decode(dec, sh->gate.n, &kind_gu, &a.dp_gu))) return st;
    if ((st = resolve_decode(dec, sh->down.n, &kind_d, &a.dp_down))) return st;
    a.x = x;
    a.xdt = dtype;
    a.R = rows;
    a.K = 1;
    a.D = sh->gate.in_features;
    a.I = sh->gate.out_features;
    a.E = 1;
    a.sh_x = x;
    a.sh_rows = rows;
    a.scale_gu = kind_scale(kind_gu);
    a.scale_down = kind_scale(kind_d);
    a.clamp = (float)clamp_limit;
    a.hprep = reinterpret_cast<uint16_t*>(ws);
    a.yslot = yslot;
    a.w_routed = 0;
    a.chunk = rows <= kSmallChunk ? kSmallChunk : 8;
    a.sh_items = (rows + a.chunk - 1) / a.chunk;
    a.sh_slot0 = slot0;
    set_shared_ptrs(a, *sh);
    const cudaError_t e = chain_launch(a, kind_gu, sh->gate.n, sh->down.n, a.sh_items, a.sh_items,
                                       reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SX_OK : cuda_status(e, "shared expert pair/down launch");
}

// The shared expert of a layer: one SwiGLU expert over the layer's hidden size, rates the
// decode serves (validateClampedProjection for each projection, src/exl3/root.zig:117-135).
sx_status check_shared_bank(const sx_bank* sh, int D, const sx_decode* dec) {
    sx_status st;
    if (!sh) return SX_ERR_NULL_POINTER;
    if ((st = check_proj(&sh->gate, 1)) || (st = check_proj(&sh->up, 1)) || (st = check_proj(&sh->down, 1))) return st;
    const int Is = sh->gate.out_features;
    if (sh->gate.in_features != D || sh->up.in_features != D || sh->up.out_features != Is ||
        sh->down.in_features != Is || sh->down.out_features != D)
        return SX_ERR_BAD_SHAPE;
    if (sh->gate.tile_order != SX_TILE_PACK || sh->up.tile_order != SX_TILE_PACK || sh->down.tile_order != SX_TILE_PACK)
        return SX_ERR_TILE_ORDER_UNSUPPORTED;
    if (sh->gate.n != sh->up.n) return SX_ERR_TRELLIS_GEOMETRY;
    int kind;
    DecParams dp;
    if ((st = resolve_decode(dec, sh->gate.n, &kind, &dp)) || (st = resolve_decode(dec, sh->down.n, &kind, &dp)))
        return st;
    return SX_OK;
}

size_t shared_expert_ws(const sx_bank* sh, int rows) {
    const int D = sh->gate.in_features, Is = sh->gate.out_features;
    if (rows <= kDecodeRowsMax) return align_up((size_t)rows * Is * sizeof(uint16_t));
    return moe_ws_layout(1, rows, 1, D, Is, sh->gate.n, sh->down.n, rows, false).total + shared_fill_bytes(rows);
}

// The shared expert alone over `rows` rows into plane [rows][D] (f32, before rounding): its own
// decode-chain launches up to 16 rows, else the tensor-core path with every row routed to it.
sx_status shared_expert_run(sx_stream stream, const sx_bank* sh, const sx_decode* dec, const void* x, sx_dtype dtype,
                            int32_t rows, int32_t clamp_limit, float* plane, uint8_t* scratch) {
    if (rows <= kDecodeRowsMax) return shared_chain(stream, sh, dec, x, dtype, rows, 0, clamp_limit, plane, scratch);
    const MoeWs L = moe_ws_layout(1, rows, 1, sh->gate.in_features, sh->gate.out_features, sh->gate.n, sh->down.n, rows,
                                  false);
    uint32_t* sh_inds = reinterpret_cast<uint32_t*>(scratch + L.total);
    float* sh_scores = reinterpret_cast<float*>(sh_inds + rows);
    shared_route_kernel<<<(rows + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(sh_inds, sh_scores, rows);
    const sx_status st = cuda_status(cudaGetLastError(), "shared route launch");
    if (st) return st;
    return moe_group(stream, sh, 0, dec, x, dtype, rows, sh_inds, sh_scores, 1, clamp_limit, plane, scratch, rows);
}

// A routed layer of groups: every group's chain into the per-slot planes, then the k-order reduce
// over all slots (rounding, shared expert; or an expert-parallel rank's f32 partial).
sx_status moe_run(sx_stream stream, const MoeGroup* groups, int ng, int Etot, const sx_decode* dec, const void* x,
                  sx_dtype dtype, int32_t rows, const uint32_t* inds, const float* scores, int32_t topk,
                  const void* shared, const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                  size_t workspace_bytes, float* partial, long long slots, const sx_bank* sh_bank,
                  const sx_decode* sh_dec, const MoeSegments* seg, float** yslot_out, const SharedRows* own) {
    if (!x || !inds || !scores || (!y && !partial && !yslot_out)) return SX_ERR_NULL_POINTER;
    if (clamp_limit < 0 || clamp_limit > 128) return SX_ERR_INVALID_CLAMP;
    if (rows < 1 || topk < 1) return SX_ERR_BAD_SHAPE;
    if (topk > 32) return SX_ERR_TOPK_EXCEEDS_REDUCE_BANK;
    if (!dtype_ok(dtype)) return SX_ERR_BAD_DTYPE;
    if (shared_gate && !shared && !sh_bank) return SX_ERR_NULL_POINTER;
    // (an expert-parallel rank's rows carry every slot, most of them other ranks' sentinels)
    if (topk > Etot && !partial && !yslot_out) return SX_ERR_TOPK_EXCEEDS_EXPERTS;
    if (Etot > 8192) return SX_ERR_BAD_SHAPE;
    const int D = groups[0].bank.gate.in_features, I = groups[0].bank.gate.out_features;
    for (int i = 0; i < ng; i++) {
        // validateClampedProjection for gate, up and down (src/exl3/root.zig:117-135).
        const sx_bank* bank = &groups[i].bank;
        const int E = bank->gate.experts;
        sx_status st;
        if ((st = check_proj(&bank->gate, E)) || (st = check_proj(&bank->up, E)) || (st = check_proj(&bank->down, E)))
            return st;
        if (bank->gate.in_features != D || bank->gate.out_features != I || bank->up.in_features != D ||
            bank->up.out_features != I || bank->down.in_features != I || bank->down.out_features != D)
            return SX_ERR_BAD_SHAPE;
        if (bank->gate.tile_order != SX_TILE_PACK || bank->up.tile_order != SX_TILE_PACK ||
            bank->down.tile_order != SX_TILE_PACK)
            return SX_ERR_TILE_ORDER_UNSUPPORTED;
        if (bank->gate.n != bank->up.n) return SX_ERR_TRELLIS_GEOMETRY;  // mixed gate/up rates: not served yet
        int kind;
        DecParams dp;
        if ((st = resolve_decode(dec, bank->gate.n, &kind, &dp)) || (st = resolve_decode(dec, bank->down.n, &kind, &dp)))
            return st;
    }
    if (sh_bank) {
        if (shared || partial) return SX_ERR_BAD_SHAPE;
        const sx_status st = check_shared_bank(sh_bank, D, sh_dec);
        if (st) return st;
    }
    const int sh_rows = own ? own->rows : rows;
    const void* sh_x = own ? own->x : x;
    if (sh_bank && sh_rows < 1) return SX_ERR_BAD_SHAPE;
    if (!workspace ||
        workspace_bytes < moe_groups_ws(groups, ng, Etot, rows, topk, slots, sh_bank, dec, sh_dec, sh_rows))
        return SX_ERR_WORKSPACE_TOO_SMALL;
    const SharedPlan plan = shared_plan(groups, ng, Etot, rows, topk, slots, sh_bank, dec, sh_dec, sh_rows);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* yslot = reinterpret_cast<float*>(ws);
    uint8_t* scratch = ws + yslot_bytes(rows, topk, D) + (sh_bank ? yslot_bytes(sh_rows, 1, D) : 0);
    MoeArgs r{};
    r.inds = inds;
    r.K = topk;
    r.D = D;
    r.E = Etot;
    r.xdt = dtype;
    r.yslot = yslot;
    r.shared = shared;
    r.shared_gate = shared_gate;
    r.y = y;
    r.partial = partial;
    r.sh_plane = sh_bank != nullptr;
    r.sh_slot0 = rows * topk;
    // One group whose every plane comes from its own decode-chain launches (no shared expert, or
    // one folded into them): the reduce rides its moe_down.  (Which path the group takes is its
    // own choice: moe_group says whether it folded.)
    const bool may_fold = ng == 1 && !partial && !yslot_out && y && (plan.mode == 0 || plan.mode == 1);
    bool folded = false;
    for (int i = 0; i < ng; i++) {
        const sx_status st = moe_group(stream, &groups[i].bank, groups[i].e_lo, dec, x, dtype, rows, inds, scores, topk,
                                       clamp_limit, yslot, scratch,
                                       group_slots(slots, rows, topk, groups[i].bank.gate.experts, Etot),
                                       plan.mode == 1 && plan.group == i ? sh_bank : nullptr, seg,
                                       may_fold ? &r : nullptr, &folded, own);
        if (st) return st;
    }
    if (plan.mode == 2) {
        const sx_status st = shared_chain(stream, sh_bank, sh_dec, sh_x, dtype, sh_rows, rows * topk, clamp_limit,
                                          yslot, scratch);
        if (st) return st;
    } else if (plan.mode == 3) {
        const sx_status st = shared_expert_run(stream, sh_bank, sh_dec, sh_x, dtype, sh_rows, clamp_limit,
                                               yslot + (size_t)rows * topk * D, scratch);
        if (st) return st;
    }
    if (yslot_out) {  // the caller reduces the per-slot planes itself (the shared plane follows them)
        *yslot_out = yslot;
        return SX_OK;
    }
    if (folded) return SX_OK;
    return cuda_status(launch_pdl(moe_reduce_kernel, dim3(rows, (D + kReduceCols - 1) / kReduceCols), dim3(128), 0,
                                  reinterpret_cast<cudaStream_t>(stream), r),
                       "moe reduce launch");
}

sx_status moe_impl(sx_stream stream, const sx_bank* bank, const sx_decode* dec, const void* x, sx_dtype dtype,
                   int32_t rows, const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                   const void* shared_gate, int32_t clamp_limit, void* y, void* workspace, size_t workspace_bytes,
                   float* partial, long long slots) {
    if (!bank) return SX_ERR_NULL_POINTER;
    const MoeGroup g{*bank, 0};
    return moe_run(stream, &g, 1, bank->gate.experts, dec, x, dtype, rows, inds, scores, topk, shared, shared_gate,
                   clamp_limit, y, workspace, workspace_bytes, partial, slots, nullptr, nullptr, nullptr, nullptr,
                   nullptr);
}

}  // namespace sx

extern "C" size_t sx_moe_workspace_bytes(const sx_bank* bank, int32_t rows, int32_t topk) {
    return moe_workspace_bytes(bank, rows, topk, 0);
}

extern "C" sx_status sx_moe(sx_stream stream, const sx_bank* bank, const sx_decode* dec, const void* x, sx_dtype dtype,
                            int32_t rows, const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                            const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                            size_t workspace_bytes) {
    return moe_impl(stream, bank, dec, x, dtype, rows, inds, scores, topk, shared, shared_gate, clamp_limit, y,
                    workspace, workspace_bytes, nullptr, 0);
}

namespace sx {

constexpr int kMetaWords = 8;  // rate_groups.META_WORDS (src/exl3/rate_groups.zig:25)

// The groups of a ragged layer from its host meta table: runs of consecutive experts with one group
// id, one rate per projection, and tiles at the stride of that rate.
sx_status ragged_groups(const sx_ragged* rb, MoeGroup* out, int* ng) {
    if (!rb || !rb->meta) return SX_ERR_NULL_POINTER;
    if (rb->experts < 1 || rb->hidden <= 0 || rb->inter <= 0 || rb->hidden % 128 || rb->inter % 128)
        return SX_ERR_BAD_SHAPE;
    for (int p = 0; p < 3; p++)
        if (!rb->trellis[p] || !rb->suh[p] || !rb->svh[p]) return SX_ERR_NULL_POINTER;
    const uint64_t tiles = (uint64_t)(rb->hidden / 16) * (rb->inter / 16);
    int n = 0;
    for (int e = 0; e < rb->experts;) {
        const uint32_t* m = rb->meta + (size_t)e * kMetaWords;
        if (n == kMaxGroups || m[7] != 0) return SX_ERR_GROUP_GEOMETRY;
        int len = 1;
        for (; e + len < rb->experts; len++) {
            const uint32_t* q = rb->meta + (size_t)(e + len) * kMetaWords;
            if (q[3] != m[3]) break;
            if (q[0] != m[0] || q[1] != m[1] || q[2] != m[2] || q[7] != (uint32_t)len) return SX_ERR_GROUP_GEOMETRY;
            for (int p = 0; p < 3; p++)
                if ((uint64_t)q[4 + p] != (uint64_t)m[4 + p] + (uint64_t)len * tiles * m[p] / 2) return SX_ERR_GROUP_GEOMETRY;
        }
        MoeGroup& g = out[n++];
        g.e_lo = e;
        sx_proj* pr[3] = {&g.bank.gate, &g.bank.up, &g.bank.down};
        for (int p = 0; p < 3; p++) {
            pr[p]->trellis = rb->trellis[p] + (size_t)m[4 + p] * 2;
            pr[p]->suh = rb->suh[p] + (size_t)e * (p == 2 ? rb->inter : rb->hidden);
            pr[p]->svh = rb->svh[p] + (size_t)e * (p == 2 ? rb->hidden : rb->inter);
            pr[p]->experts = len;
            pr[p]->in_features = p == 2 ? rb->inter : rb->hidden;
            pr[p]->out_features = p == 2 ? rb->hidden : rb->inter;
            pr[p]->n = (int32_t)m[p];
            pr[p]->tile_order = SX_TILE_PACK;
        }
        e += len;
    }
    *ng = n;
    return SX_OK;
}

}  // namespace sx

extern "C" size_t sx_moe_ragged_workspace_bytes(const sx_ragged* bank, int32_t rows, int32_t topk) {
    MoeGroup g[kMaxGroups];
    int ng = 0;
    if (rows < 1 || topk < 1 || ragged_groups(bank, g, &ng) != SX_OK) return 0;
    return moe_groups_ws(g, ng, bank->experts, rows, topk, 0);
}

extern "C" sx_status sx_moe_ragged(sx_stream stream, const sx_ragged* bank, const sx_decode* dec, const void* x,
                                   sx_dtype dtype, int32_t rows, const uint32_t* inds, const float* scores, int32_t topk,
                                   const void* shared, const void* shared_gate, int32_t clamp_limit, void* y,
                                   void* workspace, size_t workspace_bytes) {
    MoeGroup g[kMaxGroups];
    int ng = 0;
    const sx_status st = ragged_groups(bank, g, &ng);
    if (st) return st;
    return moe_run(stream, g, ng, bank->experts, dec, x, dtype, rows, inds, scores, topk, shared, shared_gate,
                   clamp_limit, y, workspace, workspace_bytes, nullptr, 0, nullptr, nullptr);
}

extern "C" size_t sx_moe_folded_workspace_bytes(const sx_bank* bank, const sx_bank* shared_bank,
                                                const sx_decode* dec, const sx_decode* shared_dec, int32_t rows,
                                                int32_t topk) {
    if (!bank || !shared_bank || rows < 1 || topk < 1) return 0;
    const MoeGroup g{*bank, 0};
    return moe_groups_ws(&g, 1, bank->gate.experts, rows, topk, 0, shared_bank, dec, shared_dec ? shared_dec : dec);
}

extern "C" sx_status sx_moe_folded(sx_stream stream, const sx_bank* bank, const sx_bank* shared_bank,
                                   const sx_decode* dec, const sx_decode* shared_dec, const void* x, sx_dtype dtype,
                                   int32_t rows, const uint32_t* inds, const float* scores, int32_t topk,
                                   const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                                   size_t workspace_bytes) {
    if (!bank || !shared_bank) return SX_ERR_NULL_POINTER;
    const MoeGroup g{*bank, 0};
    return moe_run(stream, &g, 1, bank->gate.experts, dec, x, dtype, rows, inds, scores, topk, nullptr, shared_gate,
                   clamp_limit, y, workspace, workspace_bytes, nullptr, 0, shared_bank, shared_dec ? shared_dec : dec);
}

extern "C" size_t sx_moe_ragged_folded_workspace_bytes(const sx_ragged* bank, const sx_bank* shared_bank,
                                                       const sx_decode* dec, const sx_decode* shared_dec, int32_t rows,
                                                       int32_t topk) {
    MoeGroup g[kMaxGroups];
    int ng = 0;
    if (!shared_bank || rows < 1 || topk < 1 || ragged_groups(bank, g, &ng) != SX_OK) return 0;
    return moe_groups_ws(g, ng, bank->experts, rows, topk, 0, shared_bank, dec, shared_dec ? shared_dec : dec);
}

extern "C" sx_status sx_moe_ragged_folded(sx_stream stream, const sx_ragged* bank, const sx_bank* shared_bank,
                                          const sx_decode* dec, const sx_decode* shared_dec, const void* x,
                                          sx_dtype dtype, int32_t rows, const uint32_t* inds, const float* scores,
                                          int32_t topk, const void* shared_gate, int32_t clamp_limit, void* y,
                                          void* workspace, size_t workspace_bytes) {
    if (!shared_bank) return SX_ERR_NULL_POINTER;
    MoeGroup g[kMaxGroups];
    int ng = 0;
    const sx_status st = ragged_groups(bank, g, &ng);
    if (st) return st;
    return moe_run(stream, g, ng, bank->experts, dec, x, dtype, rows, inds, scores, topk, nullptr, shared_gate,
                   clamp_limit, y, workspace, workspace_bytes, nullptr, 0, shared_bank, shared_dec ? shared_dec : dec);
}
