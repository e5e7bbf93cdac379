// Tensor-core EXL3 projection for many rows (kernel template; instantiated per codebook in
// sx_gemm_{mcg,mul1,hash,pair1}.cu): the reference's sorted-window GEMM (src/exl3/linear.zig:365,
// kernels.moePrefill src/exl3/expert_exl3_kernels.zig:2861, innerGemmSortedTable* :1379-1408)
// rebuilt on tcgen05.
//
//   D[o][t] = sum_k W[k][o] * P[t][k]      (o: 128 outputs of a block, t: NT rows, k: inputs)
//
// * A = the weights, M = 128 outputs: 16 decoder warps decode each 64-input chunk's 32 trellis
//   tiles (streamed into shared memory by 1-D bulk copies) into f16 with the reference's
//   rounding (the f16 sum of the codebook's two halves, or MUL1's f16 fma: the bit-exact inner
//   weights of sx_dequant_inner) and store them as a K-major, 128-byte-swizzled tile.
// * B = the prepared rows P = f16(H128(f16(x) * suh)), N = NT rows: a 2-D TMA tile (128-byte
//   swizzle) from a [rows, in] f16 matrix that a prep kernel wrote.  Rows past the matrix read 0.
// * One thread issues tcgen05.mma kind::f16 (f16 x f16 -> f32 in tensor memory) per 16-input
//   step and commits each stage's completion to the stage's empty barrier.
// * Split-K: the CTAs of a cluster (grid z) take contiguous input ranges; every CTA moves its
//   accumulator from tensor memory to shared memory and the rank-0 CTA sums the cluster's
//   partials over DSMEM in rank order, applies H128, svh and the codebook scale, and writes.
// Every wait is bounded (sx_common.cuh); a timed-out CTA skips its work, reaches every barrier
// and frees its tensor memory.
#pragma once

#include <cuda.h>

#include "sx_core.cuh"

namespace sx {

constexpr int kGemmDecWarps = 16;                       // decoders, then the epilogue
constexpr int kGemmThreads = (kGemmDecWarps + 2) * 32;  // + producer warp + MMA warp
constexpr int kGemmKC = 64;                             // inputs per stage (one 128-byte swizzle row)
constexpr int kGemmRows = 128;                          // NT: rows per CTA tile (the MMA's N)
constexpr int kGemmRowsNarrow = 16;                     // NT of a dense call of at most 16 rows

enum GemmMode : int {
    GEMM_OUT_ACT = 0,   // y[row][o] in the activation dtype
    GEMM_OUT_F32 = 1,   // yf[row][o] f32
    GEMM_OUT_SLOT = 2,  // yf[order[row]][o] = value * scores[order[row]] (f32 per routed slot)
};

struct GemmArgs {
    const uint16_t* trellis;   // expert 0's [in/16][out/16][n]
    size_t tr_expert;          // elements between experts
    const uint16_t* svh;       // [E][out]
    int in, out;
    DecParams dp;
    float scale;               // the codebook's output scale
    // rows: dense (rows > 0) or the routed work list of sx_moe's route_prep (chunks of NT rows)
    int rows;
    const int* meta;           // [0] = work items
    const int* act_expert;
    const int* act_start;
    const int* act_count;
    const int* work_act;
    const int* work_chunk;
    // output
    int mode;
    void* y;                   // GEMM_OUT_ACT
    int ydt;
    float* yf;                 // GEMM_OUT_F32 / GEMM_OUT_SLOT
    const int* order;          // GEMM_OUT_SLOT: sorted position -> slot
    const float* scores;       // GEMM_OUT_SLOT: [slots]
};

// RT row tiles of NT rows per CTA share each decoded weight chunk: RT accumulators of NT columns
// in tensor memory (RT * NT <= 512), RT prepared-row tiles per stage.
// PAIR: a CTA pair (cta_group::2) shares the four row tiles; each CTA holds half of each 256-row
// block's prepared rows, so it loads two 16 KB tiles per stage and the ring is four deep.
template <int N, int NT, int RT, bool PAIR = false>
struct GemmLayout {
    static constexpr int A_BYTES = 128 * kGemmKC * 2;   // 16 KB
    static constexpr int B_TILE = NT * kGemmKC * 2;     // 16 KB per row tile
    static constexpr int B_BYTES = (PAIR ? RT / 2 : RT) * B_TILE;
    static constexpr int T_BYTES = 4 * 8 * N * 2;       // 32 trellis tiles
    // One row tile: as many stages as fit in 223 KB (5 or 6 at 128 rows, 10 or 11 at 16; at most
    // 12), since a stage's cycle (copies, decode, MMA, commit) is longer than its decode and only
    // the ring depth hides it.
    static constexpr int STAGE1 = 128 * kGemmKC * 2 + NT * kGemmKC * 2 + 4 * 8 * N * 2;
    static constexpr int NST1 = (223 * 1024) / STAGE1 < 12 ? (223 * 1024) / STAGE1 : 12;
    static constexpr int NST = PAIR ? 4 : (RT == 1 ? NST1 : (RT == 2 ? 3 : 2));
    static constexpr int TMEM_COLS = NT * RT < 32 ? 32 : NT * RT;  // an allocation is 32 columns at least
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + NST * A_BYTES;
    static constexpr int T_OFF = B_OFF + NST * B_BYTES;
    static constexpr int BAR_OFF = (T_OFF + NST * T_BYTES + 15) / 16 * 16;
    static constexpr int TOTAL = BAR_OFF + (5 * NST + 1) * 8 + 16;
    // one row tile's accumulator in f32, reusing A and B (32 rows at least: the epilogue moves
    // tensor memory out 32 columns at a time)
    static constexpr int RED_BYTES = (NT < 32 ? 32 : NT) * 128 * 4;
    static_assert(RED_BYTES <= T_OFF, "accumulator staging fits in the A/B ring");
    static_assert(TMEM_COLS <= 512, "tensor memory holds 512 columns");
    static_assert(!PAIR || RT == 4, "the pair kernel holds two 256-row blocks");
    static constexpr int ALLOC = TOTAL + 1024;          // room to align the base to 1024 bytes
};

// ------------------------------------------------------------------ tcgen05 / TMA helpers
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;                // leading byte offset (unused for swizzled K-major): 16 B
    d |= (uint64_t)(1024u >> 4) << 32;      // stride byte offset: 1024 B between 8-row groups
    d |= (uint64_t)1u << 46;                // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;                // SWIZZLE_128B
    return d;
}

// Instruction descriptor: f16 A and B, f32 D, both K-major, M = 128, N = nt.
__host__ __device__ constexpr uint32_t idesc_f16_m128(int nt) {
    return (1u << 4) | ((uint32_t)(nt >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// M = 256 over a CTA pair (cta_group::2): each CTA supplies 128 rows of A and half of B's N rows.
__host__ __device__ constexpr uint32_t idesc_f16_m256(int nt) {
    return (1u << 4) | ((uint32_t)(nt >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

__device__ __forceinline__ void tc_mma2_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Completion of this thread's pair MMAs, arriving on the barrier at the same offset in both CTAs.
__device__ __forceinline__ void tc_commit2(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}

// Arrive (release at cluster scope) on the barrier at the same offset in cluster CTA `rank`.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* bar, uint32_t rank) {
    asm volatile(
        "{\n\t.reg .b32 ra;\n\t"
        "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
        "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
        "r"(rank)
        : "memory");
}

// mbar_wait with acquire at cluster scope (arrivals from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int code) {
    auto try_once = [&]() {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        return ok != 0;
    };
    if (try_once()) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0;; i++) {
        if (try_once()) return true;
        if ((i & 255u) == 255u && global_timer_ns() - t0 > kWaitLimitNs) {
            latch_error(code);
            return false;
        }
    }
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 2-D TMA tile load into this CTA's shared memory (no multicast).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 32 consecutive f32 columns of this warp's 32 tensor-memory lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Byte offset of element (row, k) of a K-major 128-byte-swizzled tile (64 f16 per row, 8-row
// groups of 1024 bytes, 16-byte chunk c of row r stored at chunk c ^ (r % 8)).
__device__ __forceinline__ uint32_t sw128_offset(int row, int k) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ row) & 7) << 4) + (k & 7) * 2);
}

// Two adjacent weights as f16x2: the f16 sums of each word's two halves (MCG, hash-mask, PAIR1:
// the reference's f16 addition) or MUL1's value (its high half is 0).
__device__ __forceinline__ uint32_t half_sums2(uint32_t qa, uint32_t qb) {
    const uint32_t lo = __byte_perm(qa, qb, 0x5410);
    const uint32_t hi = __byte_perm(qa, qb, 0x7632);
    const __half2 s = __hadd2(*reinterpret_cast<const __half2*>(&lo), *reinterpret_cast<const __half2*>(&hi));
    return *reinterpret_cast<const uint32_t*>(&s);
}

struct GemmItem {
    int e, row0, rows;
};

__device__ __forceinline__ bool gemm_item(const GemmArgs& a, int w, int NT, GemmItem& it) {  // NT: rows per item
    if (a.rows > 0) {
        it.e = 0;
        it.row0 = w * NT;
        it.rows = min(NT, a.rows - it.row0);
        return it.rows > 0;
    }
    if (w >= a.meta[0]) return false;
    const int ai = a.work_act[w];
    it.e = a.act_expert[ai];
    it.row0 = a.act_start[ai] + a.work_chunk[w] * NT;
    it.rows = min(NT, a.act_count[ai] - a.work_chunk[w] * NT);
    return true;
}

// Rows t0 .. t0+rows-1 of the item from red[t - t0][o] (summed over the cluster's S ranks in rank
// order when split): H128, svh, the codebook scale, and the store of the launch's mode.  Split-K
// ranks share the rows: rank `rank` finishes rows t = rank, rank + S, ..., one per decoder warp
// at a time, so no rank waits through every row's reduction.
__device__ __forceinline__ void gemm_store(const GemmArgs& a, const GemmItem& it, float* red, cg::cluster_group& cluster,
                                           int S, int rank, int ob, int t0, int rows) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (rank + warp * S >= rows) return;
    const uint16_t* svh = a.svh + (size_t)it.e * a.out;
    float sv[4];
#pragma unroll
    for (int i = 0; i < 4; i++) sv[i] = h2f(svh[ob * 128 + lane * 4 + i]) * a.scale;
    for (int t = rank + warp * S; t < rows; t += kGemmDecWarps * S) {
        const float4 s4 = S > 1 ? cluster_sum4(cluster, red, S, t * 128)
                                : *reinterpret_cast<const float4*>(red + t * 128 + lane * 4);
        float v[4] = {s4.x, s4.y, s4.z, s4.w};
        warp_hadamard128(v);
        const int row = it.row0 + t0 + t;
        const size_t o = (size_t)ob * 128 + lane * 4;
        if (a.mode == GEMM_OUT_ACT) {
#pragma unroll
            for (int i = 0; i < 4; i++) store_act(a.y, (size_t)row * a.out + o + i, a.ydt, v[i] * sv[i]);
        } else if (a.mode == GEMM_OUT_F32) {
            *reinterpret_cast<float4*>(a.yf + (size_t)row * a.out + o) =
                make_float4(v[0] * sv[0], v[1] * sv[1], v[2] * sv[2], v[3] * sv[3]);
        } else {
            const int slot = a.order[row];
            const float sc = a.scores[slot];
            *reinterpret_cast<float4*>(a.yf + (size_t)slot * a.out + o) =
                make_float4(v[0] * sv[0] * sc, v[1] * sv[1] * sc, v[2] * sv[2] * sc, v[3] * sv[3] * sc);
        }
    }
}

// Named barrier 1 over the decoder warps.
__device__ __forceinline__ void decoders_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kGemmDecWarps * 32) : "memory"); }

template <int KIND, int N, int NT, int RT, bool W16, bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap pmap, GemmArgs a) {
    using Lay = GemmLayout<N, NT, RT, PAIR>;
    constexpr int NST = Lay::NST;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t tmem_slot;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    cg::cluster_group cluster = cg::this_cluster();
    GemmItem it;
    // Grid x = output block, y = row item: the output blocks of one row item launch together, so
    // their shared prepared-row tiles come from HBM once and from L2 after.
    if (!gemm_item(a, blockIdx.y, NT * RT, it)) return;  // every CTA of a cluster shares blockIdx.y
    const int rt_live = (it.rows + NT - 1) / NT;          // row tiles with rows in them
    const int ob = blockIdx.x;
    const int S = gridDim.z;
    const int split = blockIdx.z;
    const int KC = a.in / kGemmKC;  // chunks of 64 inputs
    const int c0 = (int)(((long long)split * KC) / S);
    const int ncs = (int)(((long long)(split + 1) * KC) / S) - c0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // tfull: a stage's trellis rows landed (the decoders start); bfull: its prepared-row tiles
    // landed (the MMA needs them); separate so the decode overlaps the larger row-tile copies.
    uint64_t* tfull = reinterpret_cast<uint64_t*>(smem + Lay::BAR_OFF);
    uint64_t* bfull = tfull + NST;
    uint64_t* decoded = bfull + NST;
    uint64_t* empty = decoded + NST;
    uint64_t* acc_full = empty + NST;
    uint64_t* peer_ready = acc_full + 1;  // PAIR, leader: the peer's stage is decoded and loaded
    float* red = reinterpret_cast<float*>(smem);  // [NT][128], after the main loop
    const uint32_t rank = PAIR ? cluster.block_rank() : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&bfull[i], 1);
            mbar_init(&decoded[i], kGemmDecWarps);
            mbar_init(&empty[i], 1);
            mbar_init(&peer_ready[i], 1);
        }
        mbar_init(acc_full, 1);
        fence_mbar_init();
    }
    if (warp == kGemmDecWarps + 1) {  // the MMA warp owns the tensor memory (both CTAs of a pair)
        if constexpr (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                         "n"(Lay::TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                         "n"(Lay::TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster.sync();  // the peer's barriers exist before any remote arrival
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const int OT = a.out / 16;
    const uint16_t* tr = a.trellis + (size_t)it.e * a.tr_expert;
    bool acc_ok = false;  // decoder warps: the accumulator is complete

    if (warp == kGemmDecWarps) {
        // ---------------- producer: trellis rows (bulk) and the prepared rows' tile (TMA)
        if (lane == 0) {
            const uint32_t row_bytes = 8u * N * 2u;
            for (int i = 0; i < ncs; i++) {
                const int st = i % NST;
                if (i >= NST && !mbar_wait(&empty[st], ((i / NST) - 1) & 1, DEV_TIMEOUT_EMPTY)) break;
                mbar_arrive_expect_tx(&tfull[st], Lay::T_BYTES);
                const int kc = c0 + i;
#pragma unroll 1
                for (int r = 0; r < 4; r++) {
                    const size_t tk = (size_t)kc * 4 + r;
                    bulk_g2s(smem + Lay::T_OFF + st * Lay::T_BYTES + r * row_bytes, tr + (tk * OT + (size_t)ob * 8) * N,
                             row_bytes, &tfull[st]);
                }
                if constexpr (PAIR) {
                    // this CTA's half (128 rows) of each live 256-row block
                    const int nb = (it.rows + 2 * NT - 1) / (2 * NT);
                    mbar_arrive_expect_tx(&bfull[st], nb * Lay::B_TILE);
                    for (int j = 0; j < nb; j++)
                        tma_load_2d(smem + Lay::B_OFF + st * Lay::B_BYTES + j * Lay::B_TILE, &pmap, kc * kGemmKC,
                                    it.row0 + j * 2 * NT + (int)rank * NT, &bfull[st]);
                } else {
                    mbar_arrive_expect_tx(&bfull[st], rt_live * Lay::B_TILE);
                    for (int r = 0; r < rt_live; r++)
                        tma_load_2d(smem + Lay::B_OFF + st * Lay::B_BYTES + r * Lay::B_TILE, &pmap, kc * kGemmKC,
                                    it.row0 + r * NT, &bfull[st]);
                }
            }
        }
    } else if (warp == kGemmDecWarps + 1) {
        // ---------------- MMA issuer (a pair's leader; the peer forwards its readiness)
        if (lane == 0 && PAIR && rank == 1) {
            for (int i = 0; i < ncs; i++) {
                const int st = i % NST;
                mbar_wait(&decoded[st], (i / NST) & 1, DEV_TIMEOUT_FULL);
                mbar_wait(&bfull[st], (i / NST) & 1, DEV_TIMEOUT_FULL);
                mbar_arrive_remote(&peer_ready[st], 0);  // arrives even after a timeout: the leader moves on
            }
        } else if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_m128(NT);
            constexpr uint32_t idesc2 = idesc_f16_m128(2 * NT);   // N = 256
            constexpr uint32_t idescp = idesc_f16_m256(2 * NT);   // pair: M = 256, N = 256
            const int nb = (it.rows + 2 * NT - 1) / (2 * NT);
            bool ok = true;
            for (int i = 0; i < ncs; i++) {
                const int st = i % NST;
                if (ok) ok = mbar_wait(&decoded[st], (i / NST) & 1, DEV_TIMEOUT_FULL);
                if (ok) ok = mbar_wait(&bfull[st], (i / NST) & 1, DEV_TIMEOUT_FULL);
                if (PAIR && ok) ok = mbar_wait_cluster(&peer_ready[st], (i / NST) & 1, DEV_TIMEOUT_FULL);
                tc_fence_after();
                if (ok) {
                    const uint32_t a0 = smem_u32(smem + Lay::A_OFF + st * Lay::A_BYTES);
                    const uint32_t b0 = smem_u32(smem + Lay::B_OFF + st * Lay::B_BYTES);
                    if constexpr (PAIR) {
                        // block j: columns j*256.. of both CTAs' accumulators; rows 0..127 of N from
                        // this CTA's tile j, 128..255 from the peer's
                        for (int j = 0; j < nb; j++)
#pragma unroll
                            for (int kk = 0; kk < kGemmKC / 16; kk++)
                                tc_mma2_f16(tmem + (uint32_t)(j * 2 * NT), smem_desc_sw128(a0 + kk * 32),
                                            smem_desc_sw128(b0 + j * Lay::B_TILE + kk * 32), idescp,
                                            (i > 0 || kk > 0) ? 1u : 0u);
                    } else {
                        // Row tiles go two at a time as one N = 256 MMA where both are live (their
                        // prepared-row tiles and accumulators sit back to back): half the A reads
                        // from shared memory per flop of N = 128 MMAs.
                        for (int r = 0; r < rt_live; r += 2) {
                            const bool pair = r + 1 < rt_live;
                            const uint32_t id = pair ? idesc2 : idesc;
#pragma unroll
                            for (int kk = 0; kk < kGemmKC / 16; kk++)
                                tc_mma_f16(tmem + (uint32_t)(r * NT), smem_desc_sw128(a0 + kk * 32),
                                           smem_desc_sw128(b0 + r * Lay::B_TILE + kk * 32), id,
                                           (i > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                }
                if constexpr (PAIR) tc_commit2(&empty[st]);  // frees the stage in both CTAs
                else tc_commit(&empty[st]);
            }
            if constexpr (PAIR) tc_commit2(acc_full);
            else tc_commit(acc_full);
        }
    } else {
        // ---------------- decoders: warp w decodes trellis row w/4, output tiles (w%4)*2 and +1
        constexpr int TPW = 32 / kGemmDecWarps;  // tiles per warp per stage
        LaneFunnel<N> lf;
        lf.init(lane);
        const int ti = warp / (8 / TPW);
        const int to0 = (warp % (8 / TPW)) * TPW;
        const int g = lane >> 2, c = lane & 3;
        // this lane's four 32-bit stores in a decoded tile (output tile to, trellis row ti)
        const uint32_t off_lo = sw128_offset(g, ti * 16 + 2 * c);      // out g,   in 2c, 2c+1
        const uint32_t off_hi = sw128_offset(g, ti * 16 + 2 * c + 8);  // out g,   in 2c+8, 2c+9
        bool ok = true;
        for (int i = 0; i < ncs; i++) {
            const int st = i % NST;
            if (ok) ok = mbar_wait(&tfull[st], (i / NST) & 1, DEV_TIMEOUT_FULL);
            if (ok) {
                const uint32_t* trow =
                    reinterpret_cast<const uint32_t*>(smem + Lay::T_OFF + st * Lay::T_BYTES) + (ti * 8 + to0) * (N / 2);
                uint8_t* at = smem + Lay::A_OFF + st * Lay::A_BYTES;
#pragma unroll
                for (int j = 0; j < TPW; j++) {
                    uint32_t q[8];
                    decode_lane_q<KIND, N, W16>(trow + j * (N / 2), lf, a.dp, q);
                    // output rows (to0 + j)*16 + g and + 8: 8-row groups 2*(to0+j) and 2*(to0+j)+1
                    uint8_t* base = at + (to0 + j) * 2048;
                    *reinterpret_cast<uint32_t*>(base + off_lo) = half_sums2(q[0], q[1]);
                    *reinterpret_cast<uint32_t*>(base + off_hi) = half_sums2(q[2], q[3]);
                    *reinterpret_cast<uint32_t*>(base + 1024 + off_lo) = half_sums2(q[4], q[5]);
                    *reinterpret_cast<uint32_t*>(base + 1024 + off_hi) = half_sums2(q[6], q[7]);
                }
                fence_proxy_async_smem();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&decoded[st]);
        }

        acc_ok = mbar_wait(acc_full, 0, DEV_TIMEOUT_FULL);
    }

    // ---------------- epilogue, every thread (the cluster barriers count them all): per row tile,
    // warps 0..3 move the accumulator to shared memory red[t][o] (tensor-memory lane quadrant =
    // warp), then each rank sums its share of the rows over the cluster's partials in rank order
    // (split-K), applies H128, svh and the scale, and stores; the second barrier keeps every rank's
    // red alive until every rank is done reading.
    for (int r = 0; r < rt_live; r++) {
        if (warp < 4) {
            tc_fence_after();
            const int o = warp * 32 + lane;
#pragma unroll 1
            for (int col = 0; col < NT; col += 32) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(r * NT + col), v);
#pragma unroll
                for (int j = 0; j < 32; j++) red[(col + j) * 128 + o] = acc_ok ? v[j] : 0.0f;
            }
        }
        if (S > 1) cluster.sync(); else __syncthreads();
        if (warp < kGemmDecWarps) gemm_store(a, it, red, cluster, S, split, ob, r * NT, min(NT, it.rows - r * NT));
        if (S > 1) cluster.sync(); else __syncthreads();
    }
    tc_fence_before();
    if constexpr (PAIR) cluster.sync();  // both CTAs are done with the pair's MMAs and tensor memory
    else __syncthreads();
    if (warp == kGemmDecWarps + 1) {
        tc_fence_after();
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(Lay::TMEM_COLS)
                         : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(Lay::TMEM_COLS)
                         : "memory");
    }
}

}  // namespace sx
