// Building blocks of the decode-GEMV family (dense linears and the gathered MoE experts).
//
// Work unit of a CTA: one 128-wide output block (8 output tiles) of NP projections that share an
// input (NP = 1 for a linear or the down projection, 2 for an expert's gate and up), over a
// contiguous range of 128-wide input blocks, for up to 8*NB rows.
//   * producer warp: streams each input block's 8 x 8 tiles of every projection into a ring of
//     shared-memory stages with 1-D bulk (TMA) copies, 8*n*2 contiguous bytes per tile row.
//   * CW consumer warps (8 or 16): warp w decodes the TPW = 64/CW tiles of output tile w % 8 in
//     input-tile rows (w / 8)*TPW.. of every stage for NP projections and runs two m16n8k16 MMAs
//     per tile and row group (doubled k: the tensor core adds each weight's two f16 halves,
//     sx_decode.cuh), accumulating its output tile's k sum in registers.
//   * the block's partial sums land in shared memory (core_reduce), in a fixed order.
#pragma once

#include <cooperative_groups.h>

#include <type_traits>

#include "sx_decode.cuh"

namespace sx {

namespace cg = cooperative_groups;

constexpr int kConsumerWarps = 8;  // the MoE kernels' consumer warps
constexpr int kThreads = (kConsumerWarps + 1) * 32;

template <int N, int NP>
struct Ring {
    static constexpr int PROJ_BYTES = 64 * N * 2;          // 8 input tiles x 8 output tiles
    static constexpr int STAGE_BYTES = NP * PROJ_BYTES;
    static constexpr int NST = STAGE_BYTES <= 5120 ? 8 : (STAGE_BYTES <= 10240 ? 6 : 4);
};

struct CoreLayout {
    size_t stages, bfrag, red, bars, total;
};

// Bytes of one lane's B-fragment entry (four inputs of one row): 16 with each f16 stored twice, as
// the doubled-k MMA reads it; 8 in the compact form of the two-row-group (9..16 rows) kernels,
// where the duplicates are made at load time by byte permutes, so that a CTA's input slice for
// 16 rows takes half the shared memory and two CTAs fit on an SM.
template <int NB>
struct BFrag {
    static constexpr bool COMPACT = NB == 2;
    static constexpr int BYTES = COMPACT ? 8 : 16;
    using Entry = std::conditional_t<COMPACT, uint2, uint4>;
};

// Shared memory of one CTA: the stage ring, the B fragments of kbl_max input blocks per
// projection (each projection prepares the input with its own suh) for mg rows per 8-row group
// (mg = min(8, rows); the lanes of later rows read row mg-1's), the NP x (8*NB) x 128 f32
// reduction, the ring's barriers.
template <int N, int NP, int NB>
__host__ __device__ inline CoreLayout core_layout(int kbl_max, int mg = 8) {
    CoreLayout L;
    size_t off = 0;
    L.stages = off;
    off += (size_t)Ring<N, NP>::NST * Ring<N, NP>::STAGE_BYTES;
    L.bfrag = off;
    off += (size_t)NP * kbl_max * 8 * NB * mg * 4 * BFrag<NB>::BYTES;
    L.red = off;
    off += (size_t)NP * NB * 8 * 128 * 4;
    L.bars = off;
    off += (size_t)2 * Ring<N, NP>::NST * 8;
    L.total = off;
    return L;
}

struct CoreSmem {
    uint8_t* stages;
    uint4* bfrag;          // [NP][kbl_max][NB][mg][8 tiles][4] entries of BFrag<NB>::BYTES
    int bfrag_proj_stride; // entries between projections
    int mg;                // fragment rows per 8-row group
    float* red;
    uint64_t* full;
    uint64_t* empty;
};

template <int N, int NP, int NB>
__device__ __forceinline__ CoreSmem core_smem(uint8_t* smem, int kbl_max, int mg = 8) {
    const CoreLayout L = core_layout<N, NP, NB>(kbl_max, mg);
    CoreSmem s;
    s.stages = smem + L.stages;
    s.bfrag = reinterpret_cast<uint4*>(smem + L.bfrag);
    s.bfrag_proj_stride = kbl_max * 8 * NB * mg * 4;
    s.mg = mg;
    s.red = reinterpret_cast<float*>(smem + L.red);
    s.full = reinterpret_cast<uint64_t*>(smem + L.bars);
    s.empty = s.full + Ring<N, NP>::NST;
    return s;
}

// Barrier init by the producer warp's first thread (thread CW*32).
template <int N, int NP, int CW>
__device__ __forceinline__ void core_init_barriers(const CoreSmem& s) {
    if (threadIdx.x == CW * 32) {
        for (int i = 0; i < Ring<N, NP>::NST; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], CW);
        }
        fence_mbar_init();
    }
}

// Producer (one lane): input blocks kb0..kb0+kbl-1 of projection p's bank `tr[p]` ([IT][OT][N]
// tiles), output block ob.  Returns false after a timed-out wait.
template <int N, int NP>
__device__ __forceinline__ bool core_produce(const CoreSmem& s, const uint16_t* const (&tr)[NP], int OT, int ob, int kb0,
                                             int kbl) {
    constexpr int NST = Ring<N, NP>::NST;
    constexpr int PB = Ring<N, NP>::PROJ_BYTES;
    const uint32_t row_bytes = 8u * N * 2u;
    for (int i = 0; i < kbl; i++) {
        const int st = i % NST;
        if (i >= NST && !mbar_wait(&s.empty[st], ((i / NST) - 1) & 1, DEV_TIMEOUT_EMPTY)) return false;
        mbar_arrive_expect_tx(&s.full[st], Ring<N, NP>::STAGE_BYTES);
        const size_t kb = (size_t)(kb0 + i);
#pragma unroll
        for (int p = 0; p < NP; p++) {
#pragma unroll 1
            for (int r = 0; r < 8; r++) {
                const size_t tk = kb * 8 + r;
                const uint16_t* src = tr[p] + (tk * OT + (size_t)ob * 8) * N;
                bulk_g2s(s.stages + (size_t)st * Ring<N, NP>::STAGE_BYTES + p * PB + r * row_bytes, src, row_bytes,
                         &s.full[st]);
            }
        }
    }
    return true;
}

// B fragments in shared memory: entry (kbi, nb, gg, tk, c) at ((((kbi*NB + nb)*mg + gg)*8 + tk)*4 + c
// holds the inputs 2c, 2c+1, 2c+8, 2c+9 of input tile tk of local block kbi for row nb*8 + gg, the
// lane (g = gg, c)'s B registers of the doubled-k MMA (MMA1 takes inputs 2c, 2c+1 and MMA2 2c+8,
// 2c+9, each duplicated; sx_decode.cuh).  Consecutive input tiles of one row are four entries
// apart, so a consumer steps through a stage's tiles at compile-time offsets.  Rows with
// gg >= mg are not stored (their lanes read row mg-1's).
__host__ __device__ constexpr int bfrag_entry(int kbi, int nb, int gg, int tk, int c, int NB, int mg) {
    return (((kbi * NB + nb) * mg + gg) * 8 + tk) * 4 + c;
}

// The four prepared values a lane holds (positions 4*lane .. 4*lane+3 of local input block kbi,
// row m) in two stores: positions 4*lane and +1 (tile tk = lane/4, tile rows 4*(lane%4), +1) fill
// slots s0 and s0+1 of entry c0, positions +2 and +3 the same slots of entry c0+1 (c0 =
// 2*(lane&1), s0 = 2*((lane>>1)&1)).
template <int NB>
__device__ __forceinline__ void bfrag_put4(uint4* bfrag, int mg, int kbi, int m, int lane, const uint16_t (&h)[4]) {
    const int nb = m >> 3, gg = m & 7;
    if (gg >= mg) return;
    const int tk = lane >> 2;
    const int c0 = (lane & 1) * 2;
    const int s0 = ((lane >> 1) & 1) * 2;
    const size_t entry = (size_t)bfrag_entry(kbi, nb, gg, tk, c0, NB, mg);
#pragma unroll
    for (int q = 0; q < 2; q++) {
        const uint16_t a = h[2 * q], b = h[2 * q + 1];
        if constexpr (BFrag<NB>::COMPACT) {
            reinterpret_cast<uint32_t*>(reinterpret_cast<uint16_t*>(bfrag) + (entry + q) * 4 + s0)[0] =
                (uint32_t)a | ((uint32_t)b << 16);
        } else {
            reinterpret_cast<uint2*>(reinterpret_cast<uint32_t*>(&bfrag[entry + q]) + s0)[0] =
                make_uint2((uint32_t)a | ((uint32_t)a << 16), (uint32_t)b | ((uint32_t)b << 16));
        }
    }
}

// A B-fragment entry as the four doubled-k B registers (inputs 2c, 2c+1, 2c+8, 2c+9, each f16 in
// both halves).
__device__ __forceinline__ uint4 bfrag_expand(uint4 v) { return v; }
__device__ __forceinline__ uint4 bfrag_expand(uint2 u) {
    return make_uint4(__byte_perm(u.x, 0, 0x1010), __byte_perm(u.x, 0, 0x3232), __byte_perm(u.y, 0, 0x1010),
                      __byte_perm(u.y, 0, 0x3232));
}

// Named barrier 1 over the CW consumer warps only.
template <int CW>
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
}

// Consumers: decode + MMA over kbl stages.  Warp w owns output tile ot = w % 8 of the block and
// input-tile rows h*TPW .. h*TPW+TPW-1 of every stage (h = w / 8, TPW = 64 / CW), so the k sum of
// its output tile stays in its registers across the whole range; with 16 warps two warps share an
// output tile and core_reduce adds the pair.  acc[p][nb][e] is the lane's m16n8 fragment (outputs
// gq, gq+8 of the tile; rows 2cq, 2cq+1 of row group nb).
template <int KIND, int N, int NP, int NB, bool W16, int CW>
__device__ __forceinline__ bool core_consume(const CoreSmem& s, int kbl, const DecParams (&dp)[NP],
                                             float (&acc)[NP][NB][4]) {
    static_assert(CW == 8 || CW == 16, "8 or 16 consumer warps");
    constexpr int NST = Ring<N, NP>::NST;
    constexpr int TILE_WORDS = N / 2;
    constexpr int TPW = 64 / CW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ot = warp & 7;
    const int tr0 = (warp >> 3) * TPW;
    LaneFunnel<N> lf;
    lf.init(lane);
    // two accumulator sets (even and odd rows) so consecutive tiles' MMAs do not chain
    float acc2[NP][NB][4];
#pragma unroll
    for (int p = 0; p < NP; p++)
#pragma unroll
        for (int nb = 0; nb < NB; nb++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[p][nb][e] = acc2[p][nb][e] = 0.0f;
    // Lanes of rows past the stored mg read row mg-1's fragments instead of branching: their
    // output columns belong to rows no caller reads.  A lane's B-fragment entry for tile j of a
    // stage is a compile-time offset (4 j entries) from its entry for tile 0.
    const int gq = lane >> 2;
    using BE = typename BFrag<NB>::Entry;
    const int bf_lane = bfrag_entry(0, 0, min(gq, s.mg - 1), tr0, lane & 3, NB, s.mg);
    const int bf_block = NB * s.mg * 32;  // entries per local input block
    const int bf_group = s.mg * 32;       // entries between row groups
    bool ok = true;
    for (int i = 0; i < kbl; i++) {
        const int st = i % NST;
        if (ok) ok = mbar_wait(&s.full[st], (i / NST) & 1, DEV_TIMEOUT_FULL);
        if (ok) {
#pragma unroll
            for (int p = 0; p < NP; p++) {
                const uint32_t* base = reinterpret_cast<const uint32_t*>(s.stages + (size_t)st * Ring<N, NP>::STAGE_BYTES +
                                                                         p * Ring<N, NP>::PROJ_BYTES) +
                                       (tr0 * 8 + ot) * TILE_WORDS;
                const BE* bf = reinterpret_cast<const BE*>(s.bfrag) + p * s.bfrag_proj_stride + i * bf_block + bf_lane;
#pragma unroll
                for (int j = 0; j < TPW; j++) {
                    uint32_t a1[4], a2[4];
                    decode_lane_mma<KIND, N, W16>(base + j * 8 * TILE_WORDS, lf, dp[p], a1, a2);
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        const uint4 b = bfrag_expand(bf[nb * bf_group + j * 4]);
                        float(&d)[4] = (j & 1) ? acc2[p][nb] : acc[p][nb];
                        mma16816(d, a1[0], a1[1], a1[2], a1[3], b.x, b.y);
                        mma16816(d, a2[0], a2[1], a2[2], a2[3], b.z, b.w);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[st]);
    }
#pragma unroll
    for (int p = 0; p < NP; p++)
#pragma unroll
        for (int nb = 0; nb < NB; nb++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[p][nb][e] += acc2[p][nb][e];
    return ok;
}

// The block's partial sums into red[p][m][o] (m < 8*NB rows, o < 128 outputs), every entry
// written.  With 16 warps, warps 8..15 store first and warps 0..7 add theirs after a barrier of
// the consumer warps (a fixed order; the sum of two terms is the same either way).
template <int NP, int NB, int CW>
__device__ __forceinline__ void core_reduce(float* red, const float (&acc)[NP][NB][4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, cq = lane & 3;
    const int o0 = (warp & 7) * 16 + gq;
    auto put = [&](bool add) {
#pragma unroll
        for (int p = 0; p < NP; p++)
#pragma unroll
            for (int nb = 0; nb < NB; nb++) {
                float* rp = red + (size_t)p * NB * 8 * 128;
                const int m0 = nb * 8 + 2 * cq;
                float* q0 = rp + m0 * 128 + o0;
                float* q1 = rp + (m0 + 1) * 128 + o0;
                if (add) {
                    q0[0] += acc[p][nb][0];
                    q1[0] += acc[p][nb][1];
                    q0[8] += acc[p][nb][2];
                    q1[8] += acc[p][nb][3];
                } else {
                    q0[0] = acc[p][nb][0];
                    q1[0] = acc[p][nb][1];
                    q0[8] = acc[p][nb][2];
                    q1[8] = acc[p][nb][3];
                }
            }
    };
    if (CW == 8) {
        put(false);
    } else {
        if (warp >= 8) put(false);
        consumers_sync<CW>();
        if (warp < 8) put(true);
    }
}

// Sum over the cluster's S CTAs, in rank order, of the four floats red[off + 4*lane ..] of each:
// the loads go out eight ranks at a time so distributed shared memory's latency is paid S/8 times.
__device__ __forceinline__ float4 cluster_sum4(cg::cluster_group& cluster, float* red, int S, int off) {
    const int lane = threadIdx.x & 31;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    auto add = [&](const float4& t) {
        v.x += t.x;
        v.y += t.y;
        v.z += t.z;
        v.w += t.w;
    };
    int r = 0;
    for (; r + 8 <= S; r += 8) {
        float4 t[8];
#pragma unroll
        for (int q = 0; q < 8; q++)
            t[q] = *reinterpret_cast<const float4*>(cluster.map_shared_rank(red, r + q) + off + lane * 4);
#pragma unroll
        for (int q = 0; q < 8; q++) add(t[q]);
    }
    if (r + 4 <= S) {
        float4 t[4];
#pragma unroll
        for (int q = 0; q < 4; q++)
            t[q] = *reinterpret_cast<const float4*>(cluster.map_shared_rank(red, r + q) + off + lane * 4);
#pragma unroll
        for (int q = 0; q < 4; q++) add(t[q]);
        r += 4;
    }
    for (; r < S; r++) add(*reinterpret_cast<const float4*>(cluster.map_shared_rank(red, r) + off + lane * 4));
    return v;
}

// Programmatic dependent launch: wait for the grid this one depends on (a no-op when launched
// without the attribute), and let the next grid on the stream start launching.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace sx
