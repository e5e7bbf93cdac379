// Building blocks of the decode-GEMV family (dense linears and the gathered MoE experts).
//
// Work unit of a CTA: one 128-wide output block (8 output tiles) of NP projections that share an
// input (NP = 1 for a linear or the down projection, 2 for an expert's gate and up), over a
// contiguous range of 128-wide input blocks, for up to 8*NB rows.
//   * producer warp: streams each input block's 8 x 8 tiles of every projection into a ring of
//     shared-memory stages with 1-D bulk (TMA) copies, 8*n*2 contiguous bytes per tile row.
//   * CW consumer warps (8 or 16): each decodes TPW = 64/CW tiles of every stage (input-tile row
//     w / (8/TPW), output tiles from (w % (8/TPW)) * TPW) for NP projections and runs two
//     m16n8k16 MMAs per tile and row group (doubled k: the tensor core adds each weight's two f16
//     halves, sx_decode.cuh).
//   * the warps' accumulators are summed in a fixed order into shared memory.
#pragma once

#include "sx_decode.cuh"

namespace sx {

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

// Shared memory of one CTA: the stage ring, the B fragments of kbl_max input blocks per
// projection (each projection prepares the input with its own suh) for mg rows per 8-row group
// (mg = min(8, rows): only the lanes of live rows load fragments), the NP x (8*NB) x 128 f32
// reduction, the ring's barriers.
template <int N, int NP, int NB>
__host__ __device__ inline CoreLayout core_layout(int kbl_max, int mg = 8) {
    CoreLayout L;
    size_t off = 0;
    L.stages = off;
    off += (size_t)Ring<N, NP>::NST * Ring<N, NP>::STAGE_BYTES;
    L.bfrag = off;
    off += (size_t)NP * kbl_max * 8 * NB * mg * 4 * 16;
    L.red = off;
    off += (size_t)NP * NB * 8 * 128 * 4;
    L.bars = off;
    off += (size_t)2 * Ring<N, NP>::NST * 8;
    L.total = off;
    return L;
}

struct CoreSmem {
    uint8_t* stages;
    uint4* bfrag;          // [NP][kbl_max][8][NB][mg][4]
    int bfrag_proj_stride; // uint4 elements between projections
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

// One prepared value v of row m at position pos (0..127) of local input block kbi, into the
// B-fragment slot its MMA lane reads: lane (g = m%8, c), register slot by the input's row in
// the tile (sx_decode.cuh: MMA1 takes inputs 2c, 2c+1 and MMA2 2c+8, 2c+9, each duplicated).
// Rows m with m % 8 >= mg are not stored (their lanes read zeros).
template <int NB>
__device__ __forceinline__ void bfrag_put(uint4* bfrag, int mg, int kbi, int m, int pos, uint16_t h) {
    const int nb = m >> 3, gg = m & 7;
    if (gg >= mg) return;
    const int tk = pos >> 4, r = pos & 15;
    const int c = (r & 7) >> 1;
    const int slot = ((r >> 3) << 1) | (r & 1);
    uint32_t* dst = reinterpret_cast<uint32_t*>(&bfrag[(((kbi * 8 + tk) * NB + nb) * mg + gg) * 4 + c]);
    dst[slot] = (uint32_t)h | ((uint32_t)h << 16);
}

// Named barrier 1 over the CW consumer warps only.
template <int CW>
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
}

// Consumers: decode + MMA over kbl stages; acc[p][t][nb][e] per lane for its TPW tiles.
template <int KIND, int N, int NP, int NB, bool W16, int CW>
__device__ __forceinline__ bool core_consume(const CoreSmem& s, int kbl, const DecParams (&dp)[NP],
                                             float (&acc)[NP][64 / CW][NB][4]) {
    constexpr int NST = Ring<N, NP>::NST;
    constexpr int TILE_WORDS = N / 2;
    constexpr int TPW = 64 / CW;
    constexpr int WPR = 8 / TPW;  // warps per input-tile row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int trow = warp / WPR;
    const int t0 = (warp % WPR) * TPW;
    LaneFunnel<N> lf;
    lf.init(lane);
#pragma unroll
    for (int p = 0; p < NP; p++)
#pragma unroll
        for (int j = 0; j < TPW; j++)
#pragma unroll
            for (int nb = 0; nb < NB; nb++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[p][j][nb][e] = 0.0f;
    const int gq = lane >> 2;
    const bool live = gq < s.mg;
    bool ok = true;
    for (int i = 0; i < kbl; i++) {
        const int st = i % NST;
        if (ok) ok = mbar_wait(&s.full[st], (i / NST) & 1, DEV_TIMEOUT_FULL);
        if (ok) {
#pragma unroll
            for (int p = 0; p < NP; p++) {
                uint4 b[NB];
#pragma unroll
                for (int nb = 0; nb < NB; nb++)
                    b[nb] = live ? s.bfrag[p * s.bfrag_proj_stride + (((i * 8 + trow) * NB + nb) * s.mg + gq) * 4 +
                                           (lane & 3)]
                                 : make_uint4(0u, 0u, 0u, 0u);
                const uint32_t* row = reinterpret_cast<const uint32_t*>(s.stages + (size_t)st * Ring<N, NP>::STAGE_BYTES +
                                                                        p * Ring<N, NP>::PROJ_BYTES) +
                                      (trow * 8 + t0) * TILE_WORDS;
#pragma unroll
                for (int j = 0; j < TPW; j++) {
                    uint32_t a1[4], a2[4];
                    decode_lane_mma<KIND, N, W16>(row + j * TILE_WORDS, lf, dp[p], a1, a2);
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        mma16816(acc[p][j][nb], a1[0], a1[1], a1[2], a1[3], b[nb].x, b[nb].y);
                        mma16816(acc[p][j][nb], a2[0], a2[1], a2[2], a2[3], b[nb].z, b[nb].w);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[st]);
    }
    return ok;
}

// Sum of the consumer warps' accumulators, warp 0 first, into red[p][m][o] (m < 8*NB rows,
// o < 128 outputs of the block).  `red` must be zeroed and published before.
template <int NP, int NB, int CW>
__device__ __forceinline__ void core_reduce(float* red, const float (&acc)[NP][64 / CW][NB][4]) {
    constexpr int TPW = 64 / CW;
    constexpr int WPR = 8 / TPW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, cq = lane & 3;
    const int t0 = (warp % WPR) * TPW;
    for (int w = 0; w < CW; w++) {
        if (warp == w) {
#pragma unroll
            for (int p = 0; p < NP; p++)
#pragma unroll
                for (int j = 0; j < TPW; j++)
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        float* rp = red + (size_t)p * NB * 8 * 128;
                        const int m0 = nb * 8 + 2 * cq;
                        const int o0 = (t0 + j) * 16 + gq;
                        rp[m0 * 128 + o0] += acc[p][j][nb][0];
                        rp[(m0 + 1) * 128 + o0] += acc[p][j][nb][1];
                        rp[m0 * 128 + o0 + 8] += acc[p][j][nb][2];
                        rp[(m0 + 1) * 128 + o0 + 8] += acc[p][j][nb][3];
                    }
        }
        consumers_sync<CW>();
    }
}

}  // namespace sx
