// Building blocks of the decode-GEMV family (dense linears and the gathered MoE experts).
//
// Work unit of a CTA: one 128-wide output block (8 output tiles) of NP projections that share an
// input (NP = 1 for a linear or the down projection, 2 for an expert's gate and up), over a
// contiguous range of 128-wide input blocks, for up to 8*NB rows.
//   * producer warp: streams each input block's 8 x 8 tiles of every projection into a ring of
//     shared-memory stages with 1-D bulk (TMA) copies, 8*n*2 contiguous bytes per tile row.
//   * consumer warps (8): warp w decodes input-tile row w of every stage for all 8 output tiles
//     and NP projections and runs two m16n8k16 MMAs per tile and row group (doubled k: the tensor
//     core adds each weight's two f16 halves, sx_decode.cuh).
//   * the warps' accumulators are summed in a fixed order into shared memory.
#pragma once

#include "sx_decode.cuh"

namespace sx {

constexpr int kConsumerWarps = 8;
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
// projection (each projection prepares the input with its own suh), the NP x (8*NB) x 128 f32
// reduction, the ring's barriers.
template <int N, int NP, int NB>
__host__ __device__ inline CoreLayout core_layout(int kbl_max) {
    CoreLayout L;
    size_t off = 0;
    L.stages = off;
    off += (size_t)Ring<N, NP>::NST * Ring<N, NP>::STAGE_BYTES;
    L.bfrag = off;
    off += (size_t)NP * kbl_max * 8 * NB * 32 * 16;
    L.red = off;
    off += (size_t)NP * NB * 8 * 128 * 4;
    L.bars = off;
    off += (size_t)2 * Ring<N, NP>::NST * 8;
    L.total = off;
    return L;
}

struct CoreSmem {
    uint8_t* stages;
    uint4* bfrag;          // [NP][kbl_max][8][NB][32]
    int bfrag_proj_stride; // uint4 elements between projections
    float* red;
    uint64_t* full;
    uint64_t* empty;
};

template <int N, int NP, int NB>
__device__ __forceinline__ CoreSmem core_smem(uint8_t* smem, int kbl_max) {
    const CoreLayout L = core_layout<N, NP, NB>(kbl_max);
    CoreSmem s;
    s.stages = smem + L.stages;
    s.bfrag = reinterpret_cast<uint4*>(smem + L.bfrag);
    s.bfrag_proj_stride = kbl_max * 8 * NB * 32;
    s.red = reinterpret_cast<float*>(smem + L.red);
    s.full = reinterpret_cast<uint64_t*>(smem + L.bars);
    s.empty = s.full + Ring<N, NP>::NST;
    return s;
}

template <int N, int NP>
__device__ __forceinline__ void core_init_barriers(const CoreSmem& s) {
    if (threadIdx.x == kConsumerWarps * 32) {
        for (int i = 0; i < Ring<N, NP>::NST; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], kConsumerWarps);
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
template <int NB>
__device__ __forceinline__ void bfrag_put(uint4* bfrag, int kbi, int m, int pos, uint16_t h) {
    const int nb = m >> 3, gg = m & 7;
    const int tk = pos >> 4, r = pos & 15;
    const int c = (r & 7) >> 1;
    const int slot = ((r >> 3) << 1) | (r & 1);
    uint32_t* dst = reinterpret_cast<uint32_t*>(&bfrag[((kbi * 8 + tk) * NB + nb) * 32 + gg * 4 + c]);
    dst[slot] = (uint32_t)h | ((uint32_t)h << 16);
}

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// Consumers: decode + MMA over kbl stages; acc[p][j][nb][e] per lane.
template <int KIND, int N, int NP, int NB>
__device__ __forceinline__ bool core_consume(const CoreSmem& s, int kbl, const DecParams (&dp)[NP],
                                             float (&acc)[NP][8][NB][4]) {
    constexpr int NST = Ring<N, NP>::NST;
    constexpr int TILE_WORDS = N / 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    LaneFunnel<N> lf;
    lf.init(lane);
#pragma unroll
    for (int p = 0; p < NP; p++)
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
            for (int nb = 0; nb < NB; nb++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[p][j][nb][e] = 0.0f;
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
                    b[nb] = s.bfrag[p * s.bfrag_proj_stride + ((i * 8 + warp) * NB + nb) * 32 + lane];
                const uint32_t* row = reinterpret_cast<const uint32_t*>(s.stages + (size_t)st * Ring<N, NP>::STAGE_BYTES +
                                                                        p * Ring<N, NP>::PROJ_BYTES) +
                                      warp * 8 * TILE_WORDS;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    uint32_t q[8];
                    decode_lane_q<KIND, N>(row + j * TILE_WORDS, lf, dp[p], q);
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        mma16816(acc[p][j][nb], q[0], q[4], q[1], q[5], b[nb].x, b[nb].y);
                        mma16816(acc[p][j][nb], q[2], q[6], q[3], q[7], b[nb].z, b[nb].w);
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
template <int NP, int NB>
__device__ __forceinline__ void core_reduce(float* red, const float (&acc)[NP][8][NB][4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, cq = lane & 3;
    for (int w = 0; w < kConsumerWarps; w++) {
        if (warp == w) {
#pragma unroll
            for (int p = 0; p < NP; p++)
#pragma unroll
                for (int j = 0; j < 8; j++)
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        float* rp = red + (size_t)p * NB * 8 * 128;
                        const int m0 = nb * 8 + 2 * cq;
                        const int o0 = j * 16 + gq;
                        rp[m0 * 128 + o0] += acc[p][j][nb][0];
                        rp[(m0 + 1) * 128 + o0] += acc[p][j][nb][1];
                        rp[m0 * 128 + o0 + 8] += acc[p][j][nb][2];
                        rp[(m0 + 1) * 128 + o0 + 8] += acc[p][j][nb][3];
                    }
        }
        consumers_sync();
    }
}

}  // namespace sx
