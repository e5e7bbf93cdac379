// Trellis decode on the device: the lane layout, the tail-biting bit funnel and the codebooks.
//
// A 16x16 tile is 256 weights packed as n halfwords (K = n/16 bits per weight).  Weight t's
// codeword is the 16-bit window of the circular, MSB-first bitstream that ends at bit
// bitEnd(t) = ((t+1)*n) >> 4 (src/exl3/expert_exl3.zig:180-226, :317-336).  Lane L of a warp owns
// stream positions 8L..8L+7, whose row-major places (tensorCorePerm, :379-398) are exactly the
// A-fragment places of an m16n8k16 MMA: lane (g = L/4, c = L%4) holds outputs g and g+8 at inputs
// 2c, 2c+1, 2c+8, 2c+9.  So a lane decodes its eight codewords from at most n/2 - n/16 + 16
// consecutive stream bits ending at bit (L+1)*n/2, and the shift of codeword j inside that run is
// the same compile-time constant for every lane: s_j = n/2 - floor((j+1)*n/16).
#pragma once

#include "sx_common.cuh"

namespace sx {

enum Cb : int { CB_MUL1 = 0, CB_MCG = 1, CB_SPEC1 = 2, CB_PAIR1 = 3, CB_STD1 = 4 };
// Kernel-side codebook families: the hash-mask codebooks (STD1, SPEC1) share one body.
enum CbKind : int { K_MUL1 = 0, K_MCG = 1, K_HASH = 2, K_PAIR1 = 3 };

struct DecParams {
    uint32_t wmask;  // window mask, (1 << window_bits) - 1
    uint32_t mult;   // hash-mask / PAIR1 multiplier
    uint32_t mask0;  // hash-mask mask, or PAIR1 mask0
    uint32_t mask1;  // PAIR1 mask1
    uint32_t rot;    // PAIR1 rotation
};

template <int N>
struct Funnel {
    static constexpr int W = N / 2;                            // 32-bit words per tile
    static constexpr int S_MAX = N / 2 - N / 16;               // shift of codeword 0
    static constexpr int NR = (S_MAX + 16 + 31) / 32;          // 32-bit stream registers a lane needs
    static constexpr int shift(int j) { return N / 2 - ((j + 1) * N) / 16; }
    // Words a lane loads: the most, over lanes, between the first codeword's first bit and the
    // lane's last bit.
    static constexpr int words_needed() {
        int most = 0;
        for (int t = 0; t < 32; t++) {
            const int e = (t + 1) * N / 2;
            const int first = e - S_MAX - 16 + 64 * N;  // shifted positive: tail-biting wrap
            const int we = (e - 1 + 64 * N) / 32;
            const int wf = first / 32;
            const int cnt = we - wf + 1;
            most = cnt > most ? cnt : most;
        }
        return most;
    }
    static constexpr int NWL = words_needed();
};

// Per-lane constants of the funnel, computed once per kernel.
template <int N>
struct LaneFunnel {
    uint32_t idx[Funnel<N>::NWL];  // word indices inside the tile, oldest first (mod n/2)
    uint32_t sh;                   // 32 - (bits of the last word that belong to the lane)

    __device__ __forceinline__ void init(int lane) {
        const int e = (lane + 1) * N / 2;
        const int we = (e - 1) / 32;
        const int off = e - 32 * we;  // 1..32
        sh = (uint32_t)(32 - off);
#pragma unroll
        for (int k = 0; k < Funnel<N>::NWL; k++) {
            int w = we - (Funnel<N>::NWL - 1) + k;
            w %= Funnel<N>::W;
            if (w < 0) w += Funnel<N>::W;
            idx[k] = (uint32_t)w;
        }
    }
};

// The lane's stream registers: r[0] = bits [E-32, E), r[1] = [E-64, E-32), ..., E the lane's end.
template <int N>
__device__ __forceinline__ void lane_stream(const uint32_t* tile_words, const LaneFunnel<N>& lf,
                                            uint32_t (&r)[Funnel<N>::NR]) {
    constexpr int NWL = Funnel<N>::NWL;
    uint32_t w[NWL];
#pragma unroll
    for (int k = 0; k < NWL; k++) w[k] = tile_words[lf.idx[k]];
#pragma unroll
    for (int i = 0; i < Funnel<N>::NR; i++) {
        const int lo_k = NWL - 1 - i;
        const int hi_k = NWL - 2 - i;
        const uint32_t lo = lo_k >= 0 ? w[lo_k] : 0u;
        const uint32_t hi = hi_k >= 0 ? w[hi_k] : 0u;
        r[i] = __funnelshift_rc(lo, hi, lf.sh);
    }
}

// 2^(16-b) for b = 0..16, in constant memory so the compiler cannot see the value: (r * c) >> 16
// then stays a multiply on the FMA pipe plus one ALU shift, instead of the shift-and-mask pair on
// the half-rate ALU pipe that a literal power of two turns into.
extern __constant__ uint32_t c_pow2_16[17];

// Codeword j of the lane (window-masked), from its stream registers.  At window 16 a codeword
// inside one register is (r * 2^(16-b)) >> 16; other windows mask at run time.
template <int N, int J, bool W16>
__device__ __forceinline__ uint32_t codeword(const uint32_t (&r)[Funnel<N>::NR], uint32_t wmask) {
    constexpr int s = Funnel<N>::shift(J);
    constexpr int i = s / 32;
    constexpr int b = s % 32;
    if constexpr (W16) {
        if constexpr (b == 0) {
            return r[i] & 0xFFFFu;
        } else if constexpr (b == 16) {
            return r[i] >> 16;
        } else if constexpr (b < 16) {
            return (r[i] * c_pow2_16[b]) >> 16;
        } else {
            return __funnelshift_r(r[i], r[i + 1], b) & 0xFFFFu;
        }
    } else {
        if constexpr (b + 16 <= 32) {
            return (r[i] >> b) & wmask;
        } else {
            return __funnelshift_r(r[i], r[i + 1], b) & wmask;
        }
    }
}

__device__ __forceinline__ uint32_t rotl32(uint32_t v, uint32_t r) { return __funnelshift_l(v, v, r); }

// The eight MMA A-register values of the lane's codewords, stream order v0..v7.  Each register
// holds two f16 halves whose SUM is the weight (times the codebook's output scale): the MMA is run
// with its k dimension doubled, both halves against the same input, so the tensor core performs
// the half sum (src/exl3/expert_exl3.zig:267-301).  MUL1's register holds (weight, 0).
template <int KIND, int N, bool W16>
__device__ __forceinline__ void decode_r_q(const uint32_t (&r)[Funnel<N>::NR], const DecParams& dp, uint32_t (&q)[8]);

template <int KIND, int N, bool W16>
__device__ __forceinline__ void decode_lane_q(const uint32_t* tile_words, const LaneFunnel<N>& lf, const DecParams& dp,
                                              uint32_t (&q)[8]) {
    uint32_t r[Funnel<N>::NR];
    lane_stream<N>(tile_words, lf, r);
    decode_r_q<KIND, N, W16>(r, dp, q);
}

// The eight codewords of a lane's stream registers hashed into MMA A-register values.
template <int KIND, int N, bool W16>
__device__ __forceinline__ void decode_r_q(const uint32_t (&r)[Funnel<N>::NR], const DecParams& dp, uint32_t (&q)[8]) {
    if constexpr (KIND == K_PAIR1) {
#define SX_PAIR(J)                                                   \
    {                                                                \
        const uint32_t cw = codeword<N, J, W16>(r, dp.wmask);        \
        const uint32_t p = cw * dp.mult;                             \
        q[J - 1] = p & dp.mask0;                                     \
        q[J] = rotl32(p, dp.rot) & dp.mask1;                         \
    }
        SX_PAIR(1) SX_PAIR(3) SX_PAIR(5) SX_PAIR(7)
#undef SX_PAIR
    } else {
        uint32_t cw[8];
        cw[0] = codeword<N, 0, W16>(r, dp.wmask);
        cw[1] = codeword<N, 1, W16>(r, dp.wmask);
        cw[2] = codeword<N, 2, W16>(r, dp.wmask);
        cw[3] = codeword<N, 3, W16>(r, dp.wmask);
        cw[4] = codeword<N, 4, W16>(r, dp.wmask);
        cw[5] = codeword<N, 5, W16>(r, dp.wmask);
        cw[6] = codeword<N, 6, W16>(r, dp.wmask);
        cw[7] = codeword<N, 7, W16>(r, dp.wmask);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if constexpr (KIND == K_MCG) {
                // dp carries MCG's multiplier, mask and xor (0xCBAC1FED, 0x8FFF8FFF, 0x3B603B60) as
                // run-time values: with two immediates the mask-and-xor would take two LOP3s.
                const uint32_t p = cw[j] * dp.mult;
                q[j] = (p & dp.mask0) ^ dp.mask1;
            } else if constexpr (KIND == K_HASH) {
                q[j] = (cw[j] * dp.mult) & dp.mask0;
            } else {  // MUL1: f16(fma(f16(0x6400 + bytesum(cw * M)), 0x1EEE, 0xC931))
                const uint32_t p = cw[j] * 0x83DCD12Du;
                const uint32_t h = __dp4a(p, 0x01010101u, 0x6400u);
                const float w = fmaf(h2f((uint16_t)h), h2f(0x1EEEu), h2f(0xC931u));
                q[j] = (uint32_t)f2h(w);
            }
        }
    }
}

// The same eight words, written straight into the two MMAs' A-register quads:
// a1 = {v0, v4, v1, v5} (inputs 2c, 2c+1 of outputs g, g+8), a2 = {v2, v6, v3, v7} (inputs
// 2c+8, 2c+9), so the quads need no register shuffling before the MMAs.
template <int KIND, int N, bool W16>
__device__ __forceinline__ void decode_lane_mma(const uint32_t* tile_words, const LaneFunnel<N>& lf, const DecParams& dp,
                                                uint32_t (&a1)[4], uint32_t (&a2)[4]) {
    uint32_t q[8];
    decode_lane_q<KIND, N, W16>(tile_words, lf, dp, q);
    a1[0] = q[0];
    a1[1] = q[4];
    a1[2] = q[1];
    a1[3] = q[5];
    a2[0] = q[2];
    a2[1] = q[6];
    a2[2] = q[3];
    a2[3] = q[7];
}

// Output scale of the doubled-k MMA: the hash-mask and PAIR1 weights are the half sum times 4096
// (src/exl3/expert_exl3.zig:292-296); MCG and MUL1 are the sum itself.
__host__ __device__ constexpr float kind_scale(int kind) { return (kind == K_HASH || kind == K_PAIR1) ? 4096.0f : 1.0f; }

// ------------------------------------------------------------------ exact (reference-order) decode
// The reference's per-codeword f16 arithmetic, for the bit-exact dequantisation kernel.
__device__ __forceinline__ uint16_t exact_half_sum_scaled(uint32_t halves) {
    const uint16_t sum = f2h(h2f((uint16_t)(halves & 0xFFFFu)) + h2f((uint16_t)(halves >> 16)));
    return f2h(h2f(sum) * 4096.0f);
}

template <int KIND>
__device__ __forceinline__ void exact_decode(uint32_t cw, uint32_t cw_next_odd, const DecParams& dp, int slot,
                                             uint16_t& out) {
    if constexpr (KIND == K_MCG) {
        const uint32_t p = cw * 0xCBAC1FEDu;
        const uint32_t pair = 0x3B603B60u ^ (p & 0x8FFF8FFFu);
        out = f2h(h2f((uint16_t)(pair & 0xFFFFu)) + h2f((uint16_t)(pair >> 16)));
    } else if constexpr (KIND == K_MUL1) {
        const uint32_t p = cw * 0x83DCD12Du;
        const uint32_t s = (p & 0xFFu) + ((p >> 8) & 0xFFu) + ((p >> 16) & 0xFFu) + (p >> 24);
        out = f2h(fmaf(h2f((uint16_t)(0x6400u + s)), h2f(0x1EEEu), h2f(0xC931u)));
    } else if constexpr (KIND == K_HASH) {
        out = exact_half_sum_scaled((cw * dp.mult) & dp.mask0);
    } else {
        const uint32_t p = cw_next_odd * dp.mult;
        out = slot == 0 ? exact_half_sum_scaled(p & dp.mask0) : exact_half_sum_scaled(rotl32(p, dp.rot) & dp.mask1);
    }
}

}  // namespace sx
