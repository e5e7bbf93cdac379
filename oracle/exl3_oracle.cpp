// CPU oracle for the EXL3 / STQ trellis hot path.  TEST INFRASTRUCTURE ONLY.
//
// This file restates, in plain C++, the reference's host decoder, its host projection, its CPU
// encoder and quantizer, its router chain and its f32-truth MoE slot, so the CUDA library can be
// checked against it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
// load it, and only as the checker: the product library (sushi_b200/libsushi_exl3_cuda.so) never
// links or calls it.
//
// Parity pin: every decoder function here is checked byte for byte against the reference's own
// committed fixtures (tests/golden/*.npz, extracted from src/exl3/fixtures and
// src/encoder/fixtures by tests/golden/make_golden.py) and against the known-answer codewords of
// src/exl3/expert_exl3.zig:661-860.
//
// Build: oracle/Makefile (g++ -O3 -ffp-contract=off: the reference's Zig arithmetic is strict IEEE
// with no implicit fused multiply-add, and every explicit @mulAdd is an fma here).

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <algorithm>
#include <limits>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---------------------------------------------------------------- f16 / bf16 conversion
// IEEE binary16 round-to-nearest-even, as Zig's @floatCast(f32 -> f16)
// (src/exl3/expert_exl3.zig:259-265).
inline uint16_t h_from_f(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax > 0x7F800000u) return (uint16_t)(sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
    if (ax >= 0x47800000u) return (uint16_t)(sign | 0x7C00u);
    if (ax < 0x33000000u) return (uint16_t)sign;
    uint32_t exp = ax >> 23;
    uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t h;
    if (exp >= 113) {
        h = ((exp - 112) << 10) | ((mant >> 13) & 0x3FFu);
        uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    } else {
        uint32_t sh = 126 - exp;
        uint32_t q = mant >> sh;
        uint32_t rem = mant & ((1u << sh) - 1u);
        uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        h = q;
    }
    return (uint16_t)(sign | h);
}

inline float f_from_h(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            // subnormal: m * 2^-24
            float v = (float)m * 5.9604644775390625e-08f;
            std::memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7F800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

inline float round_f16(float v) { return f_from_h(h_from_f(v)); }

inline uint16_t bf_from_f(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

inline float f_from_bf(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// ---------------------------------------------------------------- rates, codebooks
// src/exl3/expert_exl3.zig:4-11 (constants), :180-226 (Rate), :102-137 (Window).
constexpr int TILE = 16;
constexpr int TILE_VALUES = 256;
constexpr int HAD_DIM = 128;
constexpr float HAD_SCALE = 0.08838834764831845f;
constexpr uint32_t MCG_MULT = 0xCBAC1FEDu;
constexpr uint32_t MUL1_MULT = 0x83DCD12Du;

enum Codebook { CB_MUL1 = 0, CB_MCG = 1, CB_SPEC1 = 2, CB_PAIR1 = 3, CB_STD1 = 4 };

inline size_t bit_end(uint32_t n, size_t t) { return ((t + 1) * (size_t)n) >> 4; }
inline size_t fresh_bits(uint32_t n, size_t t) { return bit_end(n, t) - (t == 0 ? 0 : bit_end(n, t - 1)); }

struct Pair { uint32_t mult, rot, mask0, mask1; };

// PAIR1 rows, one per even n = 24..64 (src/exl3/expert_exl3.zig:24-46).
const Pair PAIR1_ROWS[21] = {
    {0x58F41BF3u, 3, 0x8ED78C13u, 0x8EEE8C03u},  {0x58F41BF3u, 3, 0x8ED78C13u, 0x8EEE8C03u},
    {0x7AA2BE15u, 3, 0x8ED78C13u, 0x8ECE8C03u},  {0x7B229E11u, 3, 0x8ED78C13u, 0x8ECE8C03u},
    {0x3B22BE15u, 3, 0x8ED78C13u, 0x8ECE8C03u},  {0x46C63E17u, 19, 0x8F9A8E6Eu, 0x8E258FFEu},
    {0x46C63E17u, 19, 0x8F9A8E6Eu, 0x8E258FFEu}, {0x46C63E17u, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0x46C63E17u, 19, 0x8F9A8E6Eu, 0x8E258FFEu}, {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu}, {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu}, {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu}, {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0x82439F67u, 19, 0x8E6E8F9Au, 0x8E258FAEu}, {0xE2C7FC0Du, 19, 0x8F408FB0u, 0x8F918F89u},
    {0xE2C7FC0Du, 19, 0x8F408FA0u, 0x8F118FC9u}, {0xE2C7FC0Du, 19, 0x8F408FA0u, 0x8F118FC9u},
    {0xE2C7FC0Du, 19, 0x8F408FA0u, 0x8F118FC9u},
};

// STD1 / SPEC1 tables (src/exl3/codebook_tables.zig:101-214), one (mult, mask) row per even n
// from n_lo.  Index order is the reference's `tables` order; index 0 (pair1-w16-v1) has no
// hash-mask rows.
struct HashTable { uint32_t n_lo; int rows; const uint32_t (*pairs)[2]; };

const uint32_t SPEC1_W15[57][2] = {
    {0x84d1cf89u, 0x8fe08947u}, {0x84c1cf49u, 0x8fe48a47u}, {0x84d1cfe9u, 0x8fe08a47u}, {0x84d1cfc9u, 0x8ff08b67u},
    {0x84c1cf49u, 0x8fe08b47u}, {0x84c1cf99u, 0x8fa08b66u}, {0x862c1d37u, 0x8ff28c50u}, {0x84641fb7u, 0x8fa08c40u},
    {0x846c1fa7u, 0x8fe08c80u}, {0x844c1fd7u, 0x8ffe8c98u}, {0x846c1fa7u, 0x8ffe8d10u}, {0x845c1f77u, 0x8ffa8e10u},
    {0x843c1fa7u, 0x8ffe8e40u}, {0x843c1fa7u, 0x8ffe8e40u}, {0x842c1fc7u, 0x8fff8f00u}, {0x843c1fb7u, 0x8ffe8f10u},
    {0x84181fb5u, 0x8fe08f80u}, {0x84081f75u, 0x8ffa8f72u}, {0x84081f75u, 0x8fd68fd0u}, {0x84241f27u, 0x8ffc8fc0u},
    {0x84081f73u, 0x8fe08f80u}, {0x84081f75u, 0x8fbe8ff0u}, {0x3fed4cefu, 0x8fe08fe0u}, {0x3fed4cefu, 0x8fc18ff2u},
    {0x3fed4cefu, 0x8ff08ff0u}, {0x3fed4cefu, 0x8fe28ff0u}, {0x3fed4cefu, 0x8fe08fe0u}, {0x80081b7bu, 0x8ff08fc8u},
    {0x80081b7bu, 0x8ff48fc0u}, {0x400036cbu, 0x8f448fffu}, {0x400036cbu, 0x8fe48fffu}, {0x400036cbu, 0x8f448ff9u},
    {0x8000387bu, 0x8fe08ff7u}, {0x8000387bu, 0x8fc08feeu}, {0x80003779u, 0x8fe88ffeu}, {0x80003779u, 0x8fc88ffcu},
    {0x80003779u, 0x8fca8ffcu}, {0x80003779u, 0x8fcc8ffeu}, {0x80003879u, 0x8ffc8fefu}, {0x50003851u, 0x8ff98fffu},
    {0xd0003751u, 0x8ff98fffu}, {0x50003851u, 0x8ff98ff6u}, {0xd0003931u, 0x8ff98fffu}, {0xd0003931u, 0x8ff98ffau},
    {0xd0003931u, 0x8ff48ffau}, {0x300031b1u, 0x8ffb8ffcu}, {0x300031b1u, 0x8ffa8ffeu}, {0x300031b1u, 0x8ffb8ffcu},
    {0xc00031f1u, 0x8ffe8ffau}, {0x400031f1u, 0x8ffe8ffeu}, {0x400031f1u, 0x8ffe8ffeu}, {0x40003931u, 0x8ffc8ffcu},
    {0x40003931u, 0x8ffc8ffcu}, {0x40003931u, 0x8ff88ffeu}, {0x40003931u, 0x8ff88ffcu}, {0x80003811u, 0x8ffc8ffcu},
    {0x80003811u, 0x8ffc8ffcu},
};

const uint32_t SPEC1_W16[21][2] = {
    {0x862d1c19u, 0x8fee8c30u}, {0x862d1d37u, 0x8fee8c30u}, {0x862d1d37u, 0x8ffe8c10u}, {0x842f1f37u, 0x8ffc8d10u},
    {0x840f1f67u, 0x8ffc8d10u}, {0x844f1f77u, 0x8ffe8d40u}, {0x840d1f37u, 0x8ffe8e10u}, {0x84091f33u, 0x8fe88e00u},
    {0x844d1f77u, 0x8fe08e00u}, {0x843c1fa7u, 0x8ffe8e40u}, {0x844c1f7fu, 0x8ffc8f02u}, {0x841c1fb9u, 0x8fe88f04u},
    {0x842c1fc7u, 0x8ffe8fd0u}, {0x83fc1fa3u, 0x8ffe8fd0u}, {0x83fc1fa3u, 0x8ffe8fc1u}, {0x83fc1fa3u, 0x8ffe8fd0u},
    {0x83fc1fa3u, 0x8fee8fc0u}, {0x84061f77u, 0x8fd08f80u}, {0x84081f6fu, 0x8ffe8fc0u}, {0x84081f25u, 0x8ffe8fe0u},
    {0x83f81f6fu, 0x8ff48fc0u},
};

uint32_t STD1_ROWS[21][2];
uint32_t SPEC1_TEST[57][2];

struct TablesInit {
    TablesInit() {
        for (int i = 0; i < 21; i++) { STD1_ROWS[i][0] = 0x840C1F37u; STD1_ROWS[i][1] = 0x8FFE8FD0u; }
        // src/exl3/codebook_tables.zig:209-214 (the test-only per-rate table).
        const uint32_t masks[4] = {0x8FFE8FD0u, 0x8FE08FC0u, 0x8FF08FE0u, 0x8F8E8FD8u};
        for (uint32_t i = 0; i < 57; i++) {
            SPEC1_TEST[i][0] = 0x840C1F37u + (16u + 2u * i) * 0x2E0B5u;
            SPEC1_TEST[i][1] = masks[i % 4];
        }
    }
} tables_init;

// Table index: 0 pair1-w16-v1, 1 spec1-w15, 2 spec1-w16, 3 std1, 4 spec1-test-per-rate.
bool hash_row(int table, uint32_t n, uint32_t* mult, uint32_t* mask) {
    uint32_t n_lo; int rows; const uint32_t (*p)[2];
    switch (table) {
        case 1: n_lo = 16; rows = 57; p = SPEC1_W15; break;
        case 2: n_lo = 24; rows = 21; p = SPEC1_W16; break;
        case 3: n_lo = 24; rows = 21; p = STD1_ROWS; break;
        case 4: n_lo = 16; rows = 57; p = SPEC1_TEST; break;
        default: return false;
    }
    if (n % 2 != 0 || n < n_lo) return false;
    uint32_t i = (n - n_lo) / 2;
    if ((int)i >= rows) return false;
    *mult = p[i][0];
    *mask = p[i][1];
    return true;
}

bool pair1_row(uint32_t n, Pair* out) {
    if (n % 2 != 0 || n < 24 || n > 64) return false;
    *out = PAIR1_ROWS[(n - 24) / 2];
    return true;
}

// src/exl3/expert_exl3.zig:267-273
uint16_t decode_mcg(uint16_t cw) {
    uint32_t mixed = (uint32_t)cw * MCG_MULT;
    uint32_t pair = 0x3B603B60u ^ (mixed & 0x8FFF8FFFu);
    float lo = f_from_h((uint16_t)(pair & 0xFFFFu));
    float hi = f_from_h((uint16_t)(pair >> 16));
    return h_from_f(lo + hi);
}

// src/exl3/expert_exl3.zig:275-284
uint16_t decode_mul1(uint16_t cw) {
    uint32_t mixed = (uint32_t)cw * MUL1_MULT;
    uint32_t s = (mixed & 0xFFu) + ((mixed >> 8) & 0xFFu) + ((mixed >> 16) & 0xFFu) + (mixed >> 24);
    float h = f_from_h((uint16_t)(0x6400u + s));
    float inverse = f_from_h(0x1EEEu);
    float bias = f_from_h(0xC931u);
    return h_from_f(std::fma(h, inverse, bias));
}

// src/exl3/expert_exl3.zig:292-296
uint16_t half_sum_scaled(uint32_t halves, uint32_t scale) {
    uint16_t sum = h_from_f(f_from_h((uint16_t)(halves & 0xFFFFu)) + f_from_h((uint16_t)(halves >> 16)));
    return h_from_f(f_from_h(sum) * (float)scale);
}

// src/exl3/expert_exl3.zig:288-290
uint16_t decode_hash_mask(uint16_t cw, uint32_t mult, uint32_t mask) {
    return half_sum_scaled(((uint32_t)cw * mult) & mask, 4096u);
}

inline uint32_t rotl32(uint32_t v, uint32_t r) { r &= 31u; return r ? (v << r) | (v >> (32u - r)) : v; }

// src/exl3/expert_exl3.zig:298-301
void decode_pair(uint16_t cw, const Pair& p, uint16_t out[2]) {
    uint32_t product = (uint32_t)cw * p.mult;
    out[0] = half_sum_scaled(product & p.mask0, 4096u);
    out[1] = half_sum_scaled(rotl32(product, p.rot) & p.mask1, 4096u);
}

inline uint32_t word_u32(const uint16_t* words, size_t index) {
    return (uint32_t)words[index * 2] | ((uint32_t)words[index * 2 + 1] << 16);
}

// src/exl3/expert_exl3.zig:317-336
void unpack_tile(const uint16_t* words, uint32_t n, uint16_t out[TILE_VALUES]) {
    size_t word_count = n / 2;
    size_t total = (size_t)TILE * n;
    for (size_t thread = 0; thread < 128; thread++) {
        size_t e0 = bit_end(n, thread * 2);
        size_t e1 = bit_end(n, thread * 2 + 1);
        size_t bit0 = e0 + total - 16;
        size_t bit2 = e1 + total;
        size_t index0 = bit0 / 32;
        size_t index1 = (bit2 - 1) / 32;
        unsigned shift = (unsigned)((index1 + 1) * 32 - bit2);
        uint64_t merged = ((uint64_t)word_u32(words, index0 % word_count) << 32) |
                          (uint64_t)word_u32(words, index1 % word_count);
        uint32_t funnel = (uint32_t)(merged >> shift);
        unsigned fresh = (unsigned)(e1 - e0);
        out[thread * 2] = (uint16_t)((funnel >> fresh) & 0xFFFFu);
        out[thread * 2 + 1] = (uint16_t)(funnel & 0xFFFFu);
    }
}

// src/exl3/expert_exl3.zig:379-398
void tensor_core_perm(size_t out[TILE_VALUES]) {
    for (size_t thread = 0; thread < 32; thread++) {
        size_t row0 = (thread % 4) * 2, row1 = row0 + 1, row2 = row0 + 8, row3 = row0 + 9;
        size_t col0 = thread / 4, col1 = col0 + 8;
        size_t base = thread * 8;
        out[base + 0] = row0 * 16 + col0;
        out[base + 1] = row1 * 16 + col0;
        out[base + 2] = row2 * 16 + col0;
        out[base + 3] = row3 * 16 + col0;
        out[base + 4] = row0 * 16 + col1;
        out[base + 5] = row1 * 16 + col1;
        out[base + 6] = row2 * 16 + col1;
        out[base + 7] = row3 * 16 + col1;
    }
}

struct Perm { size_t p[TILE_VALUES]; Perm() { tensor_core_perm(p); } } const PERM;

struct Dec { int codebook; int window_bits; int table; };

inline uint16_t window_mask(int bits) { return (uint16_t)(((uint32_t)1 << bits) - 1u); }

// src/exl3/expert_exl3.zig:338-357.  Returns 0, or -1 for a decode without a row at this rate.
int decode_tile(const uint16_t* words, uint32_t n, const Dec& dec, uint16_t out[TILE_VALUES]) {
    uint16_t cws[TILE_VALUES];
    unpack_tile(words, n, cws);
    uint16_t mask = window_mask(dec.window_bits);
    if (dec.codebook == CB_PAIR1) {
        Pair p;
        if (!pair1_row(n, &p)) return -1;
        for (int j = 0; j < TILE_VALUES / 2; j++) {
            uint16_t w[2];
            decode_pair((uint16_t)(cws[2 * j + 1] & mask), p, w);
            out[PERM.p[2 * j]] = w[0];
            out[PERM.p[2 * j + 1]] = w[1];
        }
        return 0;
    }
    if (dec.codebook == CB_SPEC1 || dec.codebook == CB_STD1) {
        uint32_t mult, hmask;
        if (!hash_row(dec.table, n, &mult, &hmask)) return -1;
        for (int i = 0; i < TILE_VALUES; i++) out[PERM.p[i]] = decode_hash_mask((uint16_t)(cws[i] & mask), mult, hmask);
        return 0;
    }
    for (int i = 0; i < TILE_VALUES; i++) {
        uint16_t cw = (uint16_t)(cws[i] & mask);
        out[PERM.p[i]] = dec.codebook == CB_MCG ? decode_mcg(cw) : decode_mul1(cw);
    }
    return 0;
}

// src/exl3/expert_exl3.zig:400-414: the dense Sylvester product, accumulated in index order.
inline float hadamard_entry(size_t r, size_t c) {
    return (__builtin_popcountll(r & c) % 2 == 0) ? HAD_SCALE : -HAD_SCALE;
}

struct HadTable { float h[HAD_DIM][HAD_DIM]; HadTable() { for (int r = 0; r < HAD_DIM; r++) for (int c = 0; c < HAD_DIM; c++) h[r][c] = hadamard_entry(r, c); } } const HAD;

void hadamard128(float* v) {
    float tmp[HAD_DIM];
    for (int r = 0; r < HAD_DIM; r++) {
        float acc = 0.0f;
        for (int k = 0; k < HAD_DIM; k++) acc += HAD.h[r][k] * v[k];
        tmp[r] = acc;
    }
    std::memcpy(v, tmp, sizeof(tmp));
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- conversions
uint16_t orc_f32_to_f16(float v) { return h_from_f(v); }
float orc_f16_to_f32(uint16_t h) { return f_from_h(h); }
void orc_f32_to_f16_n(const float* src, uint16_t* dst, size_t n) { for (size_t i = 0; i < n; i++) dst[i] = h_from_f(src[i]); }
void orc_f16_to_f32_n(const uint16_t* src, float* dst, size_t n) { for (size_t i = 0; i < n; i++) dst[i] = f_from_h(src[i]); }
void orc_f32_to_bf16_n(const float* src, uint16_t* dst, size_t n) { for (size_t i = 0; i < n; i++) dst[i] = bf_from_f(src[i]); }

// ---------------------------------------------------------------- decode
size_t orc_bit_end(uint32_t n, size_t t) { return bit_end(n, t); }
size_t orc_fresh_bits(uint32_t n, size_t t) { return fresh_bits(n, t); }
uint16_t orc_decode_mcg(uint16_t cw) { return decode_mcg(cw); }
uint16_t orc_decode_mul1(uint16_t cw) { return decode_mul1(cw); }
uint16_t orc_decode_hash_mask(uint16_t cw, uint32_t mult, uint32_t mask) { return decode_hash_mask(cw, mult, mask); }
int orc_pair1_row(uint32_t n, uint32_t out[4]) {
    Pair p;
    if (!pair1_row(n, &p)) return -1;
    out[0] = p.mult; out[1] = p.rot; out[2] = p.mask0; out[3] = p.mask1;
    return 0;
}
int orc_hash_row(int table, uint32_t n, uint32_t out[2]) { return hash_row(table, n, &out[0], &out[1]) ? 0 : -1; }
int orc_decode_pair(uint16_t cw, uint32_t n, uint16_t out[2]) {
    Pair p;
    if (!pair1_row(n, &p)) return -1;
    decode_pair(cw, p, out);
    return 0;
}
void orc_unpack_tile(const uint16_t* words, uint32_t n, uint16_t* out) { unpack_tile(words, n, out); }

// Every codeword's decode at rate n (window-masked first): out32[cw] = weight bits, and for PAIR1
// weight 2j's bits low and 2j+1's high (the layout firstPair1PairMismatch reads,
// src/exl3/expert_exl3.zig:359-369).  Returns -1 for a decode without a row at this rate.
int orc_decode_all(int codebook, uint32_t n, int window_bits, int table, uint32_t* out32) {
    const uint16_t mask = window_mask(window_bits);
    Pair p{};
    uint32_t mult = 0, hmask = 0;
    if (codebook == CB_PAIR1 && !pair1_row(n, &p)) return -1;
    if ((codebook == CB_SPEC1 || codebook == CB_STD1) && !hash_row(table, n, &mult, &hmask)) return -1;
    for (uint32_t cw = 0; cw < 65536u; cw++) {
        const uint16_t m = (uint16_t)(cw & mask);
        if (codebook == CB_PAIR1) {
            uint16_t w[2];
            decode_pair(m, p, w);
            out32[cw] = (uint32_t)w[0] | ((uint32_t)w[1] << 16);
        } else if (codebook == CB_SPEC1 || codebook == CB_STD1) {
            out32[cw] = decode_hash_mask(m, mult, hmask);
        } else {
            out32[cw] = codebook == CB_MCG ? decode_mcg(m) : decode_mul1(m);
        }
    }
    return 0;
}
void orc_tensor_core_perm(int64_t* out) { for (int i = 0; i < TILE_VALUES; i++) out[i] = (int64_t)PERM.p[i]; }
int orc_decode_tile(const uint16_t* words, uint32_t n, int codebook, int window_bits, int table, uint16_t* out) {
    return decode_tile(words, n, Dec{codebook, window_bits, table}, out);
}
void orc_hadamard128(float* v) { hadamard128(v); }

// src/exl3/expert_exl3.zig:416-438.  trellis [in/16, out/16, n]; out [in, out] f16 bits.
int orc_reconstruct_inner(const uint16_t* trellis, size_t in, size_t out, uint32_t n, int codebook, int window_bits,
                          int table, uint16_t* dst) {
    const Dec dec{codebook, window_bits, table};
    size_t it = in / TILE, ot = out / TILE;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (long long tk = 0; tk < (long long)it; tk++) {
        uint16_t tile[TILE_VALUES];
        for (size_t tn = 0; tn < ot; tn++) {
            size_t off = ((size_t)tk * ot + tn) * n;
            if (decode_tile(trellis + off, n, dec, tile) != 0) { bad = 1; continue; }
            for (int r = 0; r < TILE; r++)
                std::memcpy(dst + ((size_t)tk * TILE + r) * out + tn * TILE, tile + r * TILE, TILE * sizeof(uint16_t));
        }
    }
    return bad ? -1 : 0;
}

// src/exl3/expert_exl3.zig:440-488.  public [in, out] f16 bits.
int orc_reconstruct_public(const uint16_t* trellis, const uint16_t* suh, const uint16_t* svh, size_t in, size_t out,
                           uint32_t n, int codebook, int window_bits, int table, uint16_t* dst) {
    std::vector<uint16_t> inner(in * out);
    if (orc_reconstruct_inner(trellis, in, out, n, codebook, window_bits, table, inner.data()) != 0) return -1;
    std::vector<float> w(in * out);
    for (size_t i = 0; i < in * out; i++) w[i] = f_from_h(inner[i]);
    for (size_t rb = 0; rb < in; rb += HAD_DIM) {
        for (size_t col = 0; col < out; col++) {
            float vec[HAD_DIM];
            for (int r = 0; r < HAD_DIM; r++) vec[r] = w[(rb + r) * out + col];
            hadamard128(vec);
            for (int r = 0; r < HAD_DIM; r++) w[(rb + r) * out + col] = vec[r];
        }
    }
    for (size_t r = 0; r < in; r++) {
        float s = f_from_h(suh[r]);
        for (size_t c = 0; c < out; c++) w[r * out + c] *= s;
    }
    for (size_t cb = 0; cb < out; cb += HAD_DIM) {
        for (size_t r = 0; r < in; r++) {
            float vec[HAD_DIM];
            for (int c = 0; c < HAD_DIM; c++) vec[c] = w[r * out + cb + c];
            hadamard128(vec);
            for (int c = 0; c < HAD_DIM; c++) w[r * out + cb + c] = vec[c];
        }
    }
    for (size_t c = 0; c < out; c++) {
        float s = f_from_h(svh[c]);
        for (size_t r = 0; r < in; r++) w[r * out + c] *= s;
    }
    for (size_t i = 0; i < in * out; i++) dst[i] = h_from_f(w[i]);
    return 0;
}

// src/exl3/linear.zig:406-431: the dense f32 twin W [in, out].
int orc_decode_dense(const uint16_t* trellis, const uint16_t* suh, const uint16_t* svh, size_t in, size_t out,
                     uint32_t n, int codebook, int window_bits, int table, float* dst) {
    const Dec dec{codebook, window_bits, table};
    size_t ot = out / TILE;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (long long tk = 0; tk < (long long)(in / TILE); tk++) {
        uint16_t tile[TILE_VALUES];
        for (size_t tn = 0; tn < ot; tn++) {
            if (decode_tile(trellis + ((size_t)tk * ot + tn) * n, n, dec, tile) != 0) { bad = 1; continue; }
            for (int r = 0; r < 16; r++)
                for (int c = 0; c < 16; c++) dst[((size_t)tk * 16 + r) * out + tn * 16 + c] = f_from_h(tile[r * 16 + c]);
        }
    }
    if (bad) return -1;
#pragma omp parallel for schedule(static)
    for (long long j = 0; j < (long long)out; j++) {
        float col[HAD_DIM];
        for (size_t b = 0; b < in; b += HAD_DIM) {
            for (int i = 0; i < HAD_DIM; i++) col[i] = dst[(b + i) * out + j];
            hadamard128(col);
            for (int i = 0; i < HAD_DIM; i++) dst[(b + i) * out + j] = col[i];
        }
    }
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)in; i++) {
        float* row = dst + (size_t)i * out;
        for (size_t o = 0; o < out; o += HAD_DIM) hadamard128(row + o);
        float su = f_from_h(suh[i]);
        for (size_t o = 0; o < out; o++) row[o] *= su * f_from_h(svh[o]);
    }
    return 0;
}

// src/exl3/expert_exl3.zig:490-501
void orc_prepare_input(const float* x, const uint16_t* suh, size_t in, float* dst) {
    for (size_t i = 0; i < in; i++) dst[i] = round_f16(x[i]) * f_from_h(suh[i]);
    for (size_t b = 0; b < in; b += HAD_DIM) {
        float vec[HAD_DIM];
        std::memcpy(vec, dst + b, sizeof(vec));
        hadamard128(vec);
        for (int i = 0; i < HAD_DIM; i++) dst[b + i] = round_f16(vec[i]);
    }
}

// src/exl3/expert_exl3.zig:503-532 (tk outer, tn inner, f32 accumulate, f16-rounded result).
int orc_inner_gemv(const uint16_t* trellis, const float* transformed, size_t in, size_t out, uint32_t n, int codebook,
                   int window_bits, int table, float* dst) {
    const Dec dec{codebook, window_bits, table};
    size_t it = in / TILE, ot = out / TILE;
    std::memset(dst, 0, out * sizeof(float));
    uint16_t tile[TILE_VALUES];
    for (size_t tk = 0; tk < it; tk++) {
        for (size_t tn = 0; tn < ot; tn++) {
            if (decode_tile(trellis + (tk * ot + tn) * n, n, dec, tile) != 0) return -1;
            for (int r = 0; r < TILE; r++) {
                float xv = transformed[tk * TILE + r];
                for (int c = 0; c < TILE; c++) dst[tn * TILE + c] += xv * f_from_h(tile[r * TILE + c]);
            }
        }
    }
    for (size_t o = 0; o < out; o++) dst[o] = round_f16(dst[o]);
    return 0;
}

// src/exl3/expert_exl3.zig:534-544
void orc_finish_output(const float* inner, const uint16_t* svh, size_t out, float* dst) {
    std::memcpy(dst, inner, out * sizeof(float));
    for (size_t b = 0; b < out; b += HAD_DIM) hadamard128(dst + b);
    for (size_t o = 0; o < out; o++) dst[o] = round_f16(dst[o] * f_from_h(svh[o]));
}

// src/exl3/expert_exl3.zig:546-566: the reference's CPU decode + matmul, one row.
int orc_project(const float* x, const uint16_t* trellis, const uint16_t* suh, const uint16_t* svh, size_t in, size_t out,
                uint32_t n, int codebook, int window_bits, int table, float* y) {
    std::vector<float> t(in), inner(out);
    orc_prepare_input(x, suh, in, t.data());
    if (orc_inner_gemv(trellis, t.data(), in, out, n, codebook, window_bits, table, inner.data()) != 0) return -1;
    orc_finish_output(inner.data(), svh, out, y);
    return 0;
}

// `orc_project` over `rows` rows, the rows split across threads (one row per task).
int orc_project_rows(const float* x, size_t rows, const uint16_t* trellis, const uint16_t* suh, const uint16_t* svh,
                     size_t in, size_t out, uint32_t n, int codebook, int window_bits, int table, float* y) {
    int bad = 0;
#pragma omp parallel for schedule(dynamic) reduction(| : bad)
    for (long long r = 0; r < (long long)rows; r++)
        bad |= orc_project(x + (size_t)r * in, trellis, suh, svh, in, out, n, codebook, window_bits, table, y + (size_t)r * out) != 0;
    return bad ? -1 : 0;
}

// `orc_project` for one row with the tile loop split by output-tile ranges across threads:
// each thread owns whole output tiles, so every output keeps the reference's tk-ordered
// accumulation and the result is identical to the single-thread call.
int orc_project_mt(const float* x, const uint16_t* trellis, const uint16_t* suh, const uint16_t* svh, size_t in, size_t out,
                   uint32_t n, int codebook, int window_bits, int table, float* y) {
    const Dec dec{codebook, window_bits, table};
    std::vector<float> t(in), inner(out, 0.0f);
    orc_prepare_input(x, suh, in, t.data());
    size_t it = in / TILE, ot = out / TILE;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (long long tn = 0; tn < (long long)ot; tn++) {
        uint16_t tile[TILE_VALUES];
        float acc[TILE] = {0};
        for (size_t tk = 0; tk < it; tk++) {
            if (decode_tile(trellis + (tk * ot + (size_t)tn) * n, n, dec, tile) != 0) { bad = 1; break; }
            for (int r = 0; r < TILE; r++) {
                float xv = t[tk * TILE + r];
                for (int c = 0; c < TILE; c++) acc[c] += xv * f_from_h(tile[r * TILE + c]);
            }
        }
        for (int c = 0; c < TILE; c++) inner[(size_t)tn * TILE + c] = round_f16(acc[c]);
    }
    if (bad) return -1;
    orc_finish_output(inner.data(), svh, out, y);
    return 0;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    omp_set_num_threads(n);
#else
    (void)n;
#endif
}

// src/exl3/layout.zig:141-150: pack order [IT][OT][n] -> pair-major [OT/2][IT][2][n].
void orc_tile_major(const uint16_t* src, uint16_t* dst, size_t it, size_t ot, size_t n) {
    for (size_t pair = 0; pair < ot / 2; pair++)
        for (size_t tk = 0; tk < it; tk++)
            for (size_t o = 0; o < 2; o++)
                std::memcpy(dst + ((pair * it + tk) * 2 + o) * n, src + (tk * ot + pair * 2 + o) * n, n * sizeof(uint16_t));
}

}  // extern "C"
