// CPU encoder and quantizer restatement.  TEST INFRASTRUCTURE ONLY (fixture generator).
//
// Restates the reference's tail-biting Viterbi tile search (src/encoder/encode.zig:132-295) and
// its tensor quantizer (src/encoder/quantize.zig:33-666: regularize, rotatedHessian, ldlFactor,
// globalScale, ldlq, signs, quantizeNamed).  It turns a seeded public weight into the
// (trellis, suh, svh) pack the CUDA library reads, so the parity tests and the bench run on
// packs the reference's own encoder would write.  Pinned byte for byte against
// src/encoder/fixtures/exl3_encode_tiles.safetensors and exl3_encode_tensor.safetensors
// (tests/golden/exl3_encode_*.npz).
//
// Arithmetic follows the Zig source operation for operation: f32 where it is f32, f64 where it
// is f64, explicit fma only where the source writes @mulAdd, path costs stored as f16 between
// Viterbi steps, first minimum wins every tie.

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <algorithm>
#include <functional>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {
uint16_t orc_f32_to_f16(float v);
float orc_f16_to_f32(uint16_t h);
uint16_t orc_decode_mcg(uint16_t cw);
uint16_t orc_decode_mul1(uint16_t cw);
size_t orc_fresh_bits(uint32_t n, size_t t);
size_t orc_bit_end(uint32_t n, size_t t);
void orc_tensor_core_perm(int64_t* out);
}

namespace {

constexpr int TILE_LEN = 256;
constexpr int HAD = 128;
constexpr float SIGMA_REG = 0.025f;
constexpr float CODEBOOK_SCALE = 1.24371088f;

inline float f16_round(float v) { return (float)(_Float16)v; }

struct Encoder {
    uint32_t n;
    int codebook;  // 0 mul1, 1 mcg
    int w;
    size_t stride;
    std::vector<float> table;
    std::vector<float> costs[2];
    std::vector<uint8_t> back;
    uint8_t ks[TILE_LEN];
    int64_t perm[TILE_LEN];
    float x[TILE_LEN];
    uint16_t path[TILE_LEN];
    std::vector<float> best;
    std::vector<uint8_t> bfresh;

    // src/encoder/encode.zig:132-165.  Returns 0 or a negative refusal.
    int init(uint32_t n_, int codebook_, int window_bits) {
        if (codebook_ != 0 && codebook_ != 1) return -5;            // CodebookUnsupported
        if (n_ % 2 != 0 || n_ < 16 || n_ > 128) return -1;         // RateUnsupported
        if (window_bits < 12 || window_bits > 16) return -3;        // WindowUnsupported
        n = n_;
        codebook = codebook_;
        w = window_bits;
        int kmin = 31, kmax = 0;
        for (int t = 0; t < TILE_LEN; t++) {
            ks[t] = (uint8_t)orc_fresh_bits(n, (size_t)t);
            kmin = std::min(kmin, (int)ks[t]);
            kmax = std::max(kmax, (int)ks[t]);
        }
        if (kmax >= w) return -2;                                   // WindowTooNarrow
        orc_tensor_core_perm(perm);
        stride = (size_t)1 << (w - kmin);
        table.resize((size_t)1 << w);
        for (size_t cw = 0; cw < table.size(); cw++)
            table[cw] = orc_f16_to_f32(codebook == 1 ? orc_decode_mcg((uint16_t)cw) : orc_decode_mul1((uint16_t)cw));
        costs[0].assign(stride, 0.0f);
        costs[1].assign(stride, 0.0f);
        back.assign((size_t)TILE_LEN * stride, 0);
        best.assign(stride, 0.0f);
        bfresh.assign(stride, 0);
        for (auto& row : tab_t)
            for (auto& t : row) t.clear();
        return 0;
    }

    // One Viterbi step after the first, for every edge: the reference's per-edge loop over
    // fresh bits, run fresh-outer so the edge loop vectorises.  Each edge still visits fresh
    // values in ascending order with a strict `<`, so best and back are the reference's.
    // Edges are walked as e = (p << k) | r with the codebook table pre-permuted to
    // [fresh][r][p], so both the table and the predecessor cost (index (fresh << (kr-k)) | p)
    // are read contiguously.
    std::vector<float> tab_t[9][9];
    std::vector<float> best_t;
    std::vector<uint32_t> bf_t;

    const float* permuted_table(int k, int k_next) {
        std::vector<float>& t = tab_t[k][k_next];
        if (t.empty()) {
            const int kr = w - k_next;
            const size_t kk = (size_t)1 << k_next, R = (size_t)1 << k, P = (size_t)1 << (kr - k);
            t.resize(kk * R * P);
            for (size_t f = 0; f < kk; f++)
                for (size_t r = 0; r < R; r++)
                    for (size_t p = 0; p < P; p++) t[(f * R + r) * P + p] = table[(f << kr) | (p << k) | r];
        }
        return t.data();
    }

    void step_rest(float* prev, float* curr, uint8_t* back_row, int k, int k_next, float target) {
        const int kr = w - k_next;
        const size_t kk = (size_t)1 << k_next;
        const size_t edges = (size_t)1 << kr;
        if (kr >= k) {
            const size_t R = (size_t)1 << k, P = (size_t)1 << (kr - k);
            const float* tt = permuted_table(k, k_next);
            if (best_t.size() < edges) {
                best_t.resize(edges);
                bf_t.resize(edges);
            }
            float* bst = best_t.data();
            uint32_t* bf = bf_t.data();
            for (size_t e = 0; e < edges; e++) { bst[e] = 65504.0f; bf[e] = 0; }
            for (size_t fresh = 0; fresh < kk; fresh++) {
                const float* pv = prev + (fresh << (kr - k));
                for (size_t r = 0; r < R; r++) {
                    const float* tab = tt + (fresh * R + r) * P;
                    float* b = bst + r * P;
                    uint32_t* bb = bf + r * P;
                    for (size_t p = 0; p < P; p++) {
                        const float dh = tab[p] - target;
                        const float err = std::fma(dh, dh, pv[p]);
                        const bool take = err < b[p];
                        b[p] = take ? err : b[p];
                        bb[p] = take ? (uint32_t)fresh : bb[p];
                    }
                }
            }
            for (size_t r = 0; r < R; r++)
                for (size_t p = 0; p < P; p++) {
                    const size_t e = (p << k) | r;
                    curr[e] = f16_round(bst[r * P + p]);
                    back_row[e] = (uint8_t)bf[r * P + p];
                }
            return;
        }
        float* bst = best.data();
        uint8_t* bf = bfresh.data();
        for (size_t e = 0; e < edges; e++) { bst[e] = 65504.0f; bf[e] = 0; }
        for (size_t fresh = 0; fresh < kk; fresh++) {
            const float* tab = table.data() + (fresh << kr);
            for (size_t e = 0; e < edges; e++) {
                const size_t cw = (fresh << kr) | e;
                const float dh = tab[e] - target;
                const float err = std::fma(dh, dh, prev[cw >> k]);
                if (err < bst[e]) { bst[e] = err; bf[e] = (uint8_t)fresh; }
            }
        }
        for (size_t e = 0; e < edges; e++) {
            curr[e] = f16_round(bst[e]);
            back_row[e] = bf[e];
        }
    }

    // src/encoder/encode.zig:173-260
    double encode_tile(const float* tile, uint16_t* packed_out, float* recon) {
        for (int i = 0; i < TILE_LEN; i++) x[i] = tile[perm[i]];
        const float h_inf = 65504.0f;
        size_t pin = 0;
        bool pinned = false;
        for (int pass = 0; pass < 2; pass++) {
            const int roll = pass == 0 ? TILE_LEN / 2 : 0;
            float* prev = costs[0].data();
            float* curr = costs[1].data();
            for (int step = 0; step < TILE_LEN; step++) {
                const int ri = (step + roll) & (TILE_LEN - 1);
                const int k = ks[ri];
                const int k_next = ks[(ri + 1) & (TILE_LEN - 1)];
                const int kr = w - k_next;
                const size_t kk = (size_t)1 << k_next;
                const size_t edges = (size_t)1 << kr;
                const float target = x[ri];
                uint8_t* back_row = back.data() + (size_t)ri * stride;
                if (step == 0) {
                    for (size_t e = 0; e < edges; e++) {
                        float bst = h_inf;
                        uint8_t bfr = 0;
                        for (size_t fresh = 0; fresh < kk; fresh++) {
                            size_t cw = (fresh << kr) | e;
                            size_t pred = cw >> k;
                            float err;
                            if (pinned && pred != pin) {
                                err = h_inf;
                            } else {
                                float dh = table[cw] - target;
                                err = std::min(dh * dh, h_inf);
                            }
                            if (err < bst) { bst = err; bfr = (uint8_t)fresh; }
                        }
                        curr[e] = f16_round(bst);
                        back_row[e] = bfr;
                    }
                } else {
                    step_rest(prev, curr, back_row, k, k_next, target);
                }
                std::swap(prev, curr);
            }
            size_t edge = pin;
            if (pass == 0) {
                const int k0 = ks[0];
                const size_t final_edges = (size_t)1 << (w - k0);
                float bst = h_inf;
                edge = 0;
                for (size_t e = 0; e < final_edges; e++) {
                    if (prev[e] < bst) { bst = prev[e]; edge = e; }
                }
            }
            int step_i = TILE_LEN;
            while (step_i > 0) {
                step_i -= 1;
                const int ri = (step_i + roll) & (TILE_LEN - 1);
                const int k = ks[ri];
                const int k_next = ks[(ri + 1) & (TILE_LEN - 1)];
                const int kr = w - k_next;
                const size_t bfr = back[(size_t)ri * stride + edge];
                const size_t state = (bfr << kr) | edge;
                edge = state >> k;
                if (pass == 1) {
                    path[ri] = (uint16_t)state;
                } else if (ri == 0) {
                    break;
                }
            }
            pin = edge;
            pinned = true;
        }
        pack_states(packed_out);
        double sse = 0;
        for (int i = 0; i < TILE_LEN; i++) {
            double d = (double)x[i] - (double)table[path[i]];
            sse += d * d;
        }
        if (recon) for (int i = 0; i < TILE_LEN; i++) recon[perm[i]] = table[path[i]];
        return sse;
    }

    // src/encoder/encode.zig:278-290
    void pack_states(uint16_t* out) const {
        std::memset(out, 0, n * sizeof(uint16_t));
        for (int t = 0; t < TILE_LEN; t++) {
            const int k = ks[t];
            const size_t end = orc_bit_end(n, (size_t)t);
            const uint16_t cw = path[t];
            for (int b = 0; b < k; b++) {
                const uint16_t bit = (uint16_t)((cw >> (k - 1 - b)) & 1u);
                const size_t p = end - (size_t)k + (size_t)b;
                const size_t half_index = (p / 32) * 2 + (p % 32 < 16 ? 1 : 0);
                out[half_index] |= (uint16_t)(bit << (15 - (p % 16)));
            }
        }
    }
};

// ------------------------------------------------------------------ quantize.zig restatement
template <typename T>
void fwht(T* v) {
    for (int h = 1; h < HAD; h *= 2)
        for (int i = 0; i < HAD; i += 2 * h)
            for (int j = i; j < i + h; j++) {
                T a = v[j], b = v[j + h];
                v[j] = a + b;
                v[j + h] = a - b;
            }
    const T scale = (T)1.0 / std::sqrt((T)HAD);
    for (int i = 0; i < HAD; i++) v[i] *= scale;
}

template <typename T>
void hadamard_rows(T* m, size_t rows, size_t cols) {
    const T scale = (T)1.0 / std::sqrt((T)HAD);
    for (size_t b = 0; b < rows; b += HAD) {
        T* blk = m + b * cols;
        for (int h = 1; h < HAD; h *= 2)
            for (int i = 0; i < HAD; i += 2 * h)
                for (int j = i; j < i + h; j++) {
                    T* x = blk + (size_t)j * cols;
                    T* y = blk + (size_t)(j + h) * cols;
                    for (size_t c = 0; c < cols; c++) {
                        T a = x[c], d = y[c];
                        x[c] = a + d;
                        y[c] = a - d;
                    }
                }
        for (size_t i = 0; i < (size_t)HAD * cols; i++) blk[i] *= scale;
    }
}

template <typename T>
void hadamard_cols(T* m, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; r++)
        for (size_t b = 0; b < cols; b += HAD) fwht(m + r * cols + b);
}

inline float block_rms(float sq, size_t n) { return std::sqrt(sq / (float)n); }

// src/encoder/quantize.zig:94-119; mode 0 auto, 1 always, 2 never.
bool choose_apply_out_scales(int mode, const float* hdiag, size_t len) {
    int forced = mode == 0 ? -1 : (mode == 1 ? 1 : 0);
    if (!hdiag) return forced >= 0 ? forced == 1 : true;
    double sum = 0;
    for (size_t i = 0; i < len; i++) sum += std::max(hdiag[i], 0.0f);
    double mean = sum / (double)len;
    if (!std::isfinite(mean) || mean < 1e-20) return forced >= 0 ? forced == 1 : false;
    if (forced >= 0) return forced == 1;
    std::vector<float> diag(len);
    const float damp = (float)((double)SIGMA_REG * mean);
    for (size_t i = 0; i < len; i++) diag[i] = std::sqrt(std::max(hdiag[i], 0.0f) + damp);
    std::sort(diag.begin(), diag.end(), std::greater<float>());
    size_t cutoff = std::max<size_t>(1, len / 50);
    double top = 0, all = 0;
    for (size_t i = 0; i < len; i++) {
        if (i < cutoff) top += diag[i];
        all += diag[i];
    }
    return top / all < 0.15;
}

// src/encoder/quantize.zig:133-196
void regularize(const float* w, size_t in, size_t out, const float* sign_in, const float* sign_out, int mode,
                const float* hdiag, std::vector<float>& weight, std::vector<float>& suh, std::vector<float>& svh) {
    weight.assign(w, w + in * out);
    suh.assign(in, 0.0f);
    svh.assign(sign_out, sign_out + out);
    std::vector<float> out_scales(out, 0.0f);
    bool apply = choose_apply_out_scales(mode, hdiag, in);
    for (size_t c = 0; c < out; c++) {
        float total = 0;
        for (size_t r0 = 0; r0 < in; r0 += 32) {
            float block = 0;
            for (size_t r = r0; r < std::min(r0 + 32, in); r++) block += weight[r * out + c] * weight[r * out + c];
            total += block;
        }
        out_scales[c] = block_rms(total, in);
    }
    double mean_sum = 0;
    for (size_t c = 0; c < out; c++) mean_sum += out_scales[c];
    double out_mean = mean_sum / (double)out;
    if (out_mean <= 1e-30) {
        std::fill(out_scales.begin(), out_scales.end(), 0.0f);
        if (mode != 0) apply = true;
    } else {
        float m = (float)out_mean;
        for (size_t c = 0; c < out; c++) out_scales[c] /= m;
    }
    if (apply)
        for (size_t c = 0; c < out; c++) svh[c] = svh[c] * (std::fabs(out_scales[c]) < 1e-30f ? 0.1f : out_scales[c]) + 1e-10f;
    for (size_t r = 0; r < in; r++)
        for (size_t c = 0; c < out; c++) weight[r * out + c] /= svh[c];
    for (size_t c = 0; c < out; c++)
        if (std::fabs(out_scales[c]) < 1e-30f) svh[c] = 0;
    hadamard_cols(weight.data(), in, out);
    for (size_t r = 0; r < in; r++) {
        float total = 0;
        for (size_t c0 = 0; c0 < out; c0 += 32) {
            float block = 0;
            for (size_t c = c0; c < std::min(c0 + 32, out); c++) block += weight[r * out + c] * weight[r * out + c];
            total += block;
        }
        float in_scale = block_rms(total, out);
        if (std::fabs(in_scale) < 1e-30f) in_scale = 0.1f;
        suh[r] = sign_in[r] * in_scale / -CODEBOOK_SCALE + 1e-10f;
    }
    for (size_t r = 0; r < in; r++)
        for (size_t c = 0; c < out; c++) weight[r * out + c] /= suh[r];
    hadamard_rows(weight.data(), in, out);
}

// src/encoder/quantize.zig:199-214
void rotated_hessian(const float* h, const float* suh, size_t n, std::vector<float>& dst) {
    std::vector<double> m(n * n);
    for (size_t i = 0; i < n; i++)
        for (size_t j = 0; j < n; j++) m[i * n + j] = (double)h[i * n + j] * (double)suh[i] * (double)suh[j];
    hadamard_rows(m.data(), n, n);
    hadamard_cols(m.data(), n, n);
    dst.resize(n * n);
    for (size_t i = 0; i < n * n; i++) dst[i] = (float)m[i];
}

// src/encoder/quantize.zig:219-230: four f64 lanes, then an ordered reduction and the tail.
inline double dot_rows(const double* a, const double* b, size_t len) {
    double acc[4] = {0, 0, 0, 0};
    size_t m = 0;
    for (; m + 4 <= len; m += 4) {
        acc[0] += a[m] * b[m];
        acc[1] += a[m + 1] * b[m + 1];
        acc[2] += a[m + 2] * b[m + 2];
        acc[3] += a[m + 3] * b[m + 3];
    }
    double sum = -0.0;
    sum += acc[0];
    sum += acc[1];
    sum += acc[2];
    sum += acc[3];
    for (; m < len; m++) sum += a[m] * b[m];
    return sum;
}

// src/encoder/quantize.zig:234-257 (the trailing update written element at a time, which the
// reference's tiled form equals bit for bit, src/encoder/quantize.zig:904-939).
size_t cholesky_lower(double* a, size_t n) {
    for (size_t k = 0; k < n; k += 64) {
        const size_t kb = std::min<size_t>(64, n - k);
        for (size_t j = 0; j < kb; j++) {
            const size_t jj = k + j;
            const double d = a[jj * n + jj] - dot_rows(a + jj * n + k, a + jj * n + k, j);
            if (!(d > 0)) return jj + 1;
            const double root = std::sqrt(d);
            a[jj * n + jj] = root;
            for (size_t i = j + 1; i < kb; i++) {
                const size_t ii = k + i;
                a[ii * n + jj] = (a[ii * n + jj] - dot_rows(a + ii * n + k, a + jj * n + k, j)) / root;
            }
        }
        for (size_t i = k + kb; i < n; i++)
            for (size_t j = 0; j < kb; j++) {
                const size_t jj = k + j;
                a[i * n + jj] = (a[i * n + jj] - dot_rows(a + i * n + k, a + jj * n + k, j)) / a[jj * n + jj];
            }
#pragma omp parallel for schedule(dynamic, 16)
        for (long long i = (long long)(k + kb); i < (long long)n; i++)
            for (size_t j = k + kb; j <= (size_t)i; j++)
                a[(size_t)i * n + j] -= dot_rows(a + (size_t)i * n + k, a + j * n + k, kb);
    }
    return 0;
}

// src/encoder/quantize.zig:302-317
bool invert_lower_block(double* blk) {
    double inv[16 * 16] = {0};
    for (int c = 0; c < 16; c++) {
        const double d = blk[c * 16 + c];
        if (d == 0 || !std::isfinite(d)) return false;
        inv[c * 16 + c] = 1.0 / d;
        for (int r = c + 1; r < 16; r++) {
            double sum = 0;
            for (int m = c; m < r; m++) sum += blk[r * 16 + m] * inv[m * 16 + c];
            inv[r * 16 + c] = -sum / blk[r * 16 + r];
        }
    }
    std::memcpy(blk, inv, sizeof(inv));
    return true;
}

// src/encoder/quantize.zig:321-337
double damp_diagonal(float* h, size_t n) {
    double diag_sum = 0;
    for (size_t i = 0; i < n; i++) {
        if (h[i * n + i] == 0) h[i * n + i] = 1;
        diag_sum += h[i * n + i];
    }
    const double diag_mean = diag_sum / (double)n;
    if (diag_mean > 0) {
        const float damp = (float)((double)SIGMA_REG * diag_mean);
        for (size_t i = 0; i < n; i++) h[i * n + i] += damp;
    }
    double damped_sum = 0;
    for (size_t i = 0; i < n; i++) damped_sum += h[i * n + i];
    return damped_sum / (double)n;
}

// src/encoder/quantize.zig:346-397
int ldl_factor(const float* h_inner, size_t n, std::vector<float>& l) {
    if (n == 0) return -10;
    if (n % 16 != 0) return -11;
    std::vector<float> h(h_inner, h_inner + n * n);
    const double damped_mean = damp_diagonal(h.data(), n);
    std::vector<double> chol64(n * n);
    int retries = 0;
    while (true) {
        for (size_t i = 0; i < n * n; i++) chol64[i] = h[i];
        if (cholesky_lower(chol64.data(), n) == 0) break;
        retries++;
        if (retries > 10 || damped_mean <= 0) return -12;  // HessianNotPositiveDefinite
        const float bump = (float)(2.0 * (double)SIGMA_REG * damped_mean);
        for (size_t i = 0; i < n; i++) h[i * n + i] += bump;
    }
    std::vector<float> chol(n * n);
    for (size_t i = 0; i < n; i++)
        for (size_t j = 0; j < n; j++) chol[i * n + j] = j <= i ? (float)chol64[i * n + j] : 0.0f;
    l = chol;
    double blk[256];
    float inv[256];
    for (size_t c0 = 0; c0 < n; c0 += 16) {
        for (int i = 0; i < 16; i++)
            for (int j = 0; j < 16; j++) blk[i * 16 + j] = j <= i ? (double)chol[(c0 + i) * n + c0 + j] : 0.0;
        if (!invert_lower_block(blk)) return -12;
        for (int i = 0; i < 16; i++)
            for (int j = 0; j < 16; j++) inv[i * 16 + j] = j <= i ? (float)blk[i * 16 + j] : 0.0f;
#pragma omp parallel for schedule(static)
        for (long long r = (long long)(c0 + 16); r < (long long)n; r++) {
            float row[16];
            for (int xx = 0; xx < 16; xx++) {
                float acc = 0;
                for (int m = 0; m < 16; m++) acc += chol[(size_t)r * n + c0 + m] * inv[m * 16 + xx];
                row[xx] = acc;
            }
            std::memcpy(&l[(size_t)r * n + c0], row, sizeof(row));
        }
        for (int i = 0; i < 16; i++) std::memset(&l[(c0 + i) * n + c0], 0, 16 * sizeof(float));
    }
    return 0;
}

double g_scale_steps_count(double low, double high, double resphi) {
    double width = high - low;
    int steps = 0;
    while (width > 0.03 && steps < 10 - 2) {
        width *= 1.0 - resphi;
        steps++;
    }
    return steps;
}

struct EncoderPool {
    std::vector<Encoder> encs;
    int init(int threads, uint32_t n, int codebook, int window_bits) {
        encs.resize((size_t)threads);
        for (auto& e : encs) {
            int rc = e.init(n, codebook, window_bits);
            if (rc) return rc;
        }
        return 0;
    }
    Encoder& mine() {
#ifdef _OPENMP
        return encs[(size_t)omp_get_thread_num()];
#else
        return encs[0];
#endif
    }
};

int max_threads() {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// src/encoder/quantize.zig:419-496
float global_scale(EncoderPool& pool, int codebook, const float* inner, size_t rows, size_t cols) {
    const size_t tk = rows / 16, tn = cols / 16;
    const size_t pair_count = std::max(tk, tn) * 3;
    const size_t stride = std::max<size_t>(1, pair_count / 128);
    std::vector<float> tiles;
    size_t count = 0;
    for (size_t p = 0; p < pair_count && count < 128; p += stride) {
        const size_t i = p / 3, wv = p % 3;
        const size_t r0 = (i % tk) * 16, c0 = ((i + wv) % tn) * 16;
        for (int r = 0; r < 16; r++)
            for (int c = 0; c < 16; c++) tiles.push_back(inner[(r0 + r) * cols + c0 + c]);
        count++;
    }
    std::vector<float> recon_all(count * TILE_LEN);
    auto score = [&](float g) -> double {
#pragma omp parallel for schedule(dynamic)
        for (long long t = 0; t < (long long)count; t++) {
            float scaled[TILE_LEN];
            uint16_t scratch[128];
            for (int i = 0; i < TILE_LEN; i++) scaled[i] = tiles[(size_t)t * TILE_LEN + i] * g;
            pool.mine().encode_tile(scaled, scratch, &recon_all[(size_t)t * TILE_LEN]);
        }
        double sse = 0;
        for (size_t t = 0; t < count; t++)
            for (int i = 0; i < TILE_LEN; i++) {
                const float d = recon_all[t * TILE_LEN + i] / g - tiles[t * TILE_LEN + i];
                sse += (double)(d * d);
            }
        return sse / (double)(count * TILE_LEN);
    };
    const double resphi64 = 2.0 - (1.0 + std::sqrt(5.0)) / 2.0;
    const float resphi = (float)resphi64;
    const float lo = codebook == 0 ? 0.4f : 0.5f;
    const float hi = codebook == 0 ? 1.2f : 1.5f;
    float a = lo, b = hi;
    float x1 = a + resphi * (b - a);
    float x2 = b - resphi * (b - a);
    double f1 = score(x1);
    double f2 = score(x2);
    const int steps = (int)g_scale_steps_count((double)lo, (double)hi, resphi64);
    for (int s = 0; s < steps; s++) {
        const bool left = f1 < f2;
        const float a_n = left ? a : x1;
        const float b_n = left ? x2 : b;
        const float probe = left ? a_n + resphi * (b_n - a_n) : b_n - resphi * (b_n - a_n);
        const double fp = score(probe);
        a = a_n;
        b = b_n;
        if (left) { x2 = x1; f2 = f1; x1 = probe; f1 = fp; }
        else { x1 = x2; f1 = f2; x2 = probe; f2 = fp; }
    }
    return (a + b) / 2.0f;
}

// src/encoder/quantize.zig:501-552
void ldlq(EncoderPool& pool, const float* inner, const float* l, size_t rows, size_t cols, uint32_t n, uint16_t* packed_out) {
    const size_t out_tiles = cols / 16;
    std::vector<float> rec(rows * cols, 0.0f), prod(rows * cols, 0.0f), comp(16 * cols), err(cols);
    size_t j = rows;
    while (j > 0) {
        const size_t i = j > 128 ? j - 128 : 0;
        const size_t chunk = j - i;
        size_t bj = chunk;
        while (bj > 0) {
            const size_t bi = bj > 16 ? bj - 16 : 0;
            const size_t height = bj - bi;
            std::memcpy(comp.data(), prod.data() + (i + bi) * cols, height * cols * sizeof(float));
            for (size_t m = bj; m < chunk; m++) {
                for (size_t c = 0; c < cols; c++) err[c] = inner[(i + m) * cols + c] - rec[(i + m) * cols + c];
                for (size_t r = 0; r < height; r++) {
                    const float lv = l[(i + m) * rows + i + bi + r];
                    float* cr = comp.data() + r * cols;
                    for (size_t c = 0; c < cols; c++) cr[c] += lv * err[c];
                }
            }
            for (size_t r = 0; r < height; r++)
                for (size_t c = 0; c < cols; c++) comp[r * cols + c] = inner[(i + bi + r) * cols + c] + comp[r * cols + c];
            const size_t tk = (i + bi) / 16;
#pragma omp parallel for schedule(dynamic)
            for (long long tn = 0; tn < (long long)out_tiles; tn++) {
                float tile[TILE_LEN], tile_rec[TILE_LEN];
                for (int r = 0; r < 16; r++)
                    for (int c = 0; c < 16; c++) tile[r * 16 + c] = comp[(size_t)r * cols + (size_t)tn * 16 + c];
                pool.mine().encode_tile(tile, packed_out + (tk * out_tiles + (size_t)tn) * n, tile_rec);
                for (int r = 0; r < 16; r++)
                    for (int c = 0; c < 16; c++) rec[(i + bi + r) * cols + (size_t)tn * 16 + c] = tile_rec[r * 16 + c];
            }
            bj -= 16;
        }
        if (i > 0) {
#pragma omp parallel for schedule(static)
            for (long long r = 0; r < (long long)i; r++) {
                float* pr = prod.data() + (size_t)r * cols;
                for (size_t m = 0; m < chunk; m++) {
                    const float lv = l[(i + m) * rows + (size_t)r];
                    const float* wrow = inner + (i + m) * cols;
                    const float* rrow = rec.data() + (i + m) * cols;
                    for (size_t c = 0; c < cols; c++) pr[c] += lv * (wrow[c] - rrow[c]);
                }
            }
        }
        j = i;
    }
}

uint64_t splitmix(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

}  // namespace

extern "C" {

// One tile search (src/encoder/encode.zig:173).  Returns the path's squared error, or a
// negative refusal code from the encoder's init.
double orc_encode_tile(const float* tile, uint32_t n, int codebook, int window_bits, uint16_t* packed_out, float* recon) {
    static thread_local Encoder enc;
    static thread_local uint32_t kn = 0;
    static thread_local int kcb = -1, kw = -1;
    if (kn != n || kcb != codebook || kw != window_bits) {
        int rc = enc.init(n, codebook, window_bits);
        if (rc) { kn = 0; return (double)rc; }
        kn = n; kcb = codebook; kw = window_bits;
    }
    return enc.encode_tile(tile, packed_out, recon);
}

// Many independent tiles (row-major 16x16 each), searched in parallel.
int orc_encode_tiles(const float* tiles, size_t count, uint32_t n, int codebook, int window_bits, uint16_t* packed_out,
                     double* costs) {
    EncoderPool pool;
    int rc = pool.init(max_threads(), n, codebook, window_bits);
    if (rc) return rc;
#pragma omp parallel for schedule(dynamic)
    for (long long t = 0; t < (long long)count; t++) {
        double c = pool.mine().encode_tile(tiles + (size_t)t * TILE_LEN, packed_out + (size_t)t * n, nullptr);
        if (costs) costs[t] = c;
    }
    return 0;
}

// src/encoder/quantize.zig:573-584
void orc_signs(uint64_t seed, const char* name, size_t len, float* out) {
    uint64_t state = seed;
    for (const char* p = name; *p; p++) state = splitmix(state ^ (uint64_t)(uint8_t)*p);
    state = splitmix(state);
    for (size_t i = 0; i < len; i++) {
        state = splitmix(state);
        out[i] = (state & 1) == 0 ? 1.0f : -1.0f;
    }
}

int orc_regularize(const float* w, size_t in, size_t out, const float* sign_in, const float* sign_out, int mode,
                   const float* hdiag, float* inner, float* suh, float* svh) {
    if (in == 0 || out == 0) return -10;
    if (in % 128 || out % 128) return -11;
    std::vector<float> wi, su, sv;
    regularize(w, in, out, sign_in, sign_out, mode, hdiag, wi, su, sv);
    std::memcpy(inner, wi.data(), wi.size() * sizeof(float));
    std::memcpy(suh, su.data(), su.size() * sizeof(float));
    std::memcpy(svh, sv.data(), sv.size() * sizeof(float));
    return 0;
}

int orc_ldl_factor(const float* h, size_t n, float* l_out) {
    std::vector<float> l;
    int rc = ldl_factor(h, n, l);
    if (rc) return rc;
    std::memcpy(l_out, l.data(), l.size() * sizeof(float));
    return 0;
}

// src/encoder/quantize.zig:604-666.  mode 0 auto, 1 always, 2 never.  Writes packed
// [in/16, out/16, n] u16, suh [in] and svh [out] f16 bits; returns 0 or a negative refusal.
int orc_quantize_tensor(const float* w, const float* h, size_t in, size_t out, const float* sign_in, const float* sign_out,
                        uint32_t n, int codebook, int window_bits, int mode, uint16_t* packed_out, uint16_t* suh_out,
                        uint16_t* svh_out, float* g_out) {
    if (in == 0 || out == 0) return -10;
    if (in % 128 || out % 128) return -11;
    EncoderPool pool;
    int rc = pool.init(max_threads(), n, codebook, window_bits);
    if (rc) return rc;
    std::vector<float> hdiag(in);
    for (size_t i = 0; i < in; i++) hdiag[i] = h[i * in + i];
    std::vector<float> inner, suh, svh;
    regularize(w, in, out, sign_in, sign_out, mode, hdiag.data(), inner, suh, svh);
    std::vector<float> rotated, l;
    rotated_hessian(h, suh.data(), in, rotated);
    rc = ldl_factor(rotated.data(), in, l);
    if (rc) return rc;
    const float g = global_scale(pool, codebook, inner.data(), in, out);
    for (auto& v : inner) v *= g;
    ldlq(pool, inner.data(), l.data(), in, out, n, packed_out);
    for (size_t i = 0; i < in; i++) suh_out[i] = orc_f32_to_f16(suh[i] / g);
    for (size_t i = 0; i < out; i++) svh_out[i] = orc_f32_to_f16(svh[i]);
    if (g_out) *g_out = g;
    return 0;
}

int orc_quantize_named(const float* w, const float* h, size_t in, size_t out, uint64_t seed, const char* name, uint32_t n,
                       int codebook, int window_bits, int mode, uint16_t* packed_out, uint16_t* suh_out, uint16_t* svh_out,
                       float* g_out) {
    std::vector<float> both(in + out);
    orc_signs(seed, name, in + out, both.data());
    return orc_quantize_tensor(w, h, in, out, both.data(), both.data() + in, n, codebook, window_bits, mode, packed_out,
                               suh_out, svh_out, g_out);
}

}  // extern "C"
