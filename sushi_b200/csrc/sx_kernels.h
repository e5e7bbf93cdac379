// Host-side declarations of the kernel launchers (internal to libsushi_exl3_cuda.so).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace sx {

struct GemvArgs {
    const uint16_t* trellis;   // [G][in/16][out/16][n]
    const uint16_t* suh;       // [G][in]
    const uint16_t* svh;       // [G][out]
    const void* x;             // [G][rows][in]
    void* y;                   // [G][rows][out]
    int in, out, rows;
    int xdt;                   // sx_dtype of x and y
    long long x_group_stride;  // elements between banks' inputs
    long long y_group_stride;
    uint32_t wmask, mult, mask0, mask1, rot;
    float out_scale;
    int vec;                   // x starts 16-byte aligned and suh 8-byte aligned: vector loads
    int pdl;                   // host side: launch with programmatic stream serialisation
    // Stacked linears sharing the input (nseg > 0): output blocks [seg_end[s-1], seg_end[s]) are
    // linear s, prepared with suh row s and written to ys[s] ([rows][ywidth[s]] in x's dtype).
    int nseg;
    int seg_end[4];
    void* ys[4];
    int ywidth[4];
    // RMS-normed first linear (norm_w != nullptr, one bank, rows <= 16): the finish leaves linear
    // 0's row as w * T(o * rsqrt(mean(o^2) + eps)), o its finished values in x's dtype T.  Each
    // output block of linear 0 writes its rows' sums of squares to norm_ssq[row][block]; the last
    // block to count itself in norm_count (left at 0 again) applies the norm.
    const void* norm_w;
    float norm_eps;
    float* norm_ssq;
    unsigned* norm_count;
};

cudaError_t launch_gemv(const GemvArgs& a, int kind, int n, int groups, cudaStream_t stream);

struct DequantArgs {
    const uint16_t* trellis;  // one expert's [in/16][out/16][n] (pack order)
    uint16_t* dst;            // [in_f][out_f] f16 bits
    int in_f, out_f, n;
    uint32_t wmask, mult, mask0, mask1, rot;
};

cudaError_t launch_dequant(const DequantArgs& a, int kind, cudaStream_t stream);
cudaError_t launch_decode_codewords(int kind, int n, uint32_t wmask, uint32_t mult, uint32_t mask0, uint32_t mask1,
                                    uint32_t rot, uint32_t* out32, cudaStream_t stream);

}  // namespace sx
