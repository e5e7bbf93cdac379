// Tile-order conversion between the pack order [IT][OT][n] and the pair-major order
// [OT/2][IT][2][n] (layout.tileMajor / tileMajorInverse, src/exl3/layout.zig:141-160;
// docs/pack-format.md "tile order"), per expert, on the device.
#include "sx_internal.h"

namespace sx {
namespace {

// One warp per (expert, input tile row, output tile pair): the pair's two tiles, 2*n halfwords
// contiguous in both orders, moved with 32-bit words (n is even).
__global__ void __launch_bounds__(256) tile_order_kernel(const uint16_t* src, uint16_t* dst, int IT, int OT, int n,
                                                         long long units, int to_pair_major) {
    const long long u = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (u >= units) return;
    const int lane = threadIdx.x & 31;
    const int P = OT / 2;
    const long long e = u / ((long long)IT * P);
    const int rem = (int)(u % ((long long)IT * P));
    const int tk = rem / P, pair = rem % P;
    const size_t per = (size_t)IT * OT * n;
    const size_t pack = e * per + ((size_t)tk * OT + pair * 2) * n;
    const size_t pm = e * per + ((size_t)pair * IT + tk) * 2 * n;
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src + (to_pair_major ? pack : pm));
    uint32_t* d = reinterpret_cast<uint32_t*>(dst + (to_pair_major ? pm : pack));
    for (int i = lane; i < n; i += 32) d[i] = s[i];  // 2n halfwords = n words
}

}  // namespace
}  // namespace sx

using namespace sx;

extern "C" sx_status sx_tile_order_convert(sx_stream stream, const uint16_t* src, uint16_t* dst, int32_t experts,
                                           int32_t in_features, int32_t out_features, int32_t n, int32_t from_order,
                                           int32_t to_order) {
    if (!src || !dst) return SX_ERR_NULL_POINTER;
    if (experts < 1 || in_features <= 0 || out_features <= 0 || in_features % 128 || out_features % 128)
        return SX_ERR_BAD_SHAPE;
    if (n < 16 || n > 128 || n % 2) return SX_ERR_TRELLIS_GEOMETRY;
    const bool ok_orders = (from_order == SX_TILE_PACK || from_order == SX_TILE_PAIR_MAJOR) &&
                           (to_order == SX_TILE_PACK || to_order == SX_TILE_PAIR_MAJOR);
    if (!ok_orders) return SX_ERR_TILE_ORDER_UNSUPPORTED;
    if (reinterpret_cast<uintptr_t>(src) % 4 || reinterpret_cast<uintptr_t>(dst) % 4) return SX_ERR_BAD_SHAPE;
    const int IT = in_features / 16, OT = out_features / 16;
    const size_t bytes = (size_t)experts * IT * OT * n * 2;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (from_order == to_order) {
        if (src == dst) return SX_OK;
        return cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s), "tile order copy");
    }
    // the orders permute whole tile pairs, so in place would overwrite unread pairs
    const uint8_t* a = reinterpret_cast<const uint8_t*>(src);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(dst);
    if (a < b + bytes && b < a + bytes) return SX_ERR_BAD_SHAPE;
    const long long units = (long long)experts * IT * (OT / 2);
    tile_order_kernel<<<(unsigned)((units + 7) / 8), 256, 0, s>>>(src, dst, IT, OT, n, units,
                                                                  to_order == SX_TILE_PAIR_MAJOR);
    return cuda_status(cudaGetLastError(), "tile order launch");
}
