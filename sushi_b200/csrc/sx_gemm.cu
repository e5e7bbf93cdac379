// Tensor-core projection: host side.  The prepared-row kernels, the TMA map of the prepared
// rows, the split choice, and sx_linear_gemm (dense rows through sx_gemm_impl.cuh).
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <utility>
#include <vector>

#include "sx_gemm_impl.cuh"
#include "sx_internal.h"

namespace sx {

template <int KIND>
cudaError_t gemm_dispatch(const CUtensorMap& pmap, const GemmArgs& a, int n, int rt, int items, int S,
                          cudaStream_t stream, bool pair, int nt);

// P[r][kb*128 + i] = f16(H128(f16(x[r]) * suh)) for one (row, 128-input block) per warp: the
// reference's prepareInput (src/exl3/expert_exl3.zig:490-501).
__global__ void __launch_bounds__(256) prep_rows_kernel(const void* x, int xdt, const uint16_t* suh, int rows, int in,
                                                        uint16_t* P) {
    const int warp = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int KB = in / 128;
    if (warp >= rows * KB) return;
    const int r = warp / KB, kb = warp % KB;
    const int base = kb * 128 + lane * 4;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = round_f16(load_act(x, (size_t)r * in + base + i, xdt)) * h2f(suh[base + i]);
    warp_hadamard128(v);
    uint2 h;
    h.x = (uint32_t)f2h(v[0]) | ((uint32_t)f2h(v[1]) << 16);
    h.y = (uint32_t)f2h(v[2]) | ((uint32_t)f2h(v[3]) << 16);
    *reinterpret_cast<uint2*>(P + (size_t)r * in + base) = h;
}

// The TMA map of a [rows, in] f16 matrix read in (box_rows x 64) tiles, 128-byte swizzled.
cudaError_t prep_map(CUtensorMap* m, const uint16_t* P, int rows, int in, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)in, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)in * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kGemmKC, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    // The driver entry point is looked up through the runtime, so the library loads on hosts
    // without a driver (its CPU-side tests) and needs no link against libcuda.
    using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static Encode encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return e != cudaSuccess ? e : cudaErrorNotSupported;
        encode = reinterpret_cast<Encode>(fn);
    }
    const CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(P), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t gemm_launch(int kind, const CUtensorMap& pmap, const GemmArgs& a, int n, int rt, int items, int S,
                        cudaStream_t stream, bool pair, int nt) {
    switch (kind) {
        case K_MCG: return gemm_dispatch<K_MCG>(pmap, a, n, rt, items, S, stream, pair, nt);
        case K_MUL1: return gemm_dispatch<K_MUL1>(pmap, a, n, rt, items, S, stream, pair, nt);
        case K_HASH: return gemm_dispatch<K_HASH>(pmap, a, n, rt, items, S, stream, pair, nt);
        case K_PAIR1: return gemm_dispatch<K_PAIR1>(pmap, a, n, rt, items, S, stream, pair, nt);
        default: return cudaErrorInvalidValue;
    }
}

namespace {
struct CoKey {
    const void* kern;
    int clusters, S;
    bool operator==(const CoKey& o) const { return kern == o.kern && clusters == o.clusters && S == o.S; }
};
std::mutex g_co_lock;
std::vector<std::pair<CoKey, int>> g_co;
}  // namespace

int gemm_coresident_split(const void* kern, int smem, int threads, dim3 grid_xy, int S) {
    const int clusters = (int)(grid_xy.x * grid_xy.y);
    const CoKey key{kern, clusters, S};
    {
        std::lock_guard<std::mutex> guard(g_co_lock);
        for (const auto& e : g_co)
            if (e.first == key) return e.second;
    }
    int best = 1;
    for (int cand = S; cand > 1; cand--) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid_xy.x, grid_xy.y, cand);
        cfg.blockDim = dim3(threads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = cand;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int active = 0;
        if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) == cudaSuccess && active >= clusters) {
            best = cand;
            break;
        }
        cudaGetLastError();
    }
    std::lock_guard<std::mutex> guard(g_co_lock);
    g_co.emplace_back(key, best);
    return best;
}

// Split-K for `ctas` (row tile, output block) CTAs over `chunks` 64-input chunks: about one wave
// of one CTA per SM, at most 16 ranks, at least 4 chunks per rank (the launch then lowers it to
// the largest split whose clusters are all co-resident, gemm_coresident_split).
int gemm_split(long long ctas, int chunks) {
    const long long want = sm_count();
    int S = (int)std::max(1LL, want / std::max(1LL, ctas));
    S = std::min(S, 16);
    S = std::min(S, std::max(1, chunks / 4));
    return std::max(1, S);
}

bool gemm_rt_rate(int n) { return n == 16 || n == 24 || n == 32 || n == 40 || n == 48 || n == 64; }

// Row tiles per CTA for `rows` rows: four (each decoded weight chunk feeds four 128-row
// accumulators, so the decode work per flop drops fourfold) from 384 rows, for rates that have the
// kernel; the split over K then fills the SMs.
int gemm_rt(long long rows, int n) { return gemm_rt_rate(n) && rows >= 3LL * kGemmRows ? 4 : 1; }

}  // namespace sx

using namespace sx;

extern "C" size_t sx_linear_gemm_workspace_bytes(const sx_proj* proj, int32_t rows) {
    if (!proj || rows < 1 || proj->in_features <= 0) return 0;
    return ((size_t)rows * proj->in_features * 2 + 255) / 256 * 256;
}

extern "C" sx_status sx_linear_gemm(sx_stream stream, const sx_proj* proj, const sx_decode* dec, const void* x,
                                    sx_dtype dtype, int32_t rows, void* y, void* workspace, size_t workspace_bytes) {
    if (proj && proj->experts != 1) return SX_ERR_BAD_SHAPE;
    sx_status st = check_proj(proj, 1);
    if (st) return st;
    if (proj->tile_order != SX_TILE_PACK) return SX_ERR_TILE_ORDER_UNSUPPORTED;
    if (!x || !y) return SX_ERR_NULL_POINTER;
    if (!dtype_ok(dtype)) return SX_ERR_BAD_DTYPE;
    if (rows < 1) return SX_ERR_BAD_SHAPE;
    int kind;
    DecParams dp;
    if ((st = resolve_decode(dec, proj->n, &kind, &dp))) return st;
    const size_t need = sx_linear_gemm_workspace_bytes(proj, rows);
    if (!workspace || workspace_bytes < need) return SX_ERR_WORKSPACE_TOO_SMALL;
    if (reinterpret_cast<uintptr_t>(workspace) % 16) return SX_ERR_BAD_SHAPE;
    const int in = proj->in_features, out = proj->out_features;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint16_t* P = static_cast<uint16_t*>(workspace);
    const int warps = rows * (in / 128);
    prep_rows_kernel<<<(warps + 7) / 8, 256, 0, s>>>(x, dtype, proj->suh, rows, in, P);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "prep launch");
    // At most 16 rows: 16-row tiles (the MMA's N and the prepared-row copy cover the live rows, so
    // a stage is 20 KB and the ring twice as deep); else 128-row tiles.
    const int nt = rows <= kGemmRowsNarrow ? kGemmRowsNarrow : kGemmRows;
    CUtensorMap pmap;
    if ((e = prep_map(&pmap, P, rows, in, nt)) != cudaSuccess) return cuda_status(e, "cuTensorMapEncodeTiled");
    GemmArgs a{};
    a.trellis = proj->trellis;
    a.tr_expert = 0;
    a.svh = proj->svh;
    a.in = in;
    a.out = out;
    a.dp = dp;
    a.scale = kind_scale(kind);
    a.rows = rows;
    a.mode = GEMM_OUT_ACT;
    a.y = y;
    a.ydt = dtype;
    const int rt = gemm_rt(rows, proj->n);
    const int items = (rows + nt * rt - 1) / (nt * rt);
    const int S = gemm_split((long long)items * (out / 128), in / kGemmKC);
    e = gemm_launch(kind, pmap, a, proj->n, rt, items, S, s, false, nt);
    return cuda_status(e, "gemm launch");
}
