// extern "C" entry points of libsushi_exl3_cuda.so (include/sushi_exl3.h): argument admission
// mirroring the reference's named refusals, decode-parameter resolution, launch geometry.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/sushi_exl3.h"
#include "sx_decode.cuh"
#include "sx_internal.h"
#include "sx_kernels.h"
#include "sx_tables.h"

namespace sx {

namespace {
thread_local char g_detail[256] = "";
}

void note_cuda_error(cudaError_t e, const char* where) {
    snprintf(g_detail, sizeof(g_detail), "%s: %s", where, cudaGetErrorName(e));
}

void note_detail(const char* what, const char* why) { snprintf(g_detail, sizeof(g_detail), "%s: %s", what, why); }

sx_status cuda_status(cudaError_t e, const char* where) {
    if (e == cudaSuccess) return SX_OK;
    note_cuda_error(e, where);
    return SX_ERR_CUDA;
}

// Decode-parameter resolution: format.Decode.requireTable / hashMask / pair1Pair
// (src/exl3/expert_exl3.zig:141-174, :49-52) and the window admission of root.zig:217-224.
sx_status resolve_decode(const sx_decode* dec, int n, int* kind, DecParams* dp) {
    if (!dec) return SX_ERR_NULL_POINTER;
    if (dec->window_bits < 8 || dec->window_bits > 16) return SX_ERR_WINDOW_UNSUPPORTED;
    if (n < 16 || n > 128 || n % 2 != 0) return SX_ERR_TRELLIS_GEOMETRY;
    std::memset(dp, 0, sizeof(*dp));
    dp->wmask = (1u << dec->window_bits) - 1u;
    uint32_t row[4];
    switch (dec->codebook) {
        case SX_CB_MCG:
            // decodeMcg (src/exl3/expert_exl3.zig:267-273): p = cw * 0xCBAC1FED, pair =
            // 0x3B603B60 ^ (p & 0x8FFF8FFF); the kernels take the constants as values.
            *kind = K_MCG;
            dp->mult = 0xCBAC1FEDu;
            dp->mask0 = 0x8FFF8FFFu;
            dp->mask1 = 0x3B603B60u;
            return SX_OK;
        case SX_CB_MUL1: *kind = K_MUL1; return SX_OK;
        case SX_CB_SPEC1:
        case SX_CB_STD1:
            if (dec->table < 0) return SX_ERR_CODEBOOK_TABLE_UNKNOWN;
            if (dec->table > 4 || kTables[dec->table].codebook != SX_CB_SPEC1 && kTables[dec->table].codebook != SX_CB_STD1)
                return SX_ERR_CODEBOOK_TABLE_UNKNOWN;
            if (!table_row(dec->table, (uint32_t)n, row)) return SX_ERR_CODEBOOK_TABLE_RATE_MISSING;
            *kind = K_HASH;
            dp->mult = row[0];
            dp->mask0 = row[1];
            return SX_OK;
        case SX_CB_PAIR1:
            // PAIR1 reads the whole 16-bit window (codebook_tables.zig:66-69).
            if (dec->window_bits != 16) return SX_ERR_CODEBOOK_TABLE_WINDOW_MISMATCH;
            if (!table_row(SX_TABLE_PAIR1_W16_V1, (uint32_t)n, row)) return SX_ERR_CODEBOOK_TABLE_RATE_MISSING;
            *kind = K_PAIR1;
            dp->mult = row[0];
            dp->rot = row[1];
            dp->mask0 = row[2];
            dp->mask1 = row[3];
            return SX_OK;
        default: return SX_ERR_CODEBOOK_UNSUPPORTED;
    }
}

// validateClampedProjection's geometry (src/exl3/root.zig:126-135) for one projection.
sx_status check_proj(const sx_proj* p, int need_experts) {
    if (!p || !p->trellis || !p->suh || !p->svh) return SX_ERR_NULL_POINTER;
    if (p->experts <= 0 || (need_experts > 0 && p->experts != need_experts)) return SX_ERR_BAD_SHAPE;
    if (p->in_features <= 0 || p->out_features <= 0 || p->in_features % 128 || p->out_features % 128)
        return SX_ERR_BAD_SHAPE;
    if (p->n < 16 || p->n > 128 || p->n % 2) return SX_ERR_TRELLIS_GEOMETRY;
    if (p->tile_order != SX_TILE_PACK && p->tile_order != SX_TILE_PAIR_MAJOR) return SX_ERR_TILE_ORDER_UNSUPPORTED;
    // The kernels stream tile rows with 16-byte bulk copies.
    if (reinterpret_cast<uintptr_t>(p->trellis) % 16) return SX_ERR_BAD_SHAPE;
    return SX_OK;
}

bool dtype_ok(int dt) { return dt == SX_DT_F32 || dt == SX_DT_F16 || dt == SX_DT_BF16; }

int sm_count() {
    static int cached = 0;
    if (!cached) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, dev);
        if (cached <= 0) cached = 148;
    }
    return cached;
}

// sx_linear_shared_normed's workspace: the block counter, then [16 rows][out/128 blocks] f32 sums.
constexpr size_t kNormHeader = 16;

cudaError_t func_attrs(const void* kern, int smem, bool nonportable) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, std::pair<int, bool>> done;  // (kernel, device) -> settings
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    auto& d = done[{kern, dev}];
    if (smem > d.first) {
        if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
        d.first = smem;
    }
    if (nonportable && !d.second) {
        if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)) != cudaSuccess) return e;
        d.second = true;
    }
    return cudaSuccess;
}

sx_status linear_impl(sx_stream stream, const sx_proj* proj, const sx_decode* dec, const void* x, sx_dtype dtype,
                      int32_t rows, void* y, int groups, uint32_t flags, const int32_t* cols = nullptr,
                      int32_t count = 0, void* const* ys = nullptr, const void* norm_w = nullptr,
                      float norm_eps = 0.0f, void* norm_ws = nullptr) {
    if (flags & ~(uint32_t)SX_LINEAR_WEIGHTS_STATIC) return SX_ERR_BAD_SHAPE;
    sx_status st = check_proj(proj, groups);
    if (st) return st;
    if (proj->tile_order != SX_TILE_PACK) return SX_ERR_TILE_ORDER_UNSUPPORTED;
    if (!x || (!y && !count)) return SX_ERR_NULL_POINTER;
    if (!dtype_ok(dtype)) return SX_ERR_BAD_DTYPE;
    if (rows < 1) return SX_ERR_BAD_SHAPE;
    int kind;
    DecParams dp;
    st = resolve_decode(dec, proj->n, &kind, &dp);
    if (st) return st;
    const int in = proj->in_features, out = proj->out_features;
    const size_t esz = dtype == SX_DT_F32 ? 4 : 2;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // Rows go through the kernel 16 at a time (two MMA column groups).
    for (int r0 = 0; r0 < rows; r0 += 16) {
        const int r = std::min(16, rows - r0);
        GemvArgs a;
        a.trellis = proj->trellis;
        a.suh = proj->suh;
        a.svh = proj->svh;
        a.x = static_cast<const uint8_t*>(x) + (size_t)r0 * in * esz;
        a.y = static_cast<uint8_t*>(y) + (size_t)r0 * out * esz;
        a.in = in;
        a.out = out;
        a.rows = r;
        a.xdt = dtype;
        a.x_group_stride = (long long)rows * in;
        a.y_group_stride = (long long)rows * out;
        a.wmask = dp.wmask;
        a.mult = dp.mult;
        a.mask0 = dp.mask0;
        a.mask1 = dp.mask1;
        a.rot = dp.rot;
        a.out_scale = kind_scale(kind);
        a.vec = reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(proj->suh) % 8 == 0;
        a.nseg = count;
        for (int i = 0; i < count; i++) {
            a.seg_end[i] = cols[i + 1] / 128;
            a.ywidth[i] = cols[i + 1] - cols[i];
            a.ys[i] = static_cast<uint8_t*>(ys[i]) + (size_t)r0 * a.ywidth[i] * esz;
        }
        a.norm_w = norm_w;
        a.norm_eps = norm_eps;
        a.norm_count = static_cast<unsigned*>(norm_ws);
        a.norm_ssq = norm_ws ? reinterpret_cast<float*>(static_cast<uint8_t*>(norm_ws) + kNormHeader) : nullptr;
        // A later 16-row chunk follows this call's own launch, which writes only y.
        a.pdl = (flags & SX_LINEAR_WEIGHTS_STATIC) || r0 > 0;
        cudaError_t e = launch_gemv(a, kind, proj->n, groups, s);
        if (e != cudaSuccess) return cuda_status(e, "gemv launch");
    }
    return SX_OK;
}

}  // namespace sx

using namespace sx;

extern "C" {

const char* sx_status_name(sx_status s) {
    switch (s) {
        case SX_OK: return "SX_OK";
        case SX_ERR_BAD_SHAPE: return "SX_ERR_BAD_SHAPE";
        case SX_ERR_BAD_DTYPE: return "SX_ERR_BAD_DTYPE";
        case SX_ERR_INVALID_CLAMP: return "SX_ERR_INVALID_CLAMP";
        case SX_ERR_TOPK_EXCEEDS_REDUCE_BANK: return "SX_ERR_TOPK_EXCEEDS_REDUCE_BANK";
        case SX_ERR_CODEBOOK_TABLE_UNKNOWN: return "SX_ERR_CODEBOOK_TABLE_UNKNOWN";
        case SX_ERR_TRELLIS_GEOMETRY: return "SX_ERR_TRELLIS_GEOMETRY";
        case SX_ERR_CODEBOOK_TABLE_RATE_MISSING: return "SX_ERR_CODEBOOK_TABLE_RATE_MISSING";
        case SX_ERR_WINDOW_UNSUPPORTED: return "SX_ERR_WINDOW_UNSUPPORTED";
        case SX_ERR_CODEBOOK_UNSUPPORTED: return "SX_ERR_CODEBOOK_UNSUPPORTED";
        case SX_ERR_CODEBOOK_TABLE_WINDOW_MISMATCH: return "SX_ERR_CODEBOOK_TABLE_WINDOW_MISMATCH";
        case SX_ERR_TOPK_EXCEEDS_EXPERTS: return "SX_ERR_TOPK_EXCEEDS_EXPERTS";
        case SX_ERR_ROUTER_DECLINED: return "SX_ERR_ROUTER_DECLINED";
        case SX_ERR_NULL_POINTER: return "SX_ERR_NULL_POINTER";
        case SX_ERR_WORKSPACE_TOO_SMALL: return "SX_ERR_WORKSPACE_TOO_SMALL";
        case SX_ERR_CUDA: return "SX_ERR_CUDA";
        case SX_ERR_DEVICE_TIMEOUT: return "SX_ERR_DEVICE_TIMEOUT";
        case SX_ERR_NCCL: return "SX_ERR_NCCL";
        case SX_ERR_TILE_ORDER_UNSUPPORTED: return "SX_ERR_TILE_ORDER_UNSUPPORTED";
        case SX_ERR_GROUP_GEOMETRY: return "SX_ERR_GROUP_GEOMETRY";
        case SX_ERR_STATIC_SCRATCH_TOO_SMALL: return "SX_ERR_STATIC_SCRATCH_TOO_SMALL";
        case SX_ERR_PEER_BUFFER_TOO_SMALL: return "SX_ERR_PEER_BUFFER_TOO_SMALL";
        case SX_ERR_PEER_ACCESS: return "SX_ERR_PEER_ACCESS";
        default: return "SX_ERR_UNKNOWN";
    }
}

const char* sx_last_error_detail(void) { return g_detail; }

const char* sx_version(void) { return "sushi-exl3-b200 0.1.0 (reference sushi 1.7.2)"; }

sx_status sx_table_row(int32_t table, int32_t n, uint32_t* out4) {
    if (!out4) return SX_ERR_NULL_POINTER;
    return table_row(table, (uint32_t)n, out4) ? SX_OK : SX_ERR_CODEBOOK_TABLE_RATE_MISSING;
}

sx_status sx_table_info(int32_t table, const char** name, int32_t* codebook, int32_t* window_bits, const char** digest,
                        int32_t* fields, int32_t* n_lo, int32_t* rows) {
    if (table < 0 || table > 4) return SX_ERR_CODEBOOK_TABLE_UNKNOWN;
    const TableDesc& t = kTables[table];
    if (name) *name = t.name;
    if (codebook) *codebook = t.codebook;
    if (window_bits) *window_bits = t.window_bits;
    if (digest) *digest = t.digest;
    if (fields) *fields = t.fields;
    if (n_lo) *n_lo = (int32_t)t.n_lo;
    if (rows) *rows = t.rows;
    return SX_OK;
}

sx_status sx_dequant_inner(sx_stream stream, const sx_proj* proj, int32_t expert, const sx_decode* dec, uint16_t* out) {
    sx_status st = check_proj(proj, 0);
    if (st) return st;
    if (proj->tile_order != SX_TILE_PACK) return SX_ERR_TILE_ORDER_UNSUPPORTED;
    if (!out) return SX_ERR_NULL_POINTER;
    if (expert < 0 || expert >= proj->experts) return SX_ERR_BAD_SHAPE;
    int kind;
    DecParams dp;
    st = resolve_decode(dec, proj->n, &kind, &dp);
    if (st) return st;
    DequantArgs a;
    const size_t per = (size_t)(proj->in_features / 16) * (proj->out_features / 16) * proj->n;
    a.trellis = proj->trellis + (size_t)expert * per;
    a.dst = out;
    a.in_f = proj->in_features;
    a.out_f = proj->out_features;
    a.n = proj->n;
    a.wmask = dp.wmask;
    a.mult = dp.mult;
    a.mask0 = dp.mask0;
    a.mask1 = dp.mask1;
    a.rot = dp.rot;
    return cuda_status(launch_dequant(a, kind, reinterpret_cast<cudaStream_t>(stream)), "dequant launch");
}

sx_status sx_decode_codewords(sx_stream stream, int32_t n, const sx_decode* dec, uint32_t* out32) {
    if (!out32) return SX_ERR_NULL_POINTER;
    int kind;
    DecParams dp;
    sx_status st = resolve_decode(dec, n, &kind, &dp);
    if (st) return st;
    return cuda_status(launch_decode_codewords(kind, n, dp.wmask, dp.mult, dp.mask0, dp.mask1, dp.rot, out32,
                                               reinterpret_cast<cudaStream_t>(stream)),
                       "codewords launch");
}

sx_status sx_linear(sx_stream stream, const sx_proj* proj, const sx_decode* dec, const void* x, sx_dtype dtype,
                    int32_t rows, void* y) {
    if (proj && proj->experts != 1) return SX_ERR_BAD_SHAPE;
    return linear_impl(stream, proj, dec, x, dtype, rows, y, 1, 0);
}

sx_status sx_linear_shared(sx_stream stream, const sx_proj* proj, const int32_t* cols, int32_t count,
                           const sx_decode* dec, const void* x, sx_dtype dtype, int32_t rows, void* const* ys) {
    if (!proj || !cols || !ys) return SX_ERR_NULL_POINTER;
    if (proj->experts != 1 || count < 1 || count > 4) return SX_ERR_BAD_SHAPE;
    if (cols[0] != 0 || cols[count] != proj->out_features) return SX_ERR_BAD_SHAPE;
    for (int i = 0; i < count; i++) {
        if (cols[i + 1] <= cols[i] || cols[i + 1] % 128) return SX_ERR_BAD_SHAPE;
        if (!ys[i]) return SX_ERR_NULL_POINTER;
    }
    return linear_impl(stream, proj, dec, x, dtype, rows, nullptr, 1, 0, cols, count, ys);
}

size_t sx_linear_shared_normed_workspace_bytes(const sx_proj* proj) {
    if (!proj || proj->out_features < 128) return 0;
    return kNormHeader + (size_t)16 * (proj->out_features / 128) * sizeof(float);
}

sx_status sx_linear_shared_normed(sx_stream stream, const sx_proj* proj, const int32_t* cols, int32_t count,
                                  const sx_decode* dec, const void* x, sx_dtype dtype, int32_t rows, void* const* ys,
                                  const void* norm_w, float eps, void* workspace, size_t workspace_bytes) {
    if (!proj || !cols || !ys || !norm_w) return SX_ERR_NULL_POINTER;
    if (proj->experts != 1 || count < 1 || count > 4) return SX_ERR_BAD_SHAPE;
    if (cols[0] != 0 || cols[count] != proj->out_features) return SX_ERR_BAD_SHAPE;
    for (int i = 0; i < count; i++) {
        if (cols[i + 1] <= cols[i] || cols[i + 1] % 128) return SX_ERR_BAD_SHAPE;
        if (!ys[i]) return SX_ERR_NULL_POINTER;
    }
    // One launch (<= 16 rows) and an output the reference's one-threadgroup finish covers
    // (project_rows.zig:914-919: out <= 4096).
    if (rows > 16 || proj->out_features > 4096) return SX_ERR_BAD_SHAPE;
    if (!(eps >= 0.0f) || !std::isfinite(eps)) return SX_ERR_BAD_SHAPE;
    if (!workspace) return SX_ERR_NULL_POINTER;
    if (workspace_bytes < sx_linear_shared_normed_workspace_bytes(proj)) return SX_ERR_WORKSPACE_TOO_SMALL;
    if (reinterpret_cast<uintptr_t>(workspace) % 16) return SX_ERR_BAD_SHAPE;
    return linear_impl(stream, proj, dec, x, dtype, rows, nullptr, 1, 0, cols, count, ys, norm_w, eps, workspace);
}

sx_status sx_linear_ex(sx_stream stream, const sx_proj* proj, const sx_decode* dec, const void* x, sx_dtype dtype,
                       int32_t rows, void* y, uint32_t flags) {
    if (proj && proj->experts != 1) return SX_ERR_BAD_SHAPE;
    return linear_impl(stream, proj, dec, x, dtype, rows, y, 1, flags);
}

sx_status sx_linear_grouped(sx_stream stream, const sx_proj* proj, const sx_decode* dec, const void* x,
                            sx_dtype dtype, int32_t rows, void* y) {
    if (!proj) return SX_ERR_NULL_POINTER;
    return linear_impl(stream, proj, dec, x, dtype, rows, y, proj->experts, 0);
}

int32_t sx_device_error(sx_stream stream) {
    cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
    int v = 0;
    cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
    int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    return v;
}

}  // extern "C"
