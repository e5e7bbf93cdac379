// sx_moe_static_scratch: sx_moe with its scratch in a buffer compiled into the library, for
// callers that cannot allocate device memory on the layer's path (an allocator that owns and bills
// every device byte, a loop that cannot take cudaMalloc's implicit device-wide synchronisation) and
// so cannot pass a workspace.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/sushi_exl3.h"

namespace {

constexpr size_t kStaticScratchBytes = 8u << 20;  // 8 MiB: a decode layer of up to ~900 slots at 2048/512

// The scratch every call shares.  In host code this name is a host-side handle, not a device
// address: only cudaGetSymbolAddress yields the pointer a kernel may be given.
static __device__ __align__(256) uint8_t g_moe_scratch[kStaticScratchBytes];

// The buffer's device address, looked up once per (device, context) with that device current: a
// module loaded into a caller's own driver-API context sits at its own address there.
constexpr int kMaxEntries = 64;
struct Entry {
    int device;
    CUcontext ctx;
    void* addr;
};
std::mutex g_lock;
Entry g_entries[kMaxEntries];
int g_count = 0;

// cuCtxGetCurrent through the runtime's driver entry point (the library does not link libcuda).
using CtxGetCurrent = CUresult (*)(CUcontext*);

sx_status current_context(CUcontext* ctx) {
    static CtxGetCurrent fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !p)
            return SX_ERR_CUDA;
        fn = reinterpret_cast<CtxGetCurrent>(p);
    }
    *ctx = nullptr;
    return fn(ctx) == CUDA_SUCCESS ? SX_OK : SX_ERR_CUDA;
}

sx_status scratch_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return SX_ERR_CUDA;
    CUcontext ctx = nullptr;
    if (current_context(&ctx) != SX_OK) return SX_ERR_CUDA;
    if (!ctx) {
        // no context current yet: bring up the device's primary one, which the launches will use
        if (cudaFree(nullptr) != cudaSuccess || current_context(&ctx) != SX_OK || !ctx) return SX_ERR_CUDA;
    }
    std::lock_guard<std::mutex> guard(g_lock);
    for (int i = 0; i < g_count; i++) {
        if (g_entries[i].device == dev && g_entries[i].ctx == ctx) {
            *out = g_entries[i].addr;
            return SX_OK;
        }
    }
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_moe_scratch) != cudaSuccess || !p) return SX_ERR_CUDA;
    if (g_count < kMaxEntries) g_entries[g_count++] = Entry{dev, ctx, p};
    *out = p;
    return SX_OK;
}

}  // namespace

extern "C" size_t sx_moe_static_scratch_bytes(void) { return kStaticScratchBytes; }

extern "C" sx_status sx_moe_static_scratch(sx_stream stream, const sx_bank* bank, const sx_decode* dec, const void* x,
                                           sx_dtype dtype, int32_t rows, const uint32_t* inds, const float* scores,
                                           int32_t topk, const void* shared, const void* shared_gate,
                                           int32_t clamp_limit, void* y) {
    // sx_moe's own admission first, with no workspace: a malformed call gets sx_moe's refusal (the
    // workspace check comes after every shape, dtype, decode and clamp check, and nothing launches)
    const sx_status pre = sx_moe(stream, bank, dec, x, dtype, rows, inds, scores, topk, shared, shared_gate,
                                 clamp_limit, y, nullptr, 0);
    if (pre != SX_ERR_WORKSPACE_TOO_SMALL) return pre;
    if (sx_moe_workspace_bytes(bank, rows, topk) > kStaticScratchBytes) return SX_ERR_STATIC_SCRATCH_TOO_SMALL;
    void* scratch = nullptr;
    const sx_status st = scratch_address(&scratch);
    if (st != SX_OK) return st;
    return sx_moe(stream, bank, dec, x, dtype, rows, inds, scores, topk, shared, shared_gate, clamp_limit, y, scratch,
                  kStaticScratchBytes);
}
