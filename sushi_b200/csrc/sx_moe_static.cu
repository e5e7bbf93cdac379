// sx_moe_static_scratch: sx_moe with its scratch in a buffer compiled into the library, for
// callers that cannot allocate device memory (stream capture, an allocator that owns every byte,
// loops that cannot take cudaMalloc's implicit synchronisation) and so cannot pass a workspace.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/sushi_exl3.h"

namespace {

constexpr size_t kStaticScratchBytes = 8u << 20;  // 8 MiB: a decode layer of up to ~900 slots at 2048/512

// The scratch every call shares.  In host code this name is a host-side handle, not a device
// address: only cudaGetSymbolAddress yields the pointer a kernel may be given.
static __device__ __align__(256) uint8_t g_moe_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_lock;
void* g_addr[kMaxDevices] = {};

// The buffer's device address on the current device, looked up once per device.
sx_status scratch_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SX_ERR_CUDA;
    std::lock_guard<std::mutex> guard(g_lock);
    if (!g_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_moe_scratch) != cudaSuccess || !p) return SX_ERR_CUDA;
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return SX_OK;
}

}  // namespace

extern "C" size_t sx_moe_static_scratch_bytes(void) { return kStaticScratchBytes; }

extern "C" sx_status sx_moe_static_scratch(sx_stream stream, const sx_bank* bank, const sx_decode* dec, const void* x,
                                           sx_dtype dtype, int32_t rows, const uint32_t* inds, const float* scores,
                                           int32_t topk, const void* shared, const void* shared_gate,
                                           int32_t clamp_limit, void* y) {
    if (!bank) return SX_ERR_NULL_POINTER;
    if (rows < 1 || topk < 1) return SX_ERR_BAD_SHAPE;
    const size_t need = sx_moe_workspace_bytes(bank, rows, topk);
    if (need > kStaticScratchBytes) return SX_ERR_STATIC_SCRATCH_TOO_SMALL;
    void* scratch = nullptr;
    const sx_status st = scratch_address(&scratch);
    if (st != SX_OK) return st;
    return sx_moe(stream, bank, dec, x, dtype, rows, inds, scores, topk, shared, shared_gate, clamp_limit, y, scratch,
                  kStaticScratchBytes);
}
