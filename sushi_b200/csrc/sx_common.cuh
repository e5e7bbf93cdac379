// Device helpers shared by the sm_100a kernels: the error latch, bounded mbarrier waits, bulk
// (TMA) copies, the legacy-layout MMA used for the decode GEMVs, and the warp Hadamard-128.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sx {

// A kernel's dynamic shared-memory limit (at least `smem` bytes) and, with `nonportable`, its
// non-portable cluster sizes, set on the current device once: later calls that ask for no more
// return without a driver call (host; sx_capi.cu).
cudaError_t func_attrs(const void* kern, int smem, bool nonportable);

// Codes a kernel latches when a bounded wait gives up (read by sx_device_error).
enum DeviceError : int {
    DEV_OK = 0,
    DEV_TIMEOUT_FULL = 1,     // a consumer waited too long for a stage's bytes
    DEV_TIMEOUT_EMPTY = 2,    // the producer waited too long for a stage to drain
    DEV_TIMEOUT_SELFTEST = 3, // sx_selftest_wait_timeout's wait gave up, as it is meant to
    DEV_TIMEOUT_PEER = 4,     // an expert-parallel rank waited too long for a peer's flag
};

extern __device__ int g_device_error;

__device__ __forceinline__ void latch_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the barrier's phase with `parity` to complete, for at most ~2 s of wall time.  On a
// timeout it latches `code` and returns false; the caller then skips its work but still reaches
// every later block- and cluster-wide barrier, so no thread is left waiting.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code,
                                          uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && global_timer_ns() - t0 > limit_ns) {
            latch_error(code);
            return false;
        }
    }
}

// ------------------------------------------------------------------ flags between GPUs
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until *flag >= seq (wrap-safe), for at most ~2 s of wall time; on a timeout latches
// DEV_TIMEOUT_PEER and returns false (the caller goes on: its outputs are undefined, nothing hangs).
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t seq) {
    if ((int32_t)(ld_acquire_sys(flag) - seq) >= 0) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0;; i++) {
        __nanosleep(64);
        if ((int32_t)(ld_acquire_sys(flag) - seq) >= 0) return true;
        if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
            latch_error(DEV_TIMEOUT_PEER);
            return false;
        }
    }
}

// ------------------------------------------------------------------ bulk copies (TMA, 1-D)
// global -> this CTA's shared memory, completing `bytes` on `bar`.  dst and src 16-byte aligned,
// bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------------ MMA (m16n8k16, f16 -> f32)
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------ conversions
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float round_f16(float f) { return __half2float(__float2half_rn(f)); }

// dtype codes as sx_dtype: 0 f32, 1 f16, 2 bf16
__device__ __forceinline__ float load_act(const void* p, size_t i, int dt) {
    if (dt == 0) return static_cast<const float*>(p)[i];
    if (dt == 1) return __half2float(static_cast<const __half*>(p)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

// Four consecutive elements from element i (a multiple of 4) of an activation row whose rows start
// 16-byte aligned: one 8- or 16-byte load.
__device__ __forceinline__ void load_act4(const void* p, size_t i, int dt, float (&v)[4]) {
    if (dt == 0) {
        const float4 t = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
        v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
        return;
    }
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p) + i);
    const uint16_t h[4] = {(uint16_t)u.x, (uint16_t)(u.x >> 16), (uint16_t)u.y, (uint16_t)(u.y >> 16)};
#pragma unroll
    for (int k = 0; k < 4; k++)
        v[k] = dt == 1 ? __half2float(__ushort_as_half(h[k])) : __bfloat162float(__ushort_as_bfloat16(h[k]));
}

// Four consecutive f16 values from element i (a multiple of 4) as floats: one 8-byte load when
// `vec` (the array starts 8-byte aligned), else four 2-byte loads.
__device__ __forceinline__ void load_half4(const uint16_t* p, size_t i, bool vec, float (&v)[4]) {
    if (vec) {
        const uint2 u = *reinterpret_cast<const uint2*>(p + i);
        v[0] = __half2float(__ushort_as_half((uint16_t)u.x));
        v[1] = __half2float(__ushort_as_half((uint16_t)(u.x >> 16)));
        v[2] = __half2float(__ushort_as_half((uint16_t)u.y));
        v[3] = __half2float(__ushort_as_half((uint16_t)(u.y >> 16)));
        return;
    }
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = __half2float(__ushort_as_half(p[i + k]));
}

// Four consecutive activations from element i (a multiple of 4): load_act4 when `vec` (rows start
// 16-byte aligned), else element by element.
__device__ __forceinline__ void load_act4v(const void* p, size_t i, int dt, bool vec, float (&v)[4]) {
    if (vec) {
        load_act4(p, i, dt, v);
        return;
    }
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = load_act(p, i + k, dt);
}

// v rounded to an activation dtype and back.
__device__ __forceinline__ float round_act(float v, int dt) {
    if (dt == 0) return v;
    if (dt == 1) return __half2float(__float2half_rn(v));
    return __bfloat162float(__float2bfloat16_rn(v));
}

// load_act past L1: for values another CTA of the same grid wrote (after a fence).
__device__ __forceinline__ float load_act_cg(const void* p, size_t i, int dt) {
    if (dt == 0) return __ldcg(static_cast<const float*>(p) + i);
    const unsigned short h = __ldcg(static_cast<const unsigned short*>(p) + i);
    return dt == 1 ? __half2float(__ushort_as_half(h)) : __bfloat162float(__ushort_as_bfloat16(h));
}

__device__ __forceinline__ void store_act(void* p, size_t i, int dt, float v) {
    if (dt == 0) static_cast<float*>(p)[i] = v;
    else if (dt == 1) static_cast<__half*>(p)[i] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// ------------------------------------------------------------------ Hadamard-128 over a warp
// Lane L holds elements 4L..4L+3 of a 128-vector; returns H128 . v (Sylvester order, scaled by
// 1/sqrt(128)), the transform of src/exl3/expert_exl3.zig:400-414 computed by butterflies.
__device__ __forceinline__ void warp_hadamard128(float (&v)[4]) {
    float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
    v[0] = a0 + a2;
    v[1] = a1 + a3;
    v[2] = a0 - a2;
    v[3] = a1 - a3;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        // upper lanes take other - v, lower lanes v + other: one fma with a lane sign (the
        // product by +-1 is exact, so the result is the same single rounding of the sum)
        const float sgn = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float other = __shfl_xor_sync(0xffffffffu, v[i], m);
            v[i] = fmaf(sgn, v[i], other);
        }
    }
    const float s = 0.08838834764831845f;
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] *= s;
}

}  // namespace sx
