// Expert-parallel routed layer: sx_ep_* (include/sushi_exl3.h).
//
// Rank g of `world` holds experts [g*El, (g+1)*El) (El = E/world).  One call:
//   1. ep_plan (one CTA per destination rank d): scans the rank's rows in order and lists the rows
//      with at least one slot on d; pos[r][d] = the row's place in d's list, or -1.
//   2. ep_gather (one CTA per (list place, d)): copies the listed row of x into the send block of
//      d, with its slots as d-local expert ids (other ranks' slots and unused places carry the
//      sentinel id 0xFFFFFFFF, which the expert chain skips) and scores.
//   3. dispatch: all-to-alls of the fixed-size blocks (rows_cap rows per peer; rows, slot ids and
//      scores) as one group of ncclSend/ncclRecv; this rank's own blocks are device copies.
//   4. the local expert chain (moe_impl) over the world*rows_cap received rows, writing each row's
//      k-order f32 sum over its slots here (the partial) instead of a rounded output.
//   5. combine: all-to-all of the partials back to the rows' owners.
//   6. ep_combine (one CTA per own row): the partials of the ranks the row went to, added in rank
//      order, rounded to the output dtype, plus the shared expert (routed_finish).
// NCCL is loaded with dlopen on first use, so the rest of the library has no NCCL dependency.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <utility>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

#include "sx_internal.h"
#include "sx_moe_impl.cuh"

// Peer transport limits: ranks a communicator can map (the flag arrays hold this many words).
constexpr int kPeerMax = 128;
constexpr int kEpPhases = 6;  // sx_ep_phase_ms

// side: a stream of the communicator's own on which a layer's shared expert runs while the
// dispatch, the local experts and the combine's exchange run on the caller's stream (fork and
// join are the events between the two).  peer: this rank's reserved peer buffer (0 bytes: the
// NCCL transport) and every rank's buffer as mapped here (peer[rank] = own).
struct sx_ep {
    ncclComm_t comm;
    int world, rank, device;
    cudaStream_t side;
    cudaEvent_t fork, join;
    uint8_t* own;
    size_t own_bytes;
    uint8_t* peer[kPeerMax];
    uint32_t* host_counts;  // pinned: the received rows and slots of a host-sized call
    cudaEvent_t phase[kEpPhases + 1];  // sx_ep_phase_timing: the last call's phase boundaries
    bool timing;
};

namespace sx {
namespace {

constexpr uint32_t kSentinel = 0xFFFFFFFFu;

// ------------------------------------------------------------------ NCCL, loaded at run time
struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclCommAbort) comm_abort = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
    char why[160] = "";
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

template <typename F>
bool bind(void* h, const char* name, F& fn) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

const NcclApi& nccl() {
    std::call_once(g_nccl_once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            snprintf(g_nccl.why, sizeof(g_nccl.why), "dlopen libnccl.so.2 failed");
            return;
        }
        NcclApi& a = g_nccl;
        a.ok = bind(h, "ncclGetUniqueId", a.get_unique_id) && bind(h, "ncclCommInitRank", a.comm_init_rank) &&
               bind(h, "ncclCommDestroy", a.comm_destroy) && bind(h, "ncclCommAbort", a.comm_abort) &&
               bind(h, "ncclGroupStart", a.group_start) && bind(h, "ncclGroupEnd", a.group_end) &&
               bind(h, "ncclSend", a.send) && bind(h, "ncclRecv", a.recv) && bind(h, "ncclAllGather", a.all_gather) &&
               bind(h, "ncclGetErrorString", a.error_string);
        if (!a.ok) snprintf(a.why, sizeof(a.why), "libnccl.so.2 lacks a needed symbol");
    });
    return g_nccl;
}

sx_status nccl_status(ncclResult_t r, const char* where) {
    if (r == ncclSuccess) return SX_OK;
    note_detail(where, g_nccl.error_string ? g_nccl.error_string(r) : "nccl error");
    return SX_ERR_NCCL;
}

sx_status nccl_missing() {
    note_detail("nccl", g_nccl.why);
    return SX_ERR_NCCL;
}

// ------------------------------------------------------------------ kernels
struct EpArgs {
    const void* x;          // [rows][D] own rows
    const uint32_t* inds;   // [rows][K] global expert ids
    const float* scores;    // [rows][K]
    int rows, cap, K, D, esz, world, El, Etot;
    int* list;              // [world][cap] own row listed at each send place, -1 past the count
    int* pos;               // [cap][world] the own row's place in each destination's block, or -1
    uint8_t* send_x;        // [world][cap][D] x dtype
    uint32_t* send_inds;    // [world][cap][K] destination-local ids or the sentinel
    float* send_scores;     // [world][cap][K]
};

// Block-wide exclusive scan of 0/1 flags over 256 threads; returns the prefix, sets *total.
__device__ __forceinline__ int block_scan_256(int flag, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned ballot = __ballot_sync(0xffffffffu, flag);
    const int in_warp = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) warp_sums[warp] = __popc(ballot);
    __syncthreads();
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const int c = warp_sums[w];
        before += w < warp ? c : 0;
        all += c;
    }
    __syncthreads();
    *total = all;
    return before + in_warp;
}

__global__ void __launch_bounds__(256) ep_plan_kernel(EpArgs a) {
    __shared__ int warp_sums[8];
    const int d = blockIdx.x;
    int base = 0;
    for (int r0 = 0; r0 < a.rows; r0 += 256) {
        const int r = r0 + threadIdx.x;
        int flag = 0;
        if (r < a.rows) {
            for (int k = 0; k < a.K; k++) {
                const uint32_t e = a.inds[(size_t)r * a.K + k];
                if (e < (uint32_t)a.Etot && (int)(e / (uint32_t)a.El) == d) flag = 1;
            }
        }
        int total;
        const int idx = block_scan_256(flag, warp_sums, &total);
        if (r < a.rows) {
            a.pos[(size_t)r * a.world + d] = flag ? base + idx : -1;
            if (flag) a.list[(size_t)d * a.cap + base + idx] = r;
        }
        base += total;
    }
    for (int i = base + threadIdx.x; i < a.cap; i += blockDim.x) a.list[(size_t)d * a.cap + i] = -1;
}

__global__ void __launch_bounds__(128) ep_gather_kernel(EpArgs a) {
    const int i = blockIdx.x, d = blockIdx.y;
    const size_t place = (size_t)d * a.cap + i;
    const int r = a.list[place];
    uint32_t* mi = a.send_inds + place * a.K;
    float* ms = a.send_scores + place * a.K;
    if (r < 0) {
        for (int k = threadIdx.x; k < a.K; k += blockDim.x) {
            mi[k] = kSentinel;
            ms[k] = 0.0f;
        }
        return;
    }
    for (int k = threadIdx.x; k < a.K; k += blockDim.x) {
        const uint32_t e = a.inds[(size_t)r * a.K + k];
        const bool here = e < (uint32_t)a.Etot && (int)(e / (uint32_t)a.El) == d;
        mi[k] = here ? e - (uint32_t)(d * a.El) : kSentinel;
        ms[k] = here ? a.scores[(size_t)r * a.K + k] : 0.0f;
    }
    const size_t row_bytes = (size_t)a.D * a.esz;  // a multiple of 256 (D % 128 == 0)
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.x) + (size_t)r * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(a.send_x + place * row_bytes);
    for (size_t v = threadIdx.x; v < row_bytes / 16; v += blockDim.x) dst[v] = src[v];
}

struct CombineArgs {
    const float* part;       // [world][cap][D]: from rank d, the partials of the rows sent to d
    const int* pos;          // [cap][world]
    const float* sh_plane;   // [rows][D] f32: the shared expert's output before rounding, or null
    const void* shared;
    const void* shared_gate;
    void* y;
    int rows, cap, D, world, xdt;
};

__global__ void __launch_bounds__(256) ep_combine_kernel(CombineArgs a) {
    const int r = blockIdx.x;
    for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
        float acc = 0.0f;
        for (int g = 0; g < a.world; g++) {
            const int p = a.pos[(size_t)r * a.world + g];
            if (p >= 0) acc += a.part[((size_t)g * a.cap + p) * a.D + d];
        }
        const size_t i = (size_t)r * a.D + d;
        const float sh = a.sh_plane ? round_act(a.sh_plane[i], a.xdt) : a.shared ? load_act(a.shared, i, a.xdt) : 0.0f;
        const float y = routed_finish(acc, a.xdt, a.sh_plane || a.shared, sh, a.shared_gate, r);
        store_act(a.y, (size_t)r * a.D + d, a.xdt, y);
    }
}

// ------------------------------------------------------------------ peer transport (NVLink)
// Every rank's peer buffer has the same layout: a control block of u32 words, then the data
// regions for the call's sizes (rows_cap C, hidden D, topk K, activation bytes esz):
//   recv_x   [G][C][D]  rows source rank g stored here (its list for this rank, in order)
//   recv_ids [G][C][K]  their slots as this rank's local expert ids (kSentinel: another rank's)
//   recv_sc  [G][C][K]  the slots' scores
//   part     [G][C][D]  f32: from expert rank g, the partial of this rank's row at place p of the
//                       list this rank sent to g
// Control words (zero at reservation; flags only grow):
//   seq                  the calls this rank has begun (its plan kernel counts them)
//   disp_flag[g]         the last call whose rows rank g has stored here
//   comb_flag[g]         the last call whose partials rank g has stored here
//   recv_cnt[g]          rows rank g stored here in that call
//   recv_slots[g]        the slots of those rows on this rank's experts
//   disp_done[g], red_done  this rank's own CTA counters (last CTA signals), reset by that CTA
constexpr int kCtrlSeq = 0, kCtrlDispFlag = kPeerMax, kCtrlCombFlag = 2 * kPeerMax, kCtrlRecvCnt = 3 * kPeerMax,
              kCtrlRecvSlots = 4 * kPeerMax, kCtrlDispDone = 5 * kPeerMax, kCtrlRedDone = 6 * kPeerMax,
              kCtrlPlanDone = 6 * kPeerMax + 1;
// Up to this many rows per rank one kernel plans and dispatches (each CTA of a destination
// recomputes that destination's list, which costs little at these sizes, and stores its share).
constexpr int kFusedDispatchRows = 64;
// From this many rows per rank a call reads the received counts back to the host (one host
// synchronisation) and sizes the expert chain's launches to the rows and slots it received; below
// it the launches are sized for every place and the call never waits on the host.
constexpr int kHostSizedRows = 1024;
// Up to this many own rows (the decode chain's row limit) the peer transport runs the layer's
// shared expert inside the local expert chain's launches (over the rank's own rows, its plane
// after the routed slots') instead of on the side stream, whose concurrent launches would hold
// the SMs the exchange's small kernels wait for.
constexpr int kEpFoldRows = 16;
constexpr size_t kCtrlBytes = 16384;

struct PeerLayout {
    size_t recv_x, recv_ids, recv_sc, part, total;
};

PeerLayout peer_layout(int G, int C, int D, int K, int esz) {
    auto up256 = [](size_t v) { return (v + 255) / 256 * 256; };
    PeerLayout l{};
    const size_t places = (size_t)G * C;
    size_t off = kCtrlBytes;
    l.recv_x = off; off = up256(off + places * D * esz);
    l.recv_ids = off; off = up256(off + places * K * sizeof(uint32_t));
    l.recv_sc = off; off = up256(off + places * K * sizeof(float));
    l.part = off; off = up256(off + places * D * sizeof(float));
    l.total = off;
    return l;
}

struct PeerArgs {
    uint8_t* base[kPeerMax];  // every rank's buffer as mapped on this device (base[me] = own)
    PeerLayout lay;
    int me;
};

__device__ __forceinline__ uint32_t* ctrl(uint8_t* base) { return reinterpret_cast<uint32_t*>(base); }

// Programmatic dependent launch of the peer kernels: the next kernel of the stream may start its
// launch at once; this one waits for its predecessor's completion before any global access (so
// the order of calls, and of the peer-buffer reuse that follows from it, is the stream order).
__device__ __forceinline__ void ep_pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// A CTA's stores (peer ones included) become visible at system scope before its arrival: called
// by thread 0 after a block barrier that follows the CTA's stores, one system fence for the whole
// CTA (the barrier orders the other threads' stores before it), as a flag protocol over NVLink
// needs no fence per thread.
__device__ __forceinline__ void cta_stores_released() { __threadfence_system(); }

// The last of `total` CTAs to arrive on `counter` (a word of this rank's own control block)
// returns true, after every arriving CTA's stores (each released by cta_stores_released before its
// arrival) are ordered before its own later stores; it resets the counter for the next call.  One
// CTA arrives last without an atomic.  Called by thread 0 after cta_stores_released().
__device__ __forceinline__ bool last_to_arrive(uint32_t* counter, uint32_t total) {
    if (total == 1) return true;
    const uint32_t prev = atomicAdd(counter, 1u);
    if (prev + 1 != total) return false;
    __threadfence_system();
    *counter = 0;
    return true;
}

// Plan for the peer transport: ep_plan_kernel's lists and places, plus the per-destination counts
// and (block 0) the start of a new call in this rank's control block.
// cnt[d]: rows for destination d; cnt[world + d]: their slots on d's experts.
__global__ void __launch_bounds__(256) ep_peer_plan_kernel(EpArgs a, int* cnt, uint32_t* own_ctrl) {
    __shared__ int warp_sums[8];
    __shared__ int slot_sum;
    const int d = blockIdx.x;
    if (d == 0 && threadIdx.x == 0) own_ctrl[kCtrlSeq] += 1u;
    if (threadIdx.x == 0) slot_sum = 0;
    int base = 0, slots = 0;
    for (int r0 = 0; r0 < a.rows; r0 += 256) {
        const int r = r0 + threadIdx.x;
        int flag = 0;
        if (r < a.rows) {
            for (int k = 0; k < a.K; k++) {
                const uint32_t e = a.inds[(size_t)r * a.K + k];
                if (e < (uint32_t)a.Etot && (int)(e / (uint32_t)a.El) == d) {
                    flag = 1;
                    slots++;
                }
            }
        }
        int total;
        const int idx = block_scan_256(flag, warp_sums, &total);
        if (r < a.rows) {
            a.pos[(size_t)r * a.world + d] = flag ? base + idx : -1;
            if (flag) a.list[(size_t)d * a.cap + base + idx] = r;
        }
        base += total;
    }
    if (slots) atomicAdd(&slot_sum, slots);
    __syncthreads();
    if (threadIdx.x == 0) {
        cnt[d] = base;
        cnt[a.world + d] = slot_sum;
    }
}

// Dispatch (grid: B x G blocks): destination d = blockIdx.y; places i = blockIdx.x, +B, ... below
// cnt[d]: row list[d][i] of x and its slots (d-local ids, scores) stored into d's recv regions at
// [me][i].  The last of d's B blocks stores the count and raises d's flag for this rank.
__global__ void __launch_bounds__(256) ep_peer_dispatch_kernel(EpArgs a, const int* cnt, PeerArgs p) {
    const int d = blockIdx.y;
    uint8_t* dst = p.base[d];
    const uint32_t seq = ctrl(p.base[p.me])[kCtrlSeq];
    const int n = cnt[d];
    const size_t row_bytes = (size_t)a.D * a.esz;  // a multiple of 256 (D % 128 == 0)
    const size_t slot0 = (size_t)p.me * a.cap;
    uint32_t* ids = reinterpret_cast<uint32_t*>(dst + p.lay.recv_ids);
    float* sc = reinterpret_cast<float*>(dst + p.lay.recv_sc);
    for (int i = blockIdx.x; i < n; i += gridDim.x) {
        const int r = a.list[(size_t)d * a.cap + i];
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.x) + (size_t)r * row_bytes);
        uint4* out = reinterpret_cast<uint4*>(dst + p.lay.recv_x + (slot0 + i) * row_bytes);
        for (size_t v = threadIdx.x; v < row_bytes / 16; v += blockDim.x) out[v] = src[v];
        for (int k = threadIdx.x; k < a.K; k += blockDim.x) {
            const uint32_t e = a.inds[(size_t)r * a.K + k];
            const bool here = e < (uint32_t)a.Etot && (int)(e / (uint32_t)a.El) == d;
            ids[(slot0 + i) * a.K + k] = here ? e - (uint32_t)(d * a.El) : kSentinel;
            sc[(slot0 + i) * a.K + k] = here ? a.scores[(size_t)r * a.K + k] : 0.0f;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        cta_stores_released();
        if (last_to_arrive(&ctrl(p.base[p.me])[kCtrlDispDone + d], gridDim.x)) {
            st_relaxed_sys(&ctrl(dst)[kCtrlRecvCnt + p.me], (uint32_t)n);
            st_relaxed_sys(&ctrl(dst)[kCtrlRecvSlots + p.me], (uint32_t)cnt[a.world + d]);
            st_release_sys(&ctrl(dst)[kCtrlDispFlag + p.me], seq);  // the counts and rows before the flag
        }
    }
}

// Plan and dispatch in one kernel for small calls (grid: B x G blocks; rows <= 256): CTA (x, d)
// computes destination d's list and slot count (x == 0 also writes the places the combine reads),
// stores its share of the list's rows and slots into d's receive region, and arrives on d's
// counter; the last to arrive stores the counts and raises d's flag.  The call's number is read
// by every CTA before it arrives, and the last CTA of the grid advances it.
__global__ void __launch_bounds__(256) ep_peer_plan_dispatch_kernel(EpArgs a, PeerArgs p) {
    __shared__ int list[256];
    __shared__ int warp_sums[8];
    __shared__ int slot_sum;
    ep_pdl_enter();
    const int d = blockIdx.y;
    uint32_t* c = ctrl(p.base[p.me]);
    uint8_t* dst = p.base[d];
    const uint32_t seq = c[kCtrlSeq] + 1u;
    if (threadIdx.x == 0) slot_sum = 0;
    const int r = threadIdx.x;
    int flag = 0, slots = 0;
    if (r < a.rows) {
        for (int k = 0; k < a.K; k++) {
            const uint32_t e = a.inds[(size_t)r * a.K + k];
            if (e < (uint32_t)a.Etot && (int)(e / (uint32_t)a.El) == d) {
                flag = 1;
                slots++;
            }
        }
    }
    int n;
    const int idx = block_scan_256(flag, warp_sums, &n);
    if (flag) list[idx] = r;
    if (slots) atomicAdd(&slot_sum, slots);
    if (blockIdx.x == 0 && r < a.rows) a.pos[(size_t)r * a.world + d] = flag ? idx : -1;
    __syncthreads();
    const size_t row_bytes = (size_t)a.D * a.esz;
    const size_t slot0 = (size_t)p.me * a.cap;
    uint32_t* ids = reinterpret_cast<uint32_t*>(dst + p.lay.recv_ids);
    float* sc = reinterpret_cast<float*>(dst + p.lay.recv_sc);
    for (int i = blockIdx.x; i < n; i += gridDim.x) {
        const int rr = list[i];
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.x) + (size_t)rr * row_bytes);
        uint4* out = reinterpret_cast<uint4*>(dst + p.lay.recv_x + (slot0 + i) * row_bytes);
        for (size_t v = threadIdx.x; v < row_bytes / 16; v += blockDim.x) out[v] = src[v];
        for (int k = threadIdx.x; k < a.K; k += blockDim.x) {
            const uint32_t e = a.inds[(size_t)rr * a.K + k];
            const bool here = e < (uint32_t)a.Etot && (int)(e / (uint32_t)a.El) == d;
            ids[(slot0 + i) * a.K + k] = here ? e - (uint32_t)(d * a.El) : kSentinel;
            sc[(slot0 + i) * a.K + k] = here ? a.scores[(size_t)rr * a.K + k] : 0.0f;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        cta_stores_released();
        if (last_to_arrive(&c[kCtrlDispDone + d], gridDim.x)) {
            st_relaxed_sys(&ctrl(dst)[kCtrlRecvCnt + p.me], (uint32_t)n);
            st_relaxed_sys(&ctrl(dst)[kCtrlRecvSlots + p.me], (uint32_t)slot_sum);
            st_release_sys(&ctrl(dst)[kCtrlDispFlag + p.me], seq);  // the counts and rows before the flag
        }
        // every CTA read the call's number before arriving: the last one advances it (later
        // kernels of the stream read it)
        if (atomicAdd(&c[kCtrlPlanDone], 1u) + 1 == gridDim.x * gridDim.y) {
            __threadfence();  // after every CTA's read of the number (each fenced before arriving)
            c[kCtrlPlanDone] = 0;
            c[kCtrlSeq] = seq;
        }
    }
}

// Every rank's rows for this call have arrived (one block; thread g waits for rank g's flag).
// The expert chain that follows reads the received rows and counts.
__global__ void ep_peer_recv_wait_kernel(PeerArgs p, int world) {
    uint32_t* c = ctrl(p.base[p.me]);
    const uint32_t seq = c[kCtrlSeq];
    for (int g = threadIdx.x; g < world; g += blockDim.x) wait_flag(&c[kCtrlDispFlag + g], seq);
}

// The received rows' partials (grid-stride over (live row, 512-column block) units): the row's
// slots on this rank summed in k order in f32, stored into the row's owner's part region at
// [me][i].  The last block raises every rank's combine flag for this rank.
struct ReducePushArgs {
    const float* yslot;     // [G*C*K][D] per-slot planes of the local chain
    const uint32_t* ids;    // [G*C][K] this rank's recv_ids
    int world, cap, K, D, El;
};

__global__ void __launch_bounds__(128) ep_peer_reduce_push_kernel(ReducePushArgs a, PeerArgs p) {
    __shared__ int pre[kPeerMax + 1];
    ep_pdl_enter();
    uint32_t* c = ctrl(p.base[p.me]);
    const uint32_t seq = c[kCtrlSeq];
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int g = 0; g < a.world; g++) {
            pre[g] = acc;
            acc += min((int)c[kCtrlRecvCnt + g], a.cap);
        }
        pre[a.world] = acc;
    }
    __syncthreads();
    const int nb = (a.D + 511) / 512;
    const long long units = (long long)pre[a.world] * nb;
    for (long long u = blockIdx.x; u < units; u += gridDim.x) {
        const int j = (int)(u / nb), cb = (int)(u % nb);
        int g = 0;
        while (g + 1 < a.world && pre[g + 1] <= j) g++;
        const int i = j - pre[g];
        const size_t place = (size_t)g * a.cap + i;
        const int d = cb * 512 + threadIdx.x * 4;
        if (d >= a.D) continue;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int k = 0; a.yslot && k < a.K; k++) {  // no planes: no expert ran (no slot reached this rank)
            if (a.ids[place * a.K + k] >= (uint32_t)a.El) continue;
            const float4 v = *reinterpret_cast<const float4*>(a.yslot + (place * a.K + k) * a.D + d);
            acc[0] += v.x;
            acc[1] += v.y;
            acc[2] += v.z;
            acc[3] += v.w;
        }
        float* dst = reinterpret_cast<float*>(p.base[g] + p.lay.part) + ((size_t)p.me * a.cap + i) * a.D + d;
        *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        cta_stores_released();
        if (last_to_arrive(&c[kCtrlRedDone], gridDim.x))
            for (int g = 0; g < a.world; g++) st_release_sys(&ctrl(p.base[g])[kCtrlCombFlag + p.me], seq);
    }
}

// Combine for the peer transport (one block per own row; at least one block): waits for every
// rank's partials of this call, then as ep_combine_kernel with the partials in this rank's part
// region ([g][place]).
__global__ void __launch_bounds__(256) ep_peer_combine_kernel(CombineArgs a, PeerArgs p) {
    ep_pdl_enter();
    uint32_t* c = ctrl(p.base[p.me]);
    const uint32_t seq = c[kCtrlSeq];
    if (threadIdx.x < 32)
        for (int g = threadIdx.x; g < a.world; g += 32) wait_flag(&c[kCtrlCombFlag + g], seq);
    __syncthreads();
    const int r = blockIdx.x;
    if (r >= a.rows) return;
    const float* part = reinterpret_cast<const float*>(p.base[p.me] + p.lay.part);
    for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
        float acc = 0.0f;
        for (int g = 0; g < a.world; g++) {
            const int q = a.pos[(size_t)r * a.world + g];
            if (q >= 0) acc += __ldcg(part + ((size_t)g * a.cap + q) * a.D + d);  // peers' stores: L2, not L1
        }
        const size_t i = (size_t)r * a.D + d;
        const float sh = a.sh_plane ? round_act(a.sh_plane[i], a.xdt) : a.shared ? load_act(a.shared, i, a.xdt) : 0.0f;
        const float y = routed_finish(acc, a.xdt, a.sh_plane || a.shared, sh, a.shared_gate, r);
        store_act(a.y, (size_t)r * a.D + d, a.xdt, y);
    }
}

// ------------------------------------------------------------------ workspace
constexpr size_t kAlign = 256;
size_t up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

struct EpWs {
    size_t list, pos, cnt, send_x, send_inds, send_scores, recv_x, recv_inds, recv_scores, part_send, part_recv, moe,
        total;
    size_t moe_bytes;
    size_t sh_plane, sh_scratch;  // the shared expert's plane [cap][D] f32 and scratch (0 bytes without one)
};

// The layout for a local layer of `ng` rate groups (one for a uniform bank) over El experts.  With
// the peer transport (peer) the exchanged blocks live in the peer buffers, not here.
EpWs ep_ws_layout(const MoeGroup* g, int ng, int El, int world, int cap, int K, int esz, const sx_bank* sh = nullptr,
                  bool peer = false) {
    EpWs w{};
    const int D = g[0].bank.gate.in_features;
    const size_t places = (size_t)world * cap;
    const size_t xfer = peer ? 0 : places;  // places of the NCCL transport's own blocks
    size_t off = 0;
    w.list = off; off = up(off + places * sizeof(int));
    w.pos = off; off = up(off + places * sizeof(int));
    w.cnt = off; off = up(off + (size_t)2 * world * sizeof(int));
    w.send_x = off; off = up(off + xfer * D * esz);
    w.send_inds = off; off = up(off + xfer * K * sizeof(uint32_t));
    w.send_scores = off; off = up(off + xfer * K * sizeof(float));
    w.recv_x = off; off = up(off + xfer * D * esz);
    w.recv_inds = off; off = up(off + xfer * K * sizeof(uint32_t));
    w.recv_scores = off; off = up(off + xfer * K * sizeof(float));
    w.part_send = off; off = up(off + xfer * D * sizeof(float));
    w.part_recv = off; off = up(off + xfer * D * sizeof(float));
    // a rank receives about rows_cap * K valid slots (every rank's rows_cap rows, K slots each,
    // spread over the world): that, not the places' sentinel-padded slots, picks its expert path
    w.moe_bytes = moe_groups_ws(g, ng, El, (int32_t)places, K, (long long)cap * K);
    if (peer && sh && cap <= kEpFoldRows)
        w.moe_bytes = std::max(w.moe_bytes, moe_groups_ws(g, ng, El, (int32_t)places, K, (long long)cap * K, sh,
                                                          nullptr, nullptr, cap));
    // a large call sizes its chain to the slots it received, which may pick the tensor-core path
    if (cap >= kHostSizedRows)
        w.moe_bytes = std::max(w.moe_bytes, moe_groups_ws(g, ng, El, (int32_t)places, K, (long long)places * K));
    w.moe = off; off = up(off + w.moe_bytes);
    w.sh_plane = w.sh_scratch = off;
    if (sh) {
        off = up(off + (size_t)cap * D * sizeof(float));
        w.sh_scratch = off;
        off = up(off + shared_expert_ws(sh, cap));
    }
    w.total = off;
    return w;
}

size_t dtype_size(int dt) { return dt == SX_DT_F32 ? 4 : 2; }

// All-to-alls of several buffers in one NCCL group: for each (send, recv, bytes), block p of send
// goes to rank p and block p of recv comes from rank p; the own blocks are device copies.
struct A2A {
    const void* send;
    void* recv;
    size_t bytes;
};

sx_status all_to_all(const sx_ep* ep, const A2A* bufs, int nb, cudaStream_t s) {
    const NcclApi& n = nccl();
    for (int b = 0; b < nb; b++) {
        const uint8_t* sb = static_cast<const uint8_t*>(bufs[b].send);
        uint8_t* rb = static_cast<uint8_t*>(bufs[b].recv);
        const size_t bytes = bufs[b].bytes;
        const cudaError_t ce = cudaMemcpyAsync(rb + (size_t)ep->rank * bytes, sb + (size_t)ep->rank * bytes, bytes,
                                               cudaMemcpyDeviceToDevice, s);
        if (ce != cudaSuccess) return cuda_status(ce, "ep own block copy");
    }
    if (ep->world == 1) return SX_OK;
    sx_status st = nccl_status(n.group_start(), "ncclGroupStart");
    if (st) return st;
    for (int b = 0; b < nb && !st; b++) {
        const uint8_t* sb = static_cast<const uint8_t*>(bufs[b].send);
        uint8_t* rb = static_cast<uint8_t*>(bufs[b].recv);
        const size_t bytes = bufs[b].bytes;
        for (int p = 0; p < ep->world && !st; p++) {
            if (p == ep->rank) continue;
            st = nccl_status(n.send(sb + (size_t)p * bytes, bytes, ncclUint8, p, ep->comm, s), "ncclSend");
            if (!st) st = nccl_status(n.recv(rb + (size_t)p * bytes, bytes, ncclUint8, p, ep->comm, s), "ncclRecv");
        }
    }
    const sx_status end = nccl_status(n.group_end(), "ncclGroupEnd");
    return st ? st : end;
}

// The side stream and its events (a failed stream sync is not reported: the handle goes anyway).
void release_side(sx_ep* ep) {
    if (ep->side) {
        cudaStreamSynchronize(ep->side);
        cudaStreamDestroy(ep->side);
    }
    if (ep->fork) cudaEventDestroy(ep->fork);
    if (ep->join) cudaEventDestroy(ep->join);
    ep->side = nullptr;
    ep->fork = ep->join = nullptr;
}

// The peer mappings and this rank's buffer (local: every peer has stopped using them once the
// caller synchronised its streams; the reservation's own barrier precedes a replacement).
void release_peer(sx_ep* ep) {
    for (int g = 0; g < kPeerMax; g++) {
        if (ep->peer[g] && g != ep->rank) cudaIpcCloseMemHandle(ep->peer[g]);
        ep->peer[g] = nullptr;
    }
    if (ep->own) cudaFree(ep->own);
    if (ep->host_counts) cudaFreeHost(ep->host_counts);
    ep->own = nullptr;
    ep->own_bytes = 0;
    ep->host_counts = nullptr;
}

// Every rank's `bytes`-byte block of `mine` gathered into `all` [world][bytes] on the host, over the
// communicator (the side stream, synchronised).  Also the reservation's barrier.
sx_status gather_host(sx_ep* ep, const void* mine, size_t bytes, void* all) {
    const NcclApi& n = nccl();
    if (!n.ok) return nccl_missing();
    uint8_t* dev = nullptr;
    cudaError_t ce = cudaMalloc(&dev, bytes * (ep->world + 1));
    if (ce != cudaSuccess) return cuda_status(ce, "peer handle exchange buffer");
    sx_status st = SX_OK;
    ce = cudaMemcpy(dev, mine, bytes, cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) st = cuda_status(ce, "peer handle exchange copy");
    if (!st) st = nccl_status(n.all_gather(dev, dev + bytes, bytes, ncclUint8, ep->comm, ep->side), "ncclAllGather");
    if (!st && (ce = cudaStreamSynchronize(ep->side)) != cudaSuccess) st = cuda_status(ce, "peer handle exchange sync");
    if (!st && (ce = cudaMemcpy(all, dev + bytes, bytes * ep->world, cudaMemcpyDeviceToHost)) != cudaSuccess)
        st = cuda_status(ce, "peer handle exchange copy back");
    cudaFree(dev);
    return st;
}

}  // namespace
}  // namespace sx

using namespace sx;

extern "C" {

size_t sx_ep_peer_bytes(const sx_ep* ep, int32_t rows_cap, int32_t hidden, int32_t topk, sx_dtype dtype) {
    if (!ep || rows_cap < 1 || hidden < 128 || hidden % 128 || topk < 1 || !dtype_ok(dtype)) return 0;
    return peer_layout(ep->world, rows_cap, hidden, topk, (int)dtype_size(dtype)).total;
}

size_t sx_ep_peer_reserved(const sx_ep* ep) { return ep ? ep->own_bytes : 0; }

sx_status sx_ep_phase_timing(sx_ep* ep, int32_t enable) {
    if (!ep) return SX_ERR_NULL_POINTER;
    if (enable && !ep->timing) {
        for (int i = 0; i <= kEpPhases; i++) {
            const cudaError_t ce = cudaEventCreate(&ep->phase[i]);
            if (ce != cudaSuccess) {
                for (int j = 0; j < i; j++) cudaEventDestroy(ep->phase[j]);
                return cuda_status(ce, "phase timing events");
            }
        }
        ep->timing = true;
    } else if (!enable && ep->timing) {
        for (int i = 0; i <= kEpPhases; i++) cudaEventDestroy(ep->phase[i]);
        ep->timing = false;
    }
    return SX_OK;
}

sx_status sx_ep_phase_ms(sx_ep* ep, float ms[6]) {
    if (!ep || !ms) return SX_ERR_NULL_POINTER;
    if (!ep->timing) return SX_ERR_BAD_SHAPE;
    cudaError_t ce = cudaEventSynchronize(ep->phase[kEpPhases]);
    for (int i = 0; ce == cudaSuccess && i < kEpPhases; i++) ce = cudaEventElapsedTime(&ms[i], ep->phase[i], ep->phase[i + 1]);
    return ce == cudaSuccess ? SX_OK : cuda_status(ce, "phase timing");
}

sx_status sx_ep_reserve_peer(sx_ep* ep, size_t bytes) {
    if (!ep) return SX_ERR_NULL_POINTER;
    if (ep->world > kPeerMax) return SX_ERR_BAD_SHAPE;
    if (bytes > 0 && bytes <= ep->own_bytes) return SX_OK;
    if (bytes == 0 && !ep->own) return SX_OK;
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != ep->device) return SX_ERR_BAD_SHAPE;  // the communicator's device must be current
    cudaError_t ce = cudaDeviceSynchronize();
    if (ce != cudaSuccess) return cuda_status(ce, "peer reservation sync");
    int32_t one = 1;
    int32_t* all = new (std::nothrow) int32_t[ep->world];
    if (!all) return SX_ERR_BAD_SHAPE;
    // every rank has finished with the old buffers before any rank frees its own
    sx_status st = gather_host(ep, &one, sizeof(one), all);
    delete[] all;
    if (st) return st;
    release_peer(ep);
    if (bytes == 0) return SX_OK;
    const size_t size = (bytes + (2u << 20) - 1) / (2u << 20) * (2u << 20);
    uint8_t* own = nullptr;
    int32_t ok = 1;
    cudaIpcMemHandle_t h{};
    if ((ce = cudaMallocHost(&ep->host_counts, 2 * kPeerMax * sizeof(uint32_t))) != cudaSuccess ||
        (ce = cudaMalloc(&own, size)) != cudaSuccess || (ce = cudaMemset(own, 0, size)) != cudaSuccess ||
        (ce = cudaDeviceSynchronize()) != cudaSuccess || (ce = cudaIpcGetMemHandle(&h, own)) != cudaSuccess) {
        note_cuda_error(ce, "peer buffer");
        ok = 0;
    }
    struct Entry {
        cudaIpcMemHandle_t h;
        int32_t ok;
    };
    Entry mine{h, ok};
    Entry* ents = new (std::nothrow) Entry[ep->world];
    if (!ents) {
        if (own) cudaFree(own);
        return SX_ERR_BAD_SHAPE;
    }
    st = gather_host(ep, &mine, sizeof(mine), ents);
    bool every = st == SX_OK;
    for (int g = 0; every && g < ep->world; g++) every = ents[g].ok != 0;
    ep->own = own;
    ep->peer[ep->rank] = own;
    int32_t mapped = every ? 1 : 0;
    for (int g = 0; mapped && g < ep->world; g++) {
        if (g == ep->rank) continue;
        void* p = nullptr;
        if ((ce = cudaIpcOpenMemHandle(&p, ents[g].h, cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) {
            note_cuda_error(ce, "cudaIpcOpenMemHandle");
            mapped = 0;
            break;
        }
        ep->peer[g] = static_cast<uint8_t*>(p);
    }
    delete[] ents;
    if (st) {
        release_peer(ep);
        return st;
    }
    // every rank learns whether every rank mapped every peer: all keep the buffers or none does
    int32_t* agree = new (std::nothrow) int32_t[ep->world];
    if (!agree) {
        release_peer(ep);
        return SX_ERR_BAD_SHAPE;
    }
    st = gather_host(ep, &mapped, sizeof(mapped), agree);
    bool all_mapped = st == SX_OK;
    for (int g = 0; all_mapped && g < ep->world; g++) all_mapped = agree[g] != 0;
    delete[] agree;
    if (!all_mapped) {
        release_peer(ep);
        return st ? st : SX_ERR_PEER_ACCESS;
    }
    ep->own_bytes = size;
    return SX_OK;
}

sx_status sx_ep_unique_id(uint8_t id[128]) {
    if (!id) return SX_ERR_NULL_POINTER;
    const NcclApi& n = nccl();
    if (!n.ok) return nccl_missing();
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    ncclUniqueId u;
    sx_status st = nccl_status(n.get_unique_id(&u), "ncclGetUniqueId");
    if (st) return st;
    memcpy(id, &u, 128);
    return SX_OK;
}

sx_status sx_ep_init(const uint8_t id[128], int32_t world, int32_t rank, sx_ep** out) {
    if (!id || !out) return SX_ERR_NULL_POINTER;
    *out = nullptr;
    if (world < 1 || rank < 0 || rank >= world) return SX_ERR_BAD_SHAPE;
    const NcclApi& n = nccl();
    if (!n.ok) return nccl_missing();
    ncclUniqueId u;
    memcpy(&u, id, 128);
    sx_ep* ep = new (std::nothrow) sx_ep();
    if (!ep) return SX_ERR_BAD_SHAPE;
    ep->world = world;
    ep->rank = rank;
    cudaGetDevice(&ep->device);
    ep->side = nullptr;
    ep->fork = ep->join = nullptr;
    cudaError_t ce = cudaStreamCreateWithFlags(&ep->side, cudaStreamNonBlocking);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&ep->fork, cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&ep->join, cudaEventDisableTiming);
    if (ce != cudaSuccess) {
        release_side(ep);
        delete ep;
        return cuda_status(ce, "expert-parallel side stream");
    }
    sx_status st = nccl_status(n.comm_init_rank(&ep->comm, world, u, rank), "ncclCommInitRank");
    if (st) {
        release_side(ep);
        delete ep;
        return st;
    }
    *out = ep;
    return SX_OK;
}

sx_status sx_ep_destroy(sx_ep* ep) {
    if (!ep) return SX_ERR_NULL_POINTER;
    release_side(ep);
    release_peer(ep);
    sx_ep_phase_timing(ep, 0);
    const sx_status st = nccl_status(nccl().comm_destroy(ep->comm), "ncclCommDestroy");
    delete ep;
    return st;
}

sx_status sx_ep_abort(sx_ep* ep) {
    if (!ep) return SX_ERR_NULL_POINTER;
    const sx_status st = nccl_status(nccl().comm_abort(ep->comm), "ncclCommAbort");
    release_side(ep);
    release_peer(ep);
    sx_ep_phase_timing(ep, 0);
    delete ep;
    return st;
}

sx_status sx_ep_info(const sx_ep* ep, int32_t* world, int32_t* rank) {
    if (!ep) return SX_ERR_NULL_POINTER;
    if (world) *world = ep->world;
    if (rank) *rank = ep->rank;
    return SX_OK;
}

size_t sx_ep_workspace_bytes(const sx_ep* ep, const sx_bank* local_bank, int32_t rows_cap, int32_t topk,
                             sx_dtype dtype) {
    if (!ep || !local_bank || rows_cap < 1 || topk < 1 || !dtype_ok(dtype)) return 0;
    const MoeGroup g{*local_bank, 0};
    return ep_ws_layout(&g, 1, local_bank->gate.experts, ep->world, rows_cap, topk, (int)dtype_size(dtype), nullptr,
                        ep->own_bytes > 0)
        .total;
}

size_t sx_ep_ragged_workspace_bytes(const sx_ep* ep, const sx_ragged* local, int32_t rows_cap, int32_t topk,
                                    sx_dtype dtype) {
    if (!ep || !local || rows_cap < 1 || topk < 1 || !dtype_ok(dtype)) return 0;
    MoeGroup g[kMaxGroups];
    int ng = 0;
    if (ragged_groups(local, g, &ng) != SX_OK) return 0;
    return ep_ws_layout(g, ng, local->experts, ep->world, rows_cap, topk, (int)dtype_size(dtype), nullptr,
                        ep->own_bytes > 0)
        .total;
}

}  // extern "C"

namespace sx {
namespace {

// A peer kernel launched with programmatic dependent launch (its first act: ep_pdl_enter).
template <typename... KArgs, typename... Args>
cudaError_t launch_ep(void (*kern)(KArgs...), dim3 grid, int threads, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Records phase boundary i of the call on `s` when phase timing is on: a plain record, or during
// stream capture an external one (the graph records it at each replay).
void mark(sx_ep* ep, int i, cudaStream_t s) {
    if (!ep->timing) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) cs = cudaStreamCaptureStatusNone;
    if (cs == cudaStreamCaptureStatusActive) cudaEventRecordWithFlags(ep->phase[i], s, cudaEventRecordExternal);
    else cudaEventRecord(ep->phase[i], s);
}

// The peer transport's call after the admission checks and the shared-expert fork: plan,
// dispatch into the owners' buffers, wait for every rank's rows, the local chain over the received
// rows only, reduce + push of the partials into the token owners' buffers, join, combine.
// `join` joins the side stream into the caller's before the combine (which reads its plane).
template <typename Join, typename Fork>
sx_status ep_peer_moe(sx_ep* ep, sx_stream stream, const MoeGroup* groups, int ng, int El, const sx_decode* dec,
                      const EpArgs& a, const PeerLayout& PL, const EpWs& L, uint8_t* ws, int rows, int topk,
                      int clamp_limit, const float* sh_plane, const void* shared, const void* shared_gate, void* y,
                      sx_dtype dtype, Join& join, const sx_bank* fold_bank, const sx_decode* fold_dec,
                      Fork& fork_side) {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int G = ep->world, C = a.cap, D = a.D;
    const size_t places = (size_t)G * C;
    PeerArgs pa{};
    for (int g = 0; g < G; g++) pa.base[g] = ep->peer[g];
    pa.lay = PL;
    pa.me = ep->rank;
    uint8_t* own = ep->own;
    int* cnt = reinterpret_cast<int*>(ws + L.cnt);

    mark(ep, 0, s);
    cudaError_t e = cudaSuccess;
    if (C <= kFusedDispatchRows) {
        const int B = std::max(1, std::min(C, 8));
        if ((e = launch_ep(ep_peer_plan_dispatch_kernel, dim3(B, G), 256, s, a, pa)) != cudaSuccess)
            return cuda_status(e, "ep peer plan+dispatch launch");
    } else {
        ep_peer_plan_kernel<<<G, 256, 0, s>>>(a, cnt, reinterpret_cast<uint32_t*>(own));
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "ep peer plan launch");
        const int B = std::max(1, std::min(C, std::max(4, 8 * sm_count() / G)));
        ep_peer_dispatch_kernel<<<dim3(B, G), 256, 0, s>>>(a, cnt, pa);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "ep peer dispatch launch");
    }
    sx_status st = fork_side();  // the shared expert on the side stream (large calls)
    if (st) return st;
    mark(ep, 1, s);
    // The wait for every rank's rows: its own kernel when the counts come back to the host, else
    // the first thing route_prep does (MoeSegments::wait_flags).
    const bool host_sized = C >= kHostSizedRows;
    if (host_sized) {
        ep_peer_recv_wait_kernel<<<1, 128, 0, s>>>(pa, G);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "ep peer wait launch");
    }

    // Large calls: the received counts come back to the host, and the chain's launches are sized
    // to them (the places' bound would launch mostly idle CTAs once rows_cap x world is large).
    long long live_rows = (long long)places, live_slots = -1;
    if (host_sized) {
        e = cudaMemcpyAsync(ep->host_counts, own + kCtrlRecvCnt * sizeof(uint32_t), 2 * kPeerMax * sizeof(uint32_t),
                            cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_status(e, "ep peer received counts");
        live_rows = live_slots = 0;
        for (int g = 0; g < G; g++) {
            live_rows += std::min<long long>(ep->host_counts[g], C);
            live_slots += ep->host_counts[kPeerMax + g];
        }
        live_slots = std::min(live_slots, live_rows * topk);
    }
    mark(ep, 2, s);
    const MoeSegments seg{reinterpret_cast<const int*>(own) + kCtrlRecvCnt, C, G, live_slots,
                          host_sized ? nullptr : reinterpret_cast<const uint32_t*>(own) + kCtrlDispFlag,
                          reinterpret_cast<const uint32_t*>(own) + kCtrlSeq};
    const uint32_t* ids = reinterpret_cast<const uint32_t*>(own + PL.recv_ids);
    float* yslot = nullptr;
    // the shared expert over this rank's own rows rides the local chain (fold_bank, small calls)
    const SharedRows own_rows{a.x, rows};
    const sx_bank* fb = fold_bank && rows > 0 ? fold_bank : nullptr;
    if (live_slots != 0 || fb)  // a rank no slot reached (skewed routing) has no experts to run
        st = moe_run(stream, groups, ng, El, dec, own + PL.recv_x, dtype, (int32_t)places, ids,
                     reinterpret_cast<const float*>(own + PL.recv_sc), topk, nullptr, nullptr, clamp_limit, nullptr,
                     ws + L.moe, L.moe_bytes, nullptr, live_slots >= 0 ? live_slots : (long long)C * topk, fb,
                     fold_dec, &seg, &yslot, fb ? &own_rows : nullptr);
    if (st) return st;
    if (fb) sh_plane = yslot + places * topk * D;
    mark(ep, 3, s);
    const ReducePushArgs rp{yslot, ids, G, C, topk, D, El};
    const long long units = std::max(1LL, live_rows) * ((D + 511) / 512);
    const int grid = (int)std::max(1LL, std::min(units, (long long)8 * sm_count()));
    if ((e = launch_ep(ep_peer_reduce_push_kernel, dim3(grid), 128, s, rp, pa)) != cudaSuccess)
        return cuda_status(e, "ep peer reduce launch");
    mark(ep, 4, s);

    if ((st = join(SX_OK))) return st;
    mark(ep, 5, s);
    CombineArgs c{};
    c.pos = a.pos;
    c.sh_plane = sh_plane;
    c.shared = shared;
    c.shared_gate = shared_gate;
    c.y = y;
    c.rows = rows;
    c.cap = C;
    c.D = D;
    c.world = G;
    c.xdt = dtype;
    e = launch_ep(ep_peer_combine_kernel, dim3(std::max(rows, 1)), 256, s, c, pa);
    mark(ep, 6, s);
    return cuda_status(e, "ep peer combine launch");
}

// sx_ep_moe over the local layer's rate groups (one group for a uniform bank) of El experts.
sx_status ep_moe_groups(sx_ep* ep, sx_stream stream, const MoeGroup* groups, int ng, int El, int32_t experts_total,
                        const sx_decode* dec, const void* x, sx_dtype dtype, int32_t rows, int32_t rows_cap,
                        const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                        const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                        size_t workspace_bytes, const sx_bank* sh_bank = nullptr, const sx_decode* sh_dec = nullptr) {
    if (rows > 0 && (!x || !inds || !scores || !y)) return SX_ERR_NULL_POINTER;
    if (shared_gate && !shared && !sh_bank) return SX_ERR_NULL_POINTER;
    if (sh_bank && shared) return SX_ERR_BAD_SHAPE;
    if (rows < 0 || rows_cap < 1 || rows > rows_cap || topk < 1) return SX_ERR_BAD_SHAPE;
    if (topk > 32) return SX_ERR_TOPK_EXCEEDS_REDUCE_BANK;
    if (!dtype_ok(dtype)) return SX_ERR_BAD_DTYPE;
    if (clamp_limit < 0 || clamp_limit > 128) return SX_ERR_INVALID_CLAMP;
    if (El < 1 || (long long)El * ep->world != experts_total) return SX_ERR_BAD_SHAPE;
    if (topk > experts_total) return SX_ERR_TOPK_EXCEEDS_EXPERTS;
    const int D = groups[0].bank.gate.in_features;
    if (D % 128) return SX_ERR_BAD_SHAPE;
    if (reinterpret_cast<uintptr_t>(x) % 16) return SX_ERR_BAD_SHAPE;  // rows move as 16-byte vectors
    if (sh_bank) {
        const sx_status st = check_shared_bank(sh_bank, D, sh_dec);
        if (st) return st;
    }
    const int esz = (int)dtype_size(dtype);
    const bool peer = ep->own_bytes > 0;
    const EpWs L = ep_ws_layout(groups, ng, El, ep->world, rows_cap, topk, esz, sh_bank, peer);
    if (!workspace || workspace_bytes < L.total) return SX_ERR_WORKSPACE_TOO_SMALL;
    const PeerLayout PL = peer_layout(ep->world, rows_cap, D, topk, esz);
    if (peer && ep->own_bytes < PL.total) return SX_ERR_PEER_BUFFER_TOO_SMALL;
    if (!peer && !nccl().ok) return nccl_missing();

    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int G = ep->world, C = rows_cap;
    const size_t places = (size_t)G * C;

    // 0. the shared expert over this rank's own rows, on the side stream: it needs only x, so it
    // runs while the rows are exchanged and the experts computed; the combine waits for it.
    // (the peer transport's small calls fold it into the local expert chain instead)
    const bool fold_shared = peer && sh_bank && rows_cap <= kEpFoldRows;
    float* sh_plane = sh_bank && rows > 0 && !fold_shared ? reinterpret_cast<float*>(ws + L.sh_plane) : nullptr;
    // (the NCCL transport forks it first; the peer transport after its dispatch kernel, so the
    // exchange's kernels are not queued behind the shared expert's)
    bool forked = false;
    auto fork_side = [&]() -> sx_status {
        if (!sh_plane) return SX_OK;
        forked = true;
        cudaError_t ce = cudaEventRecord(ep->fork, s);
        if (ce == cudaSuccess) ce = cudaStreamWaitEvent(ep->side, ep->fork, 0);
        if (ce != cudaSuccess) return cuda_status(ce, "expert-parallel fork");
        const sx_status st = shared_expert_run(reinterpret_cast<sx_stream>(ep->side), sh_bank, sh_dec, x, dtype, rows,
                                               clamp_limit, sh_plane, ws + L.sh_scratch);
        ce = cudaEventRecord(ep->join, ep->side);
        return st ? st : (ce != cudaSuccess ? cuda_status(ce, "expert-parallel join") : SX_OK);
    };
    if (!peer) {
        const sx_status st = fork_side();
        if (st) {
            if (forked) cudaStreamWaitEvent(s, ep->join, 0);
            return st;
        }
    }
    // Every return below joins the side stream back into the caller's (the combine reads the plane).
    bool joined = false;
    auto join = [&](sx_status st) {
        if (forked && !joined) {
            const cudaError_t ce = cudaStreamWaitEvent(s, ep->join, 0);
            joined = true;
            if (!st && ce != cudaSuccess) st = cuda_status(ce, "expert-parallel join");
        }
        return st;
    };

    EpArgs a{};
    a.x = x;
    a.inds = inds;
    a.scores = scores;
    a.rows = rows;
    a.cap = C;
    a.K = topk;
    a.D = D;
    a.esz = esz;
    a.world = G;
    a.El = El;
    a.Etot = experts_total;
    a.list = reinterpret_cast<int*>(ws + L.list);
    a.pos = reinterpret_cast<int*>(ws + L.pos);
    a.send_x = ws + L.send_x;
    a.send_inds = reinterpret_cast<uint32_t*>(ws + L.send_inds);
    a.send_scores = reinterpret_cast<float*>(ws + L.send_scores);

    if (peer)
        return join(ep_peer_moe(ep, stream, groups, ng, El, dec, a, PL, L, ws, rows, topk, clamp_limit, sh_plane,
                                shared, shared_gate, y, dtype, join, fold_shared ? sh_bank : nullptr, sh_dec,
                                fork_side));

    // 1-2. plan and gather this rank's send blocks
    mark(ep, 0, s);
    ep_plan_kernel<<<G, 256, 0, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return join(cuda_status(e, "ep plan launch"));
    ep_gather_kernel<<<dim3(C, G), 128, 0, s>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return join(cuda_status(e, "ep gather launch"));

    // 3. dispatch: rows, slot ids and scores in one NCCL group
    sx_status st;
    const A2A dispatch[3] = {{ws + L.send_x, ws + L.recv_x, (size_t)C * D * esz},
                             {ws + L.send_inds, ws + L.recv_inds, (size_t)C * topk * 4},
                             {ws + L.send_scores, ws + L.recv_scores, (size_t)C * topk * 4}};
    mark(ep, 1, s);
    if ((st = all_to_all(ep, dispatch, 3, s))) return join(st);
    mark(ep, 2, s);

    // 4. the local experts over every received row, partials in f32
    float* part_send = reinterpret_cast<float*>(ws + L.part_send);
    st = moe_run(stream, groups, ng, El, dec, ws + L.recv_x, dtype, (int32_t)places,
                 reinterpret_cast<const uint32_t*>(ws + L.recv_inds), reinterpret_cast<const float*>(ws + L.recv_scores),
                 topk, nullptr, nullptr, clamp_limit, nullptr, ws + L.moe, L.moe_bytes, part_send, (long long)C * topk);
    if (st) return join(st);

    // 5. combine: partials back to the rows' owners
    mark(ep, 3, s);
    const A2A combine[1] = {{part_send, ws + L.part_recv, (size_t)C * D * sizeof(float)}};
    if ((st = all_to_all(ep, combine, 1, s))) return join(st);
    mark(ep, 4, s);

    // 6. rank-order sum, rounding, shared expert
    if ((st = join(SX_OK))) return st;
    mark(ep, 5, s);
    if (rows == 0) {
        mark(ep, 6, s);
        return SX_OK;
    }
    CombineArgs c{};
    c.part = reinterpret_cast<const float*>(ws + L.part_recv);
    c.pos = a.pos;
    c.sh_plane = sh_plane;
    c.shared = shared;
    c.shared_gate = shared_gate;
    c.y = y;
    c.rows = rows;
    c.cap = C;
    c.D = D;
    c.world = G;
    c.xdt = dtype;
    ep_combine_kernel<<<rows, 256, 0, s>>>(c);
    const cudaError_t ce = cudaGetLastError();
    mark(ep, 6, s);
    return cuda_status(ce, "ep combine launch");
}

}  // namespace
}  // namespace sx

extern "C" {

sx_status sx_ep_moe(sx_ep* ep, sx_stream stream, const sx_bank* local_bank, int32_t experts_total,
                    const sx_decode* dec, const void* x, sx_dtype dtype, int32_t rows, int32_t rows_cap,
                    const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                    const void* shared_gate, int32_t clamp_limit, void* y, void* workspace, size_t workspace_bytes) {
    if (!ep || !local_bank) return SX_ERR_NULL_POINTER;
    const MoeGroup g{*local_bank, 0};
    return ep_moe_groups(ep, stream, &g, 1, local_bank->gate.experts, experts_total, dec, x, dtype, rows, rows_cap,
                         inds, scores, topk, shared, shared_gate, clamp_limit, y, workspace, workspace_bytes);
}

sx_status sx_ep_moe_ragged(sx_ep* ep, sx_stream stream, const sx_ragged* local, int32_t experts_total,
                           const sx_decode* dec, const void* x, sx_dtype dtype, int32_t rows, int32_t rows_cap,
                           const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                           const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                           size_t workspace_bytes) {
    if (!ep || !local) return SX_ERR_NULL_POINTER;
    MoeGroup g[kMaxGroups];
    int ng = 0;
    const sx_status st = ragged_groups(local, g, &ng);
    if (st) return st;
    return ep_moe_groups(ep, stream, g, ng, local->experts, experts_total, dec, x, dtype, rows, rows_cap, inds, scores,
                         topk, shared, shared_gate, clamp_limit, y, workspace, workspace_bytes);
}

size_t sx_ep_folded_workspace_bytes(const sx_ep* ep, const sx_bank* local_bank, const sx_bank* shared_bank,
                                    int32_t rows_cap, int32_t topk, sx_dtype dtype) {
    if (!ep || !local_bank || !shared_bank || rows_cap < 1 || topk < 1 || !dtype_ok(dtype)) return 0;
    const MoeGroup g{*local_bank, 0};
    return ep_ws_layout(&g, 1, local_bank->gate.experts, ep->world, rows_cap, topk, (int)dtype_size(dtype), shared_bank,
                        ep->own_bytes > 0)
        .total;
}

size_t sx_ep_ragged_folded_workspace_bytes(const sx_ep* ep, const sx_ragged* local, const sx_bank* shared_bank,
                                           int32_t rows_cap, int32_t topk, sx_dtype dtype) {
    if (!ep || !local || !shared_bank || rows_cap < 1 || topk < 1 || !dtype_ok(dtype)) return 0;
    MoeGroup g[kMaxGroups];
    int ng = 0;
    if (ragged_groups(local, g, &ng) != SX_OK) return 0;
    return ep_ws_layout(g, ng, local->experts, ep->world, rows_cap, topk, (int)dtype_size(dtype), shared_bank,
                        ep->own_bytes > 0)
        .total;
}

sx_status sx_ep_moe_folded(sx_ep* ep, sx_stream stream, const sx_bank* local_bank, const sx_bank* shared_bank,
                           int32_t experts_total, const sx_decode* dec, const sx_decode* shared_dec, const void* x,
                           sx_dtype dtype, int32_t rows, int32_t rows_cap, const uint32_t* inds, const float* scores,
                           int32_t topk, const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                           size_t workspace_bytes) {
    if (!ep || !local_bank || !shared_bank) return SX_ERR_NULL_POINTER;
    const MoeGroup g{*local_bank, 0};
    return ep_moe_groups(ep, stream, &g, 1, local_bank->gate.experts, experts_total, dec, x, dtype, rows, rows_cap,
                         inds, scores, topk, nullptr, shared_gate, clamp_limit, y, workspace, workspace_bytes,
                         shared_bank, shared_dec ? shared_dec : dec);
}

sx_status sx_ep_moe_ragged_folded(sx_ep* ep, sx_stream stream, const sx_ragged* local, const sx_bank* shared_bank,
                                  int32_t experts_total, const sx_decode* dec, const sx_decode* shared_dec,
                                  const void* x, sx_dtype dtype, int32_t rows, int32_t rows_cap, const uint32_t* inds,
                                  const float* scores, int32_t topk, const void* shared_gate, int32_t clamp_limit,
                                  void* y, void* workspace, size_t workspace_bytes) {
    if (!ep || !local || !shared_bank) return SX_ERR_NULL_POINTER;
    MoeGroup g[kMaxGroups];
    int ng = 0;
    const sx_status st = ragged_groups(local, g, &ng);
    if (st) return st;
    return ep_moe_groups(ep, stream, g, ng, local->experts, experts_total, dec, x, dtype, rows, rows_cap, inds, scores,
                         topk, nullptr, shared_gate, clamp_limit, y, workspace, workspace_bytes, shared_bank,
                         shared_dec ? shared_dec : dec);
}

}  // extern "C"
