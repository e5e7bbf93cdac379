// Internal helpers shared by the entry-point files of libsushi_exl3_cuda.so.
#pragma once

#include "../../include/sushi_exl3.h"
#include "sx_decode.cuh"

namespace sx {

sx_status cuda_status(cudaError_t e, const char* where = "cuda");
void note_cuda_error(cudaError_t e, const char* where);
void note_detail(const char* what, const char* why);  // the text sx_last_error_detail returns
sx_status resolve_decode(const sx_decode* dec, int n, int* kind, DecParams* dp);
sx_status check_proj(const sx_proj* p, int need_experts);
bool dtype_ok(int dt);
int sm_count();

struct GemmArgs;
// The tensor-core projection (sx_gemm.cu): the TMA map of a [rows, in] f16 matrix of prepared
// rows, the split-K choice, and the launch over codebook families and rates.
// box_rows: the rows of one tile (the launch's NT: 128, or 16 for a dense call of at most 16 rows).
cudaError_t prep_map(CUtensorMap* m, const uint16_t* P, int rows, int in, int box_rows);
int gemm_split(long long ctas, int chunks);
int gemm_rt(long long rows, int n);
bool gemm_rt_rate(int n);  // rates with four-row-tile tensor-core kernels
// pair: the CTA-pair (cta_group::2) kernel for rt == 4 (no split, an even count of output blocks).
// nt: rows per tile, 128, or 16 (one row tile, no pair: the MMA's N and the prepared-row tile are
// the 16 live rows).
cudaError_t gemm_launch(int kind, const CUtensorMap& pmap, const GemmArgs& a, int n, int rt, int items, int S,
                        cudaStream_t stream, bool pair = false, int nt = 128);

// sx_moe's body; with `partial` set, the routed k-order sums land there in f32, unrounded and
// without the shared expert (an expert-parallel rank's share of its peers' tokens), and y is unused.
// `slots` bounds the routed slots that can be valid (0: rows * topk); it picks the decode chain or
// the tensor-core path, and moe_workspace_bytes must be asked with the same value.
sx_status moe_impl(sx_stream stream, const sx_bank* bank, const sx_decode* dec, const void* x, sx_dtype dtype,
                   int32_t rows, const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                   const void* shared_gate, int32_t clamp_limit, void* y, void* workspace, size_t workspace_bytes,
                   float* partial, long long slots);
size_t moe_workspace_bytes(const sx_bank* bank, int32_t rows, int32_t topk, long long slots);

// One rate group of a routed layer: its experts are ids [e_lo, e_lo + bank.experts) of the layer.
struct MoeGroup {
    sx_bank bank;
    int e_lo;
};
constexpr int kMaxGroups = 32;  // layout.max_groups (src/exl3/layout.zig:4)

// An expert-parallel rank's received rows: `n` segments of `cap` places, segment g live in its
// first cnt[g] places (device counts, read by route_prep after its dependency wait).  moe_groups_ws
// must be asked for the worst case (every place live) whichever live_slots a call passes.
struct MoeSegments {
    const int* cnt;
    int cap, n;
    long long live_slots;  // the segments' routed slots when the host knows them (sizes the launches), else -1
    // route_prep first waits (bounded) for wait_flags[g] >= *seq for every segment g, when set:
    // the rows and counts arrive from other GPUs behind those flags
    const uint32_t* wait_flags;
    const uint32_t* seq;
};

// The rows a layer's shared expert runs over when they are not the routed rows (an expert-parallel
// rank routes the rows it received, and runs its shared expert over its own).
struct SharedRows {
    const void* x;
    int rows;
};

// moe_impl over the rate groups of a layer of Etot experts (sx_moe_ragged's body).  seg: only
// the segments' live places are routed.  yslot_out: no reduce is launched; the per-slot planes
// (slot s at [s][D] f32, score included, written for the routed slots only) are left for the
// caller at *yslot_out, the start of the workspace, followed by the shared expert's plane (rows
// sh_bank runs over, at slot rows*topk + row).  own: the shared expert's rows, if not x's.
sx_status moe_run(sx_stream stream, const MoeGroup* groups, int ng, int Etot, const sx_decode* dec, const void* x,
                  sx_dtype dtype, int32_t rows, const uint32_t* inds, const float* scores, int32_t topk,
                  const void* shared, const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                  size_t workspace_bytes, float* partial, long long slots, const sx_bank* sh_bank = nullptr,
                  const sx_decode* sh_dec = nullptr, const MoeSegments* seg = nullptr, float** yslot_out = nullptr,
                  const SharedRows* own = nullptr);
size_t moe_groups_ws(const MoeGroup* g, int ng, int Etot, int rows, int topk, long long slots);
// With a shared expert over sh_rows rows (its plane follows the routed slots' planes).
size_t moe_groups_ws(const MoeGroup* g, int ng, int Etot, int rows, int topk, long long slots, const sx_bank* sh,
                     const sx_decode* dec, const sx_decode* sh_dec, int sh_rows);
// A layer's shared expert (one SwiGLU expert over hidden size D): its admission, and its output
// over `rows` rows alone into plane [rows][D] f32 with shared_expert_ws(sh, rows) bytes of scratch.
sx_status check_shared_bank(const sx_bank* sh, int D, const sx_decode* dec);
size_t shared_expert_ws(const sx_bank* sh, int rows);
sx_status shared_expert_run(sx_stream stream, const sx_bank* sh, const sx_decode* dec, const void* x, sx_dtype dtype,
                            int32_t rows, int32_t clamp_limit, float* plane, uint8_t* scratch);
// The groups of a ragged layer (at most kMaxGroups) from its host meta table.
sx_status ragged_groups(const sx_ragged* rb, MoeGroup* out, int* ng);

}  // namespace sx
