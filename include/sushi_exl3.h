/*
 * sushi_exl3.h: C ABI of libsushi_exl3_cuda.so, the B200 (sm_100a) EXL3 / STQ trellis kernels.
 *
 * This is the drop-in boundary for the reference's `sushi_exl3` Zig module
 * (beamivalice/sushi 1.7.2, src/exl3/root.zig), whose host code reaches Metal through MLX.
 * A Zig host declares these functions `extern fn` and calls them where root.zig / linear.zig /
 * moe_router.zig dispatch Metal kernels today.  Every pointer is a device pointer borrowed from
 * the caller; outputs go to caller-allocated buffers; no call allocates device memory.  Scratch,
 * where a call needs any, is a caller-owned workspace sized by the matching *_workspace_bytes()
 * query.  Calls are stream-ordered on the stream given and stateless: the decode parameters
 * travel with each call (the reference sets a process global before each dispatch instead,
 * src/exl3/expert_exl3_kernels.zig:938).  No call aborts, traps or prints; each returns a status.
 *
 * Pack layout (docs/pack-format.md "Routed-expert tensors"): a projection's trellis is U16
 * [E, in/16, out/16, n] in pack order, or [E, out/32, in/16, 2, n] pair-major
 * (src/exl3/layout.zig:141); suh is F16 [E, in], svh is F16 [E, out]; n is the packed halfwords
 * per 16x16 tile (even, 16..128; K = n/16 bits per weight).  The weight a bank applies is
 * W = diag(suh) H128 inner H128 diag(svh), y = x . W (src/exl3/expert_exl3.zig:440-566).
 */
#ifndef SUSHI_EXL3_H
#define SUSHI_EXL3_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  Each non-zero code mirrors one of the reference's named refusals. */
typedef int32_t sx_status;
enum {
    SX_OK = 0,
    SX_ERR_BAD_SHAPE = 1,                  /* error.BadExl3Shape (src/exl3/root.zig:104-130) */
    SX_ERR_BAD_DTYPE = 2,                  /* error.BadExl3Dtype (src/exl3/root.zig:110-113) */
    SX_ERR_INVALID_CLAMP = 3,              /* error.InvalidExl3Clamp (src/exl3/root.zig:103) */
    SX_ERR_TOPK_EXCEEDS_REDUCE_BANK = 4,   /* error.Exl3TopKExceedsReduceBank (src/exl3/root.zig:421) */
    SX_ERR_CODEBOOK_TABLE_UNKNOWN = 5,     /* error.Exl3CodebookTableUnknown (src/exl3/expert_exl3.zig:162) */
    SX_ERR_TRELLIS_GEOMETRY = 6,           /* error.Exl3TrellisGeometry (src/exl3/layout.zig:57-63) */
    SX_ERR_CODEBOOK_TABLE_RATE_MISSING = 7,/* error.Exl3CodebookTableRateMissing (src/exl3/layout.zig:92) */
    SX_ERR_WINDOW_UNSUPPORTED = 8,         /* error.Exl3WindowUnsupported (src/exl3/root.zig:223) */
    SX_ERR_CODEBOOK_UNSUPPORTED = 9,       /* error.ExpertLayoutUnsupported for an unknown codebook */
    SX_ERR_CODEBOOK_TABLE_WINDOW_MISMATCH = 10, /* error.Exl3CodebookTableWindowMismatch (codebook_tables.zig:276) */
    SX_ERR_TOPK_EXCEEDS_EXPERTS = 11,      /* error.Exl3TopKExceedsExperts (src/exl3/layout.zig:117) */
    SX_ERR_ROUTER_DECLINED = 12,           /* moeRouterTopK returned null (src/moe_router.zig:466-490) */
    SX_ERR_NULL_POINTER = 13,
    SX_ERR_WORKSPACE_TOO_SMALL = 14,
    SX_ERR_CUDA = 15,                      /* a CUDA runtime call failed (launch, attribute) */
    SX_ERR_DEVICE_TIMEOUT = 16,            /* a bounded device-side wait gave up (see sx_device_error) */
    SX_ERR_NCCL = 17,                      /* an NCCL call failed (expert-parallel calls) */
    SX_ERR_TILE_ORDER_UNSUPPORTED = 18,    /* error.Exl3TileOrderUnsupported (docs/pack-format.md) */
    SX_ERR_GROUP_GEOMETRY = 19,            /* error.Exl3GroupGeometry (src/exl3/layout.zig:80-95) */
    SX_ERR_STATIC_SCRATCH_TOO_SMALL = 20,  /* the call needs more scratch than sx_moe_static_scratch holds */
    SX_ERR_PEER_BUFFER_TOO_SMALL = 21,     /* the expert-parallel call needs more peer buffer than is reserved */
    SX_ERR_PEER_ACCESS = 22                /* a peer's buffer could not be mapped (sx_ep_reserve_peer) */
};

/* The status's name ("SX_OK", "SX_ERR_BAD_SHAPE", ...); a static string. */
const char* sx_status_name(sx_status s);

/* Element types of activations and outputs. */
typedef enum { SX_DT_F32 = 0, SX_DT_F16 = 1, SX_DT_BF16 = 2 } sx_dtype;

/* Codebooks, numbered as the reference's `Codebook` enum (src/exl3/expert_exl3.zig:54-61). */
typedef enum { SX_CB_MUL1 = 0, SX_CB_MCG = 1, SX_CB_SPEC1 = 2, SX_CB_PAIR1 = 3, SX_CB_STD1 = 4 } sx_codebook;

/* Codebook tables, numbered as the reference's `tables` (src/exl3/codebook_tables.zig:101-106,
 * 216-220): 0 pair1-w16-v1, 1 spec1-w15, 2 spec1-w16, 3 std1, 4 spec1-test-per-rate (the
 * reference's test-only table whose row differs at every rate).  -1 names no table. */
enum { SX_TABLE_NONE = -1, SX_TABLE_PAIR1_W16_V1 = 0, SX_TABLE_SPEC1_W15 = 1, SX_TABLE_SPEC1_W16 = 2,
       SX_TABLE_STD1 = 3, SX_TABLE_SPEC1_TEST = 4 };

/* How a pack's trellis decodes: format.Decode (src/exl3/expert_exl3.zig:141-174).
 * window_bits is the codeword width the search hashed, 8..16 (16 masks nothing). */
typedef struct sx_decode {
    int32_t codebook;     /* sx_codebook */
    int32_t window_bits;  /* 8..16 */
    int32_t table;        /* SX_TABLE_*; required for SPEC1 and STD1 */
} sx_decode;

/* Tile orders (src/exl3/expert_exl3.zig:249-257). */
typedef enum { SX_TILE_PACK = 0, SX_TILE_PAIR_MAJOR = 1 } sx_tile_order;

/* One projection's bank: root.Proj (src/exl3/root.zig:30). */
typedef struct sx_proj {
    const uint16_t* trellis;  /* U16, see tile_order */
    const uint16_t* suh;      /* F16 bits [experts, in_features] */
    const uint16_t* svh;      /* F16 bits [experts, out_features] */
    int32_t experts;
    int32_t in_features;      /* multiple of 128 */
    int32_t out_features;     /* multiple of 128 */
    int32_t n;                /* packed halfwords per tile: even, 16..128 */
    int32_t tile_order;       /* sx_tile_order */
} sx_proj;

/* A routed MoE layer's three banks: root.Bank (src/exl3/root.zig:39). */
typedef struct sx_bank {
    sx_proj gate, up, down;
} sx_bank;

/* Opaque CUDA stream (cudaStream_t / CUstream). */
typedef void* sx_stream;

/* ------------------------------------------------------------------ decode
 * The dequantised inner matrix of expert `expert`: `out` [in, out] F16 bits, row-major, bit-exact
 * with the reference's host decode `reconstructInner` (src/exl3/expert_exl3.zig:416-438). */
sx_status sx_dequant_inner(sx_stream stream, const sx_proj* proj, int32_t expert, const sx_decode* dec,
                           uint16_t* out);

/* Every codeword's decoded weight (or PAIR1 weight pair) at rate n: out[cw] for cw in 0..65535,
 * F16 bits; PAIR1 writes weight 2j in the low half and 2j+1 in the high half of out32[cw].  The
 * device codebook against the host truth over all codewords, as firstPair1PairMismatch does
 * (src/exl3/expert_exl3.zig:361-369). */
sx_status sx_decode_codewords(sx_stream stream, int32_t n, const sx_decode* dec, uint32_t* out32);

/* Converts trellis tiles between the pack order [E, IT, OT, n] and the pair-major order
 * [E, OT/2, IT, 2, n] (layout.tileMajor / tileMajorInverse, src/exl3/layout.zig:141-160;
 * `trellis_pm` tensors, docs/pack-format.md "tile order").  The projection kernels read the pack
 * order; a host that loads pair-major packs converts each routed trellis once after loading.
 * src and dst are device buffers of experts*in/16*out/16*n halfwords that must not overlap
 * (SX_ERR_BAD_SHAPE) unless the orders are equal. */
sx_status sx_tile_order_convert(sx_stream stream, const uint16_t* src, uint16_t* dst, int32_t experts,
                                int32_t in_features, int32_t out_features, int32_t n, int32_t from_order,
                                int32_t to_order);

/* ------------------------------------------------------------------ dense linears
 * y = x . W for `rows` rows through the one-bank projection `proj` (experts == 1):
 * linear.linear (src/exl3/linear.zig:27-35), trunk.matmul (src/exl3/trunk.zig:53).
 * x [rows, in] and y [rows, out], row-major, both of `dtype` (BF16, F16 or F32; the output is in
 * the input's dtype as the reference's).  The prepared input is rounded to f16 as the reference's
 * prepareInput does; products accumulate in f32; y is rounded once.  rows >= 1. */
sx_status sx_linear(sx_stream stream, const sx_proj* proj, const sx_decode* dec, const void* x, sx_dtype dtype,
                    int32_t rows, void* y);

/* Flags of sx_linear_ex. */
enum {
    /* The projection's trellis, suh and svh are not written by the work queued on `stream` just
     * before this call.  The launch then uses programmatic dependent launch: its CTAs start
     * streaming weights while the previous kernel on the stream finishes, and wait for it only
     * before reading x and writing y.  Decode loops whose weights are loaded once set it. */
    SX_LINEAR_WEIGHTS_STATIC = 1u
};

/* sx_linear with launch flags (SX_LINEAR_*); flags == 0 is sx_linear.  No reference counterpart:
 * the reference's Metal dispatch has no launch overlap to ask for.  Unknown flag bits:
 * SX_ERR_BAD_SHAPE. */
sx_status sx_linear_ex(sx_stream stream, const sx_proj* proj, const sx_decode* dec, const void* x, sx_dtype dtype,
                       int32_t rows, void* y, uint32_t flags);

/* The many-row projection on the tensor cores: the reference's sorted-window GEMM for rows past
 * the decode chain (src/exl3/linear.zig:365; kernels.moePrefill's inner GEMM,
 * src/exl3/expert_exl3_kernels.zig:1379-1408).  Same arguments and result bar as sx_linear, plus
 * a workspace of sx_linear_gemm_workspace_bytes(proj, rows) bytes (16-byte aligned) for the
 * prepared rows.  The weights are decoded to the reference's f16 inner weights in shared memory
 * and multiplied by tcgen05 MMAs with f32 accumulation. */
size_t sx_linear_gemm_workspace_bytes(const sx_proj* proj, int32_t rows);
sx_status sx_linear_gemm(sx_stream stream, const sx_proj* proj, const sx_decode* dec, const void* x, sx_dtype dtype,
                         int32_t rows, void* y, void* workspace, size_t workspace_bytes);

/* linear.linearShared (src/exl3/linear.zig:144-247): up to 4 linears that read the same rows,
 * stacked along the output into one bank (trellis [1, in/16, out/16, n], svh [1, out]) with one suh
 * row per linear (suh [count, in]); linear s owns columns cols[s]..cols[s+1] (host array of
 * count+1 bounds, multiples of 128, cols[0] = 0, cols[count] = out).  One launch (per 16 rows)
 * writes ys[s] [rows, cols[s+1]-cols[s]] in x's dtype. */
sx_status sx_linear_shared(sx_stream stream, const sx_proj* proj, const int32_t* cols, int32_t count,
                           const sx_decode* dec, const void* x, sx_dtype dtype, int32_t rows, void* const* ys);

/* linear.linearSharedNormed (src/exl3/linear.zig:269-290; project_rows.zig:394-456, 908-919): as
 * sx_linear_shared, with linear 0's rows leaving RMS-normed in the same launch:
 *   ys[0][r][c] = T( w[c] * T( o[r][c] * rsqrt(sum_c' o[r][c']^2 / cols[1] + eps) ) )
 * where o is linear 0's finished output in x's dtype T and w = norm_w [cols[1]] in that dtype (MLX's
 * fast rms_norm on the finished row).  rows 1..16, out <= 4096, eps >= 0 (else SX_ERR_BAD_SHAPE).
 * workspace: sx_linear_shared_normed_workspace_bytes(proj) bytes, 16-byte aligned, ZEROED before
 * its first use; every call leaves it zeroed again.  Calls that may run at the same time (other
 * streams) need their own workspace. */
size_t sx_linear_shared_normed_workspace_bytes(const sx_proj* proj);
sx_status sx_linear_shared_normed(sx_stream stream, const sx_proj* proj, const int32_t* cols, int32_t count,
                                  const sx_decode* dec, const void* x, sx_dtype dtype, int32_t rows, void* const* ys,
                                  const void* norm_w, float eps, void* workspace, size_t workspace_bytes);

/* linear.linearGrouped (src/exl3/linear.zig:38-54): x [G, rows, in] through the G-bank proj
 * (experts == G, bank g serves x[g]) into y [G, rows, out]. */
sx_status sx_linear_grouped(sx_stream stream, const sx_proj* proj, const sx_decode* dec, const void* x,
                            sx_dtype dtype, int32_t rows, void* y);

/* ------------------------------------------------------------------ router
 * Router modes (src/moe_router.zig:105). */
typedef enum { SX_ROUTER_SOFTMAX = 0, SX_ROUTER_SIGMOID_BIAS = 1, SX_ROUTER_SIGMOID_BIAS_GROUPED = 2 } sx_router_mode;

/* moeRouterTopK (src/moe_router.zig:442): per row of logits [rows, experts] (F32), the top-k
 * experts by key (softmax: the logit; sigmoid modes: sigmoid(logit) + bias[e], with the group
 * limit for the grouped mode), ties to the lowest id, and their weights (softmax probabilities
 * renormalised over the picks; sigmoid modes: sigmoid scores, renormalised when `renorm` and k > 1,
 * times `scale`).  inds [rows, k] U32, scores [rows, k] F32.  Returns SX_ERR_ROUTER_DECLINED where
 * the reference's kernel declines (k outside 1..32, more than 2048 experts, a group limit it
 * cannot take), so the caller keeps its own chain. */
sx_status sx_router_topk(sx_stream stream, const float* logits, const float* bias, int32_t rows, int32_t experts,
                         int32_t k, int32_t mode, int32_t renorm, float scale, int32_t n_group, int32_t topk_group,
                         uint32_t* inds, float* scores);

/* moeRouterTopKGate (src/moe_router.zig:457): sx_router_topk over logits of any activation dtype
 * (`logits_dtype` F32, F16 or BF16, as the reference admits, :478), and, in the softmax mode, the
 * reference's softmax_gate: the shared-expert gate's logit x . w computed in the same launch
 * (gate_x [gate_k] and gate_w [gate_k] of `gate_dtype`, F16 or BF16; gate_logit [1] written in
 * `gate_dtype`, the `shared_gate` operand of sx_moe / sx_moe_folded).  The dot is summed in the
 * order of MLX's dot_product that the reference kernel restates (:200-218, :328-332), products
 * and sums rounded separately.  Pass null gate pointers for no gate; in the sigmoid modes they
 * are ignored (:471).  Declines (SX_ERR_ROUTER_DECLINED) where the reference does: more than one
 * row with a gate, gate_k outside 1..16384 or not a multiple of 8, a gate dtype other than F16 and
 * BF16 (:499-506), and everything sx_router_topk declines. */
sx_status sx_router_topk_gate(sx_stream stream, const void* logits, sx_dtype logits_dtype, const float* bias,
                              int32_t rows, int32_t experts, int32_t k, int32_t mode, int32_t renorm, float scale,
                              int32_t n_group, int32_t topk_group, const void* gate_x, const void* gate_w,
                              int32_t gate_k, sx_dtype gate_dtype, void* gate_logit, uint32_t* inds, float* scores);

/* ------------------------------------------------------------------ routed experts
 * The workspace sx_moe needs for `rows` rows at top-k `topk` over `bank` (bytes). */
size_t sx_moe_workspace_bytes(const sx_bank* bank, int32_t rows, int32_t topk);

/* Routed SwiGLU experts: root.moe / moeWithShared / moeWithGatedShared / moeClamped
 * (src/exl3/root.zig:51-125).  x [rows, hidden] (BF16, F16 or F32), inds [rows, topk] U32 expert
 * ids, scores [rows, topk] F32 weights; y [rows, hidden] in x's dtype:
 *   y[r] = sum_k scores[r,k] * down_e(silu(gate_e(x[r])) * up_e(x[r]))      e = inds[r,k]
 * with the gate upper-clamped and up clipped to +-clamp_limit first when clamp_limit > 0 (the
 * clamped SwiGLU, src/exl3/root.zig:96-125; 1..128, else SX_ERR_INVALID_CLAMP).  When `shared`
 * ([rows, hidden], x's dtype) is given it is added to every row; with `shared_gate` ([rows] x's
 * dtype logits) it is added as sigmoid(gate) * shared (moeWithGatedShared).  topk <= 32.
 * `workspace` holds at least sx_moe_workspace_bytes(bank, rows, topk).  Layers the tensor-core path
 * serves (more than 16 rows averaging 16 or more per routed expert) need x and the workspace
 * 16-byte aligned and the gate/up suh 8-byte aligned (else SX_ERR_BAD_SHAPE). */
sx_status sx_moe(sx_stream stream, const sx_bank* bank, const sx_decode* dec, const void* x, sx_dtype dtype,
                 int32_t rows, const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                 const void* shared_gate, int32_t clamp_limit, void* y, void* workspace, size_t workspace_bytes);

/* ------------------------------------------------------------------ rate-grouped routed experts
 * A layer whose experts come in rate groups (`.gN` groups, each with its own gate/up/down rates)
 * held as one ragged bank per projection: rate_groups.Ragged (src/exl3/rate_groups.zig:23-130).
 * trellis[p] is projection p's flat U16 storage (gate, up, down), groups back to back and each
 * expert's tiles contiguous; suh[p] / svh[p] hold one F16 row per expert over all groups; meta is
 * the reference's table of 8 u32 words per expert (rate_groups.zig:23-25): gate n, up n, down n,
 * group, the gate/up/down offsets of the expert's tiles in trellis[p] counted in u32 words, and the
 * expert's index in its group.  meta is HOST memory (the library reads the groups from it at each
 * call); every other pointer is device memory.  Each group must be a run of consecutive expert ids
 * with one rate per projection and tiles at a fixed stride (else SX_ERR_GROUP_GEOMETRY); groups
 * whose gate and up rates differ are refused with SX_ERR_TRELLIS_GEOMETRY. */
typedef struct sx_ragged {
    const uint16_t* trellis[3];
    const uint16_t* suh[3];
    const uint16_t* svh[3];
    const uint32_t* meta;     /* host [experts][8] */
    int32_t experts;
    int32_t hidden;           /* the gate/up input and down output width, multiple of 128 */
    int32_t inter;            /* the gate/up output and down input width, multiple of 128 */
} sx_ragged;

/* The workspace sx_moe_ragged needs (bytes); 0 for a malformed meta table. */
size_t sx_moe_ragged_workspace_bytes(const sx_ragged* bank, int32_t rows, int32_t topk);

/* root.moeRagged (src/exl3/root.zig:582; rate_groups.moeDecode :1659 / moePrefill :2042): sx_moe
 * over a rate-grouped layer.  inds are the layer's expert ids; every slot decodes at its expert's
 * group rates; y as sx_moe (k-order sum, rounding, optional shared / gated shared, clamp). */
sx_status sx_moe_ragged(sx_stream stream, const sx_ragged* bank, const sx_decode* dec, const void* x, sx_dtype dtype,
                        int32_t rows, const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                        const void* shared_gate, int32_t clamp_limit, void* y, void* workspace, size_t workspace_bytes);

/* The routed layer with its shared expert folded in (moe_shared_fold.folded, src/moe_shared_fold.zig:24;
 * fold_gated.moeGatedSharedFolded, src/exl3/fold_gated.zig:122-160; rate_groups'
 * moeGatedSharedFolded): y as sx_moe / sx_moe_ragged with `shared` = the shared expert's output
 * over the same rows, rounded to x's dtype (a one-expert SwiGLU bank, `shared_bank`, experts = 1,
 * decoded with `shared_dec`, or `dec` when null; the same clamp_limit), optionally sigmoid-gated by
 * shared_gate [rows].  The shared expert rides the routed decode chain's launches when its rates,
 * decode and intermediate size match a routed group's; otherwise it runs as its own launches.
 * Each output matches the unfused composition (the same arithmetic per row); where the two take
 * different k splits for the shared expert's products the f32 sums may differ in their last bit
 * before rounding.  workspace: the matching
 * *_folded_workspace_bytes(...). */
size_t sx_moe_folded_workspace_bytes(const sx_bank* bank, const sx_bank* shared_bank, const sx_decode* dec,
                                     const sx_decode* shared_dec, int32_t rows, int32_t topk);
sx_status sx_moe_folded(sx_stream stream, const sx_bank* bank, const sx_bank* shared_bank, const sx_decode* dec,
                        const sx_decode* shared_dec, const void* x, sx_dtype dtype, int32_t rows, const uint32_t* inds,
                        const float* scores, int32_t topk, const void* shared_gate, int32_t clamp_limit, void* y,
                        void* workspace, size_t workspace_bytes);
size_t sx_moe_ragged_folded_workspace_bytes(const sx_ragged* bank, const sx_bank* shared_bank, const sx_decode* dec,
                                            const sx_decode* shared_dec, int32_t rows, int32_t topk);
sx_status sx_moe_ragged_folded(sx_stream stream, const sx_ragged* bank, const sx_bank* shared_bank,
                               const sx_decode* dec, const sx_decode* shared_dec, const void* x, sx_dtype dtype,
                               int32_t rows, const uint32_t* inds, const float* scores, int32_t topk,
                               const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                               size_t workspace_bytes);

/* ------------------------------------------------------------------ routed experts, no allocation
 * sx_moe for callers that cannot allocate device memory at all.  Some hosts never call cudaMalloc
 * on the path that runs the layer: a caller whose allocator owns and bills every device byte
 * (memory admission that a hidden allocation would bypass, an arena sized once at start-up), or a
 * latency-critical loop that cannot afford the device-wide synchronisation cudaMalloc implies.
 * They cannot hand sx_moe a workspace either, so this entry point takes none: its scratch is a
 * fixed buffer compiled into the library (sx_moe_static_scratch_bytes(), 8 MiB), held by every GPU
 * that loads the library until the process exits.  No counterpart in the reference, whose MLX host
 * allocates per call.
 *
 * Arguments, semantics and refusals are sx_moe's: a malformed call gets sx_moe's own refusal.  A
 * well-formed call whose workspace (sx_moe_workspace_bytes(bank, rows, topk)) exceeds the buffer
 * returns SX_ERR_STATIC_SCRATCH_TOO_SMALL before launching anything.  The first call on a device
 * (per CUDA context) looks up the buffer's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture.  A cudaDeviceReset while the library
 * is loaded leaves that looked-up address stale: not supported.  Every call on a device shares
 * the one buffer and the buffer keeps the last call's contents (nothing in it needs to start at
 * zero): calls that overlap on the GPU race, so issue them on one stream or order them. */
sx_status sx_moe_static_scratch(sx_stream stream, const sx_bank* bank, const sx_decode* dec, const void* x,
                                sx_dtype dtype, int32_t rows, const uint32_t* inds, const float* scores, int32_t topk,
                                const void* shared, const void* shared_gate, int32_t clamp_limit, void* y);

/* The size of sx_moe_static_scratch's buffer in bytes. */
size_t sx_moe_static_scratch_bytes(void);

/* ------------------------------------------------------------------ expert parallel
 * The routed layer with its experts sharded over `world` GPUs (one process or thread per GPU):
 * rank g holds experts [g*E/world, (g+1)*E/world) of an E-expert layer as a local bank of E/world
 * experts.  Each rank routes its own tokens; a token's hidden row travels once to every rank that
 * owns one of its experts, together with its slots there (dispatch), the ranks run their local
 * expert chains, and each token's partial sums come back to its owner (combine), which adds them
 * in rank order, rounds to the output dtype and adds the shared expert.  Dispatch and combine are
 * NCCL all-to-alls (grouped ncclSend/ncclRecv) of fixed-size blocks: `rows_cap` rows per peer,
 * so no host synchronisation sits between the steps.  No reference counterpart: the reference
 * serves its experts from one GPU.  The library loads NCCL (libnccl.so.2) when an sx_ep call
 * first needs it. */
typedef struct sx_ep sx_ep;

/* A new NCCL unique id (128 bytes) for sx_ep_init: made on one rank and handed to every rank by
 * the host's own means. */
sx_status sx_ep_unique_id(uint8_t id[128]);

/* Joins the `world`-rank communicator named by `id` as `rank`, on the current CUDA device.
 * Collective: every rank calls it. */
sx_status sx_ep_init(const uint8_t id[128], int32_t world, int32_t rank, sx_ep** out);

/* Frees the communicator (ncclCommDestroy).  Synchronise the streams that used it first. */
sx_status sx_ep_destroy(sx_ep* ep);

/* Aborts the communicator (ncclCommAbort) and frees it: a host watchdog's way out of a collective
 * that a failed peer will never complete. */
sx_status sx_ep_abort(sx_ep* ep);

/* Workspace of sx_ep_moe in bytes, for a local bank `local_bank` at `rows_cap` rows per rank. */
size_t sx_ep_workspace_bytes(const sx_ep* ep, const sx_bank* local_bank, int32_t rows_cap, int32_t topk,
                             sx_dtype dtype);

/* The expert-parallel routed layer.  Collective over the communicator: every rank calls it with
 * the same rows_cap, topk, experts_total and dtype, in the same order as its other sx_ep calls.
 * local_bank: this rank's experts_total/world experts (gate, up, down as in sx_moe).  x [rows,
 * hidden] (16-byte aligned), inds [rows, topk] U32 GLOBAL expert ids (ids >= experts_total are
 * skipped), scores [rows, topk] F32, shared / shared_gate / clamp_limit as sx_moe; 0 <= rows <=
 * rows_cap (ranks may hold different row counts).  y [rows, hidden] in x's dtype:
 *   y[r] = round( sum over ranks d in order of P_d[r] ) (+ shared), P_d[r] = the k-order f32 sum
 * of score * expert output over r's slots whose expert rank d owns.  experts_total must be
 * world * local_bank experts.  `workspace` holds sx_ep_workspace_bytes(...) bytes. */
sx_status sx_ep_moe(sx_ep* ep, sx_stream stream, const sx_bank* local_bank, int32_t experts_total,
                    const sx_decode* dec, const void* x, sx_dtype dtype, int32_t rows, int32_t rows_cap,
                    const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                    const void* shared_gate, int32_t clamp_limit, void* y, void* workspace, size_t workspace_bytes);

/* sx_ep_moe over a rate-grouped local layer (rate_groups.Ragged, src/exl3/rate_groups.zig:23-130;
 * root.moeRagged, src/exl3/root.zig:582): `local` holds this rank's experts_total/world experts
 * (local->experts), in rate groups as sx_moe_ragged takes them; everything else as sx_ep_moe.
 * Ranks may hold different rates (a rank's experts are a contiguous id range of the layer). */
size_t sx_ep_ragged_workspace_bytes(const sx_ep* ep, const sx_ragged* local, int32_t rows_cap, int32_t topk,
                                    sx_dtype dtype);
sx_status sx_ep_moe_ragged(sx_ep* ep, sx_stream stream, const sx_ragged* local, int32_t experts_total,
                           const sx_decode* dec, const void* x, sx_dtype dtype, int32_t rows, int32_t rows_cap,
                           const uint32_t* inds, const float* scores, int32_t topk, const void* shared,
                           const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                           size_t workspace_bytes);

/* sx_ep_moe / sx_ep_moe_ragged with the layer's shared expert folded in (moe_shared_fold.folded,
 * src/moe_shared_fold.zig:24): each rank runs the shared expert (a one-expert `shared_bank`,
 * replicated on every rank; `shared_dec` or `dec`) over its own rows on the communicator's side
 * stream, concurrently with the dispatch, the local experts and the combine exchange, and the
 * combine adds it (rounded, optionally sigmoid-gated by shared_gate [rows]) as sx_moe_folded does.
 * The caller's stream waits for the side stream before the call returns its work. */
size_t sx_ep_folded_workspace_bytes(const sx_ep* ep, const sx_bank* local_bank, const sx_bank* shared_bank,
                                    int32_t rows_cap, int32_t topk, sx_dtype dtype);
sx_status sx_ep_moe_folded(sx_ep* ep, sx_stream stream, const sx_bank* local_bank, const sx_bank* shared_bank,
                           int32_t experts_total, const sx_decode* dec, const sx_decode* shared_dec, const void* x,
                           sx_dtype dtype, int32_t rows, int32_t rows_cap, const uint32_t* inds, const float* scores,
                           int32_t topk, const void* shared_gate, int32_t clamp_limit, void* y, void* workspace,
                           size_t workspace_bytes);
size_t sx_ep_ragged_folded_workspace_bytes(const sx_ep* ep, const sx_ragged* local, const sx_bank* shared_bank,
                                           int32_t rows_cap, int32_t topk, sx_dtype dtype);
sx_status sx_ep_moe_ragged_folded(sx_ep* ep, sx_stream stream, const sx_ragged* local, const sx_bank* shared_bank,
                                  int32_t experts_total, const sx_decode* dec, const sx_decode* shared_dec,
                                  const void* x, sx_dtype dtype, int32_t rows, int32_t rows_cap, const uint32_t* inds,
                                  const float* scores, int32_t topk, const void* shared_gate, int32_t clamp_limit,
                                  void* y, void* workspace, size_t workspace_bytes);

/* ------------------------------------------------------------------ expert parallel over NVLink
 * With a peer buffer reserved (sx_ep_reserve_peer), every sx_ep_moe* call of the communicator
 * moves its rows over NVLink peer memory instead of NCCL: each rank's buffer is mapped into every
 * other rank's address space (CUDA IPC), the dispatch kernel stores each routed row and its slots
 * straight into the owning rank's buffer and raises a flag there, the owner's expert chain runs
 * over the rows it received (only those), its reduce kernel stores each row's f32 partial straight
 * into the token owner's buffer and raises a flag, and the owner's combine waits for the flags and
 * adds the partials in rank order.  Only routed rows cross NVLink (no fixed-size blocks).  Calls
 * with rows_cap < 1024 (decode sizes) never wait on the host and can be recorded in a CUDA graph
 * after the reservation.  Calls with rows_cap >= 1024 (prefill sizes) read the received row and
 * slot counts back to the host once, after the dispatch, and size the local expert chain's
 * launches to them: those calls synchronise the host with the stream and cannot be recorded.  Every
 * wait is bounded (~2 s); a wait that gives up latches SX_ERR_DEVICE_TIMEOUT's device code
 * (sx_device_error) and the call's outputs are then undefined.  Results equal the NCCL transport's
 * bit for bit.  Requires every rank on one node with peer access (NVLink / NVSwitch).  No
 * reference counterpart. */

/* Peer-buffer bytes a call with these sizes needs (the same on every rank). */
size_t sx_ep_peer_bytes(const sx_ep* ep, int32_t rows_cap, int32_t hidden, int32_t topk, sx_dtype dtype);

/* Reserves `bytes` of peer buffer on every rank and maps each rank's into every other's (CUDA
 * IPC handles exchanged over the communicator).  Collective: every rank calls it with the same
 * bytes, with no sx_ep call of the communicator in flight (it synchronises the device).  A smaller
 * or equal request than the current reservation does nothing; a larger one replaces it.  bytes = 0
 * releases the reservation and returns the communicator to the NCCL transport. */
sx_status sx_ep_reserve_peer(sx_ep* ep, size_t bytes);

/* The reserved peer-buffer bytes (0: the NCCL transport). */
size_t sx_ep_peer_reserved(const sx_ep* ep);

/* Phase timing of the communicator's calls (diagnostics): with `enable`, every sx_ep_moe* call
 * records CUDA events on its stream at its phase boundaries (external event records, so a call
 * recorded in a CUDA graph records them at each replay), and sx_ep_phase_ms gives the last
 * recorded call's six phase durations in ms (waiting for its end):
 *   [0] plan + dispatch (peer: the row stores; NCCL: the send blocks' gather)
 *   [1] peer: waiting for every rank's rows; NCCL: the dispatch all-to-all
 *   [2] the local experts over the received rows
 *   [3] peer: the partials' reduce and stores into the owners' buffers; NCCL: the combine all-to-all
 *   [4] waiting for the shared expert on the side stream
 *   [5] the combine (peer: including the wait for every rank's partials)
 * Calls that run past a host-sized read of the received counts include that read in [1]. */
sx_status sx_ep_phase_timing(sx_ep* ep, int32_t enable);
sx_status sx_ep_phase_ms(sx_ep* ep, float ms[6]);

/* The communicator's world size and rank (either pointer may be null). */
sx_status sx_ep_info(const sx_ep* ep, int32_t* world, int32_t* rank);

/* ------------------------------------------------------------------ device error latch
 * Every bounded device-side wait that gives up records a code in a per-device latch instead of
 * hanging; the call that launched it may already have returned SX_OK.  Returns the latched code
 * (0 = none) and clears it; synchronises `stream` first. */
int32_t sx_device_error(sx_stream stream);

/* Failure-detection self-test: launches one kernel whose bounded wait nothing satisfies (an
 * mbarrier no thread arrives at).  The wait gives up after limit_ms (1..2000) and latches code 3,
 * which the next sx_device_error returns; the context stays usable.  No reference counterpart: it
 * checks the timeout path every kernel here relies on, without faulting or hanging the GPU. */
sx_status sx_selftest_wait_timeout(sx_stream stream, int32_t limit_ms);

/* Detail of the last SX_ERR_CUDA or SX_ERR_NCCL this thread got: the failing call's error and where
 * ("cudaLaunchKernelEx gemv: cudaErrorInvalidValue"); "" when there is none. */
const char* sx_last_error_detail(void);

/* The library's version string. */
const char* sx_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SUSHI_EXL3_H */
