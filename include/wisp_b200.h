/*
 * wisp_b200.h -- C ABI of libwisp_b200.so, the B200-native (sm_100a)
 * routed-expert int4 FFN hot path for the WISP engine.
 *
 * Part 1 re-exports the reference engine's GPU launcher ABI with identical
 * names and signatures, so the reference C engine links against this
 * library in place of its csrc/cuda/*.cu objects.
 * Part 2 adds the fused entry points the reference's gpu_expert_ffn /
 * run_moe would call instead of the dequant -> gemv -> scale_accum chain.
 *
 * No entry point allocates device memory per call: the caller passes every
 * buffer (workspace sizes come from the *_workspace_bytes queries). All
 * pointers named d_* are device pointers; launches are asynchronous on the
 * given stream.
 */
#ifndef WISP_B200_H
#define WISP_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* --------------------------------------------------------------------------
 * Engine types shared with the reference ABI. A translation unit that has
 * already included the reference's csrc/core/wisp_engine.h defines
 * WISP_B200_NO_ENGINE_TYPES before including this header.
 * Layouts are identical to csrc/core/wisp_engine.h:32-40, 50-64, 214-251.
 * ------------------------------------------------------------------------ */
#ifndef WISP_B200_NO_ENGINE_TYPES
typedef uint16_t wisp_half; /* raw fp16 bits (the reference's C view) */

typedef enum {
    WISP_OK = 0,
    WISP_ERR_OOM = 1,
    WISP_ERR_IO = 2,
    WISP_ERR_CUDA = 3,
    WISP_ERR_INVALID_ARG = 4,
    WISP_ERR_EXPERT_MISS = 5,
    WISP_ERR_MODEL = 6,
    WISP_ERR_TIMEOUT = 7,
} WispError;

typedef struct {
    WispError code;
    char message[512];
    const char* file;
    int line;
} WispErrCtx;

#define WISP_EXPERT_MAGIC 0x57455850u
#define WISP_EXPERT_VERSION 1u
#define WISP_EXPERT_NMATS 3

#pragma pack(push, 1)
typedef struct {
    uint32_t rows;
    uint32_t cols;
    uint64_t packed_bytes;
    uint64_t scales_bytes;
    uint64_t zeros_bytes;
} WispExpertMat;

typedef struct {
    uint32_t magic;
    uint32_t version;
    uint32_t layer_id;
    uint32_t expert_id;
    uint32_t group_size;
    uint32_t n_mats;
    WispExpertMat mats[WISP_EXPERT_NMATS];
} WispExpertHeader; /* exactly 120 bytes */
#pragma pack(pop)

typedef struct {
    size_t packed_off[WISP_EXPERT_NMATS];
    size_t scales_off[WISP_EXPERT_NMATS];
    size_t zeros_off[WISP_EXPERT_NMATS];
    uint32_t rows[WISP_EXPERT_NMATS];
    uint32_t cols[WISP_EXPERT_NMATS];
    uint32_t group_size;
    size_t total_bytes;
    int valid;
} WispExpertMeta;
#endif /* WISP_B200_NO_ENGINE_TYPES */

/* ==========================================================================
 * Part 1 -- reference launcher ABI (drop-in)
 * ======================================================================== */

/* Replaces csrc/cuda/expert_loader.cu:46-63 (declared at
 * csrc/core/wisp_engine.h:545-550). cudaErrorInvalidValue when
 * n_elements <= 0 or group_size <= 0, else the launch status. */
cudaError_t launch_dequant_expert(const uint8_t* d_packed, const wisp_half* d_scales,
                                  const wisp_half* d_zeros, wisp_half* d_output,
                                  int n_elements, int group_size, cudaStream_t stream);

/* Replaces csrc/cuda/expert_loader.cu:67-97 (wisp_engine.h:551-559). */
cudaError_t async_load_expert(const uint8_t* h_packed, const wisp_half* h_scales,
                              const wisp_half* h_zeros, uint8_t* d_packed_tmp,
                              wisp_half* d_scales_tmp, wisp_half* d_zeros_tmp,
                              wisp_half* d_output, int n_elements, int group_size,
                              cudaStream_t stream);

/* Replaces csrc/cuda/matmul.cu:58-65 (wisp_engine.h:499-500): y = W x. */
void wisp_gpu_gemv_f16(const wisp_half* W, const float* x, float* y, int rows, int cols,
                       cudaStream_t s);

/* Replaces csrc/cuda/matmul.cu:141-148 (wisp_engine.h:507-508). */
void wisp_gpu_swiglu(const float* gate, const float* up, float* out, int n, cudaStream_t s);

/* Replaces csrc/cuda/matmul.cu:198-205 (wisp_engine.h:509-511):
 * h[r] = silu(Wg[r].x) * (Wu[r].x). */
void wisp_gpu_swiglu_ffn(const wisp_half* Wg, const wisp_half* Wu, const float* x, float* h,
                         int inter, int cols, cudaStream_t s);

/* Replaces csrc/cuda/matmul.cu:156-161 (wisp_engine.h:512-513): acc += w x. */
void wisp_gpu_scale_accum(float* acc, const float* x, float w, int n, cudaStream_t s);

/* Replaces csrc/cuda/router.cu:140-171 (wisp_engine.h:534-537). Softmax
 * top-k with renormalised weights; ties go to the lower expert index.
 * out_idx / out_w are host (pinned) buffers filled by async copies on `s`;
 * the caller synchronises `s` before reading them. top_k is clamped to 64;
 * any n_experts (logits_scratch [n_experts] is working memory, as in the
 * reference: it holds exp(logit - max) afterwards). */
void wisp_gpu_router_topk(const wisp_half* W, const wisp_half* bias, const float* x,
                          float* logits_scratch, int n_experts, int hidden, int top_k,
                          int* out_idx, float* out_w, cudaStream_t s);

/* ==========================================================================
 * Part 2 -- fused entry points
 * ======================================================================== */

/* Parse an expert blob header held in HOST memory. Same contract as the
 * reference's wisp_expert_parse_header (csrc/core/wisp_engine.c:268-303):
 * WISP_ERR_MODEL on a bad magic/version/n_mats or a truncated blob. */
WispError wisp_b200_parse_expert_header(const void* blob, size_t blob_size,
                                        WispExpertMeta* meta, WispErrCtx* err);

/* One token, several experts, reference precision (fp32 activations):
 *   d_acc[hidden] += sum_j weights[j] * down_j(silu(gate_j x) * up_j x)
 * Replaces the per-expert loop of gpu_expert_ffn (csrc/core/wisp_engine.c:
 * 1507-1531) as called from run_moe (:1666-1670), plus an int4 shared
 * expert passed as one more blob with weight 1.0. d_blobs[j] is the device
 * address of blob j (header at offset 0; the packed weights must be at least
 * 8-byte aligned). weights is a HOST array. 1 <= n_blobs <= 16. The scratch
 * holds the intermediate activations; its size comes from
 * wisp_b200_expert_ffn_scratch_bytes. */
size_t wisp_b200_expert_ffn_scratch_bytes(const WispExpertMeta* meta, int n_blobs);
WispError wisp_b200_expert_ffn(const WispExpertMeta* meta, const void* const* d_blobs,
                               const float* weights, int n_blobs, const float* d_x,
                               float* d_acc, void* d_scratch, size_t scratch_bytes,
                               cudaStream_t stream, WispErrCtx* err);

/* The same computation for callers that cannot allocate device memory (an
 * engine whose VRAM budget is fully committed to the expert cache, or a
 * host callback where cudaMalloc would synchronise the device). No
 * counterpart in the reference. The intermediate activations use a fixed
 * 227 KB array per device compiled into the library, so n_blobs * inter must
 * be <= 58112 (else WISP_ERR_INVALID_ARG). The first call on a device looks
 * up that array's device address in the device's primary context; make it
 * before any stream capture, and do not use this entry after a
 * cudaDeviceReset or from another driver context. Calls share the array:
 * calls that overlap on the GPU race on it. */
WispError wisp_b200_expert_ffn_noalloc(const WispExpertMeta* meta, const void* const* d_blobs,
                                       const float* weights, int n_blobs, const float* d_x,
                                       float* d_acc, cudaStream_t stream, WispErrCtx* err);

/* --------------------------------------------------------------------------
 * Batched MoE layer (T tokens, bf16 activations).
 * ------------------------------------------------------------------------ */
enum { WISP_SCORE_SOFTMAX = 0, WISP_SCORE_SIGMOID_GROUPED = 1 };

typedef struct {
    int tokens;        /* T */
    int hidden;        /* M: multiple of 128 */
    int inter;         /* I: multiple of 128 */
    int n_experts;     /* routed experts E (<= 1024) */
    int top_k;         /* <= min(32, n_experts) */
    int group_size;    /* int4 quantisation group along K: 64 or 128 */
    int scoring;       /* WISP_SCORE_* */
    int n_groups;      /* sigmoid scoring: expert groups (E % n_groups == 0) */
    int topk_groups;   /* sigmoid scoring: groups kept */
    float routed_scaling; /* sigmoid scoring: weight multiplier */
    int has_shared;    /* 1: an always-on shared expert of the same shape */
    int router_fp16;   /* router weight dtype: 0 = bf16, 1 = fp16 (the
                          reference's router ABI, wisp_engine.h:534-537) */
    int deterministic; /* wisp_b200_moe_forward only (other entry points
                          ignore it). 0: expert outputs meet in fp32 atomics,
                          so results may differ in the last bits from run to
                          run. 1: the expert outputs are written as rows and
                          each token's are summed in a fixed order, so every
                          run gives the same bits; costs a (T x (top_k +
                          shared)) x hidden fp32 buffer in the workspace and
                          the single-token decode fast path. */
} WispMoeConfig;

/* One int4 matrix in the reference's packing (low nibble = even index,
 * value = (nibble - 8) * scale + zero, groups along K). zeros may be NULL
 * (symmetric). packed / scales / zeros must be 16-byte aligned. */
typedef struct {
    const uint8_t* packed;
    const wisp_half* scales;
    const wisp_half* zeros;
} WispInt4Mat;

/* gate [I x M], up [I x M], down [M x I]. */
typedef struct {
    WispInt4Mat gate, up, down;
} WispInt4Expert;

typedef struct {
    const uint16_t* router_w;       /* bf16 or fp16 [E x M] (cfg->router_fp16) */
    const float* router_bias;       /* fp32 [E], added before scoring; may be NULL */
    const WispInt4Expert* experts;  /* DEVICE array: E routed experts, then the
                                       shared expert when cfg->has_shared */
    const void* prepared;           /* from wisp_b200_prepare_experts over the
                                       same E (+1) entries */
} WispMoeWeights;

/* One-time preparation of a weight set for the tensor-core kernels (once per
 * layer when the weights are loaded, or when an expert blob is promoted into
 * the VRAM tier): per matrix a TMA descriptor of its packed nibbles, and its
 * scales / zero points transposed to [128-row tile][group][row] so each
 * stage's scales are one contiguous run. The packed nibbles stay where they
 * are and must stay valid. d_experts is a DEVICE array of n_entries; the call
 * copies it to the host, so it synchronises `stream`. */
size_t wisp_b200_prepared_bytes(const WispMoeConfig* cfg, int n_entries);
WispError wisp_b200_prepare_experts(const WispMoeConfig* cfg, const WispInt4Expert* d_experts,
                                    int n_entries, void* d_prepared, size_t prepared_bytes,
                                    cudaStream_t stream, WispErrCtx* err);

/* Re-prepares entry `slot` (0 <= slot < n_entries) of a prepared set in
 * place from a HOST copy of its expert-table entry and leaves every other
 * entry as it is: the hook for an expert blob that has just been promoted
 * into a VRAM slot (csrc/core/wisp_engine.c:1164-1203 copies the blob into
 * VRAM; this call then builds that slot's TMA descriptors and transposed
 * scales). The bytes it writes equal those wisp_b200_prepare_experts writes
 * for the same entry. The packed nibbles are used where they lie, in the
 * blob's own layout. Asynchronous on `stream`, with no host staging (the
 * descriptors travel as kernel parameters); updating the device expert
 * table entry itself is the caller's part. */
WispError wisp_b200_prepare_expert_slot(const WispMoeConfig* cfg, int n_entries, int slot,
                                        const WispInt4Expert* entry, void* d_prepared,
                                        size_t prepared_bytes, cudaStream_t stream,
                                        WispErrCtx* err);

/* The expert-table entry of a reference expert blob that lies at device
 * address d_blob: pointers to its gate, up and down packed nibbles, scales
 * and (when the blob carries them) zero points, at the offsets of the
 * parsed header (csrc/core/wisp_engine.c:268-303). Host-only pointer
 * arithmetic: d_blob is never dereferenced. WISP_ERR_INVALID_ARG when meta
 * is invalid or a matrix's packed data or scales would not be 16-byte
 * aligned (a blob placed at an address = 8 mod 16 has both aligned, since
 * its packed data starts at offset 120). */
WispError wisp_b200_blob_expert(const WispExpertMeta* meta, const void* d_blob,
                                WispInt4Expert* out, WispErrCtx* err);

size_t wisp_b200_moe_workspace_bytes(const WispMoeConfig* cfg);

/* out[T x M] (fp32) = sum_k w[t,k] * expert_{idx[t,k]}(x_t) + shared(x_t).
 * x: bf16 [T x M]. topk_idx / topk_w ([T x k], int32 / fp32) receive the
 * routing and may be NULL. */
WispError wisp_b200_moe_forward(const WispMoeConfig* cfg, const WispMoeWeights* w,
                                const uint16_t* d_x, float* d_out, int* d_topk_idx,
                                float* d_topk_w, void* d_workspace, size_t workspace_bytes,
                                cudaStream_t stream, WispErrCtx* err);

/* Dense int4 MLP over T tokens (the MLP of the first dense layers of
 * DeepSeek/GLM models, csrc/core/wisp_engine.c:1676-1686, and any
 * always-on MLP quantised to int4):
 *   d_out[T x M] (fp32) = down(silu(gate x) * up x), x bf16 [T x M].
 * d_mlp is a DEVICE array holding the MLP's one WispInt4Expert entry and
 * d_prepared its prepared set (wisp_b200_prepare_experts over that entry).
 * Uses cfg's tokens, hidden, inter and group_size only. The output rows are
 * written, not accumulated. d_error_flag as for wisp_b200_grouped_ffn (may
 * be NULL). One call at a time per workspace. */
size_t wisp_b200_dense_mlp_workspace_bytes(const WispMoeConfig* cfg);
WispError wisp_b200_dense_mlp(const WispMoeConfig* cfg, const void* d_prepared,
                              const WispInt4Expert* d_mlp, const uint16_t* d_x, float* d_out,
                              void* d_workspace, size_t workspace_bytes, int* d_error_flag,
                              cudaStream_t stream, WispErrCtx* err);

/* --------------------------------------------------------------------------
 * Building blocks (used by the expert-parallel path and by tests).
 * ------------------------------------------------------------------------ */

/* Router only: d_idx / d_w [T x k]; d_logits (fp32 [T x E]) receives the
 * logits, bias included. */
WispError wisp_b200_route(const WispMoeConfig* cfg, const WispMoeWeights* w, const uint16_t* d_x,
                          float* d_logits, int* d_idx, float* d_w, cudaStream_t stream,
                          WispErrCtx* err);

/* The same routing with the logits summed over K splits, so that a few
 * tokens still spread over the SMs (wisp_b200_route computes each token
 * tile's logits in one pass over K). d_workspace holds the split partial
 * sums (wisp_b200_route_workspace_bytes, 16-byte aligned; one call at a
 * time per workspace); d_logits may be NULL. Same results as
 * wisp_b200_route within fp32 summation order. */
size_t wisp_b200_route_workspace_bytes(const WispMoeConfig* cfg);
WispError wisp_b200_route_ws(const WispMoeConfig* cfg, const WispMoeWeights* w,
                             const uint16_t* d_x, float* d_logits, int* d_idx, float* d_w,
                             void* d_workspace, size_t workspace_bytes, cudaStream_t stream,
                             WispErrCtx* err);

/* A contiguous run of activation rows that all go through one expert. */
typedef struct {
    int32_t expert;    /* index into the expert table */
    int32_t row_begin; /* first row in the activation buffer */
    int32_t rows;      /* number of rows (0 allowed) */
    int32_t reserved;
} WispSegment;

/* Grouped expert FFN over pre-permuted rows. d_prepared / d_experts /
 * n_entries: a prepared weight set and its device expert table (segment
 * experts index its entries). Segments of at most 32 rows (decode) run on
 * the register-fed integer tensor-core kernel, larger ones on the tcgen05
 * kernel.
 *   d_xp:   fp16 [R x M] activation rows in interleaved K order (within each
 *           8 K: 0,4,1,5,2,6,3,7) -- produced by wisp_b200_pack_rows.
 *   d_segs: DEVICE array of n_segs segments.
 *   d_h:    [R x I] scratch of 2 bytes per element (the SwiGLU output: fp16
 *           rows for tensor-core segments, 16-bit integer rows with
 *           per-128-K scales in the workspace for register-path segments).
 *   mode 0: d_out[row_token[p] * M + m] += row_weight[p] * y[p, m] (atomic fp32)
 *   mode 1: d_y[p * M + m] = y[p, m] (fp32 rows, no weighting)
 * d_workspace: wisp_b200_grouped_workspace_bytes(cfg, n_segs, rows_capacity)
 *          bytes, 256-byte aligned (tile and unit plans, the register path's
 *          integer activation rows and their scales, and ~33.5 MB for the
 *          partial sums of a K-split gate/up); one call at a time per
 *          workspace.
 * d_error_flag: device int set to nonzero if a bounded wait gave up (may be
 * NULL); check it with wisp_b200_check_error_flag. */
size_t wisp_b200_grouped_workspace_bytes(const WispMoeConfig* cfg, int n_segs, int rows_capacity);
WispError wisp_b200_grouped_ffn(const WispMoeConfig* cfg, const void* d_prepared,
                                const WispInt4Expert* d_experts, int n_entries,
                                const WispSegment* d_segs, int n_segs, int rows_capacity,
                                const uint16_t* d_xp, uint16_t* d_h, int mode,
                                const int* d_row_token, const float* d_row_weight,
                                float* d_out, void* d_workspace, size_t workspace_bytes,
                                int* d_error_flag, cudaStream_t stream, WispErrCtx* err);

/* Dispatch plan from a routing: one segment per expert (then the shared
 * expert with every token when cfg->has_shared), rows sorted by (token,
 * slot) inside each expert. d_counts [V], d_segs [V], d_row_token /
 * d_row_weight [T*k (+T)], V = E (+1). Deterministic. */
WispError wisp_b200_dispatch_plan(const WispMoeConfig* cfg, const int* d_idx, const float* d_w,
                                  int* d_counts, WispSegment* d_segs, int* d_row_token,
                                  float* d_row_weight, cudaStream_t stream, WispErrCtx* err);

/* d_out[row_token[p]] += row_weight[p] * d_y[p] for p < n_rows (fp32 rows;
 * atomic adds): the combine step of the expert-parallel path. */
WispError wisp_b200_combine_rows(const float* d_y, const int* d_row_token, const float* d_row_weight,
                                 int n_rows, int hidden, float* d_out, cudaStream_t stream,
                                 WispErrCtx* err);

/* --------------------------------------------------------------------------
 * Expert-parallel exchange (no counterpart in the reference, which runs on one
 * GPU). Experts are sharded in contiguous blocks of e_loc = n_experts/world.
 * Each rank pair exchanges one fixed-size block per direction, so all counts
 * stay on the device; a token travels to an owner rank once, whatever the
 * number of its experts there. cap = the most tokens any rank holds. Block
 * layout (wisp_b200_ep_block_bytes bytes, 16-byte aligned parts):
 *   int32 n_rows, 3 pad; int32 cnt[e_loc]           header
 *   int32 ent_row[cap*top_k]; float ent_w[cap*top_k] entries, expert-major
 *   fp16 rows[cap][hidden]                           interleaved K order
 * ------------------------------------------------------------------------ */
size_t wisp_b200_ep_block_bytes(int hidden, int e_loc, int cap, int top_k);

/* Send side: d_send [world blocks] from this rank's routing (d_topk_idx
 * [tokens x top_k], global experts) and its dispatch plan over the n_experts
 * routed experts (d_plan_segs, d_row_token, d_row_weight from
 * wisp_b200_dispatch_plan with has_shared = 0). d_slot [tokens x world]
 * receives the row of each token in each block (-1: not sent there). d_own
 * (may be NULL) receives the same rows for this rank's own tokens [tokens x
 * hidden] (fp16, interleaved K order), the shared expert's input. */
WispError wisp_b200_ep_dispatch(const uint16_t* d_x, int tokens, int hidden, const int* d_topk_idx,
                                int top_k, const WispSegment* d_plan_segs, const int* d_row_token,
                                const float* d_row_weight, int n_experts, int world, int cap,
                                uint8_t* d_send, int* d_slot, uint16_t* d_own,
                                cudaStream_t stream, WispErrCtx* err);

/* Receive side, from the received blocks d_recv [world blocks] (world * e_loc
 * <= 1024): the entries are gathered expert-contiguous (expert, then source)
 * so each local expert is one segment: d_segs [e_loc] over the gathered
 * rows, d_src_pos[j] = receive row (source * cap + block row) and
 * d_weight[j] = routing weight of gathered row j, *d_total = entries.
 * own_rows > 0 (<= cap) appends this rank's own own_rows token rows as
 * segment e_loc (the shared expert's entry of the local table), with
 * d_src_pos = world * cap + t and weight 1, so the shared expert runs in the
 * same grouped call as the routed experts. d_src_pos and d_weight hold
 * world * cap * top_k + own_rows entries, d_segs e_loc (+1). */
WispError wisp_b200_ep_recv_plan(const uint8_t* d_recv, int world, int e_loc, int cap, int top_k,
                                 int hidden, int own_rows, WispSegment* d_segs, int* d_src_pos,
                                 float* d_weight, int* d_total, cudaStream_t stream,
                                 WispErrCtx* err);

/* d_sorted[j] = receive row d_src_pos[j] for j < *d_total + own_rows (fp16
 * rows; a d_src_pos of world * cap + t reads row t of d_own, this rank's own
 * token rows packed with wisp_b200_pack_rows; max_rows bounds the launch,
 * normally world * cap * top_k + own_rows). The grouped FFN then runs in
 * mode 0 with row_token = d_src_pos and row_weight = d_weight into fp32 rows
 * [(world * cap + own_rows) x hidden] (zeroed first): one row per received
 * token, which the return exchange sends back, then the shared expert's
 * output for each own token. */
WispError wisp_b200_ep_gather_rows(const uint8_t* d_recv, int world, int e_loc, int cap, int top_k,
                                   int hidden, const int* d_src_pos, const int* d_total,
                                   const uint16_t* d_own, int own_rows, int max_rows,
                                   uint16_t* d_sorted, cudaStream_t stream, WispErrCtx* err);

/* d_out[t] += d_yback[q * cap + d_slot[t * world + q]] over q = 0..world-1
 * with a slot >= 0, in rank order (fp32 rows; one block per token). */
WispError wisp_b200_ep_combine(const float* d_yback, const int* d_slot, int tokens, int world,
                               int cap, int hidden, float* d_out, cudaStream_t stream,
                               WispErrCtx* err);

/* The return exchange in fp16 (half the bytes of fp32 rows): the owner
 * rounds its fp32 return rows to fp16 (d_y16[i] = fp16(d_y[i]) for rows x
 * hidden values), the rows travel, and the home rank adds them in rank
 * order with wisp_b200_ep_combine_f16 (wisp_b200_ep_combine's contract with
 * fp16 rows; with d_local non-NULL, fp32 [tokens x hidden], the result is
 * d_out[t] = d_local[t] + the returned rows, written rather than added). */
WispError wisp_b200_ep_return_rows(const float* d_y, int rows, int hidden, uint16_t* d_y16,
                                   cudaStream_t stream, WispErrCtx* err);
WispError wisp_b200_ep_combine_f16(const uint16_t* d_yback, const int* d_slot,
                                   const float* d_local, int tokens, int world, int cap,
                                   int hidden, float* d_out, cudaStream_t stream,
                                   WispErrCtx* err);

/* Between stacked layers: d_out[t] = bf16(d_in[t] / rms(d_in[t])), fp32 in. */
WispError wisp_b200_rms_rescale(const float* d_in, uint16_t* d_out, int tokens, int hidden,
                                float eps, cudaStream_t stream, WispErrCtx* err);

/* Copy bf16 rows into fp16 interleaved-K rows: xp[p] = x[src[p]] for
 * p < n_rows (src may be NULL: identity). */
WispError wisp_b200_pack_rows(const uint16_t* d_x, const int* d_src, int n_rows, int hidden,
                              uint16_t* d_xp, cudaStream_t stream, WispErrCtx* err);

/* Device error word written by the tcgen05 kernels when a bounded wait gave
 * up (nonzero = the results of that launch are invalid). */
WispError wisp_b200_check_error_flag(const int* d_error_flag, cudaStream_t stream,
                                     WispErrCtx* err);

/* Address of the device error word inside a wisp_b200_moe_forward
 * workspace (cleared at the start of every forward). */
int* wisp_b200_moe_error_word(const WispMoeConfig* cfg, void* d_workspace);

/* Diagnostics: when d_counters (38 uint64, zeroed by the caller) is
 * non-NULL, the grouped kernels accumulate the clock cycles each role spends
 * in each of its waits: the tensor-core gate/up kernel in [0,15), its down
 * kernel in [15,30), the register-path gate/up kernel in [30,34) and its
 * down kernel in [34,38). Pass NULL to switch off. Not thread-safe; for
 * profiling runs only. */
void wisp_b200_debug_set_counters(unsigned long long* d_counters);

/* Largest segment (rows) routed to the register-fed kernel, which takes any
 * segment in chunks of 16 rows; 0 sends every segment to the tcgen05 kernel,
 * a negative value restores the default. Process-wide; for tests and
 * tuning. */
void wisp_b200_set_skinny_max_rows(int rows);

/* Library version string. */
const char* wisp_b200_version(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* WISP_B200_H */
