// moe.cu -- host orchestration of the batched MoE layer and the small
// host-side pieces of the ABI (blob header parsing, error word, version).
//
// wisp_b200_moe_forward runs, on one stream and without any host sync:
//   route (logits + top-k) -> dispatch plan (segments, row -> token map)
//   -> pack rows (q16 rows for register-path segments, fp16 interleaved
//      rows for tensor-core ones) -> zero out
//   -> grouped gate/up + SwiGLU -> grouped down + weighted scatter-combine
//      (fp32 atomics into out), each on the register-path kernel for
//      segments of up to 32 rows and on the tcgen05 kernel for larger ones.
// Decode batches of at most 4 tokens take a shorter chain: router logits,
// one planner launch (top-k, plan, q16 rows, zeroing, unit plans), then the
// register-path gate/up and down launches.
// It is the batched counterpart of run_moe (csrc/core/wisp_engine.c:
// 1563-1674), which the reference can only run one token at a time.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace wb {
size_t router_splits(int T, int E, int M);
WispError launch_route(const WispMoeConfig* c, const uint16_t* x, const uint16_t* W,
                       const float* bias, float* part, size_t splits, float* logits_out, int* idx,
                       float* w, cudaStream_t st, WispErrCtx* err);
WispError launch_plan(const WispMoeConfig* c, const int* idx, const float* w, int* counts,
                      WispSegment* segs, int* row_token, float* row_weight, cudaStream_t st,
                      WispErrCtx* err, int* scratch);
size_t plan_scratch_ints(const WispMoeConfig* c);
WispError launch_pack(const uint16_t* x, const int* src, int n_rows, int M, uint16_t* xp,
                      cudaStream_t st, WispErrCtx* err);
WispError launch_pack_q16(const uint16_t* x, const int* src, int n_rows, int M, uint16_t* xp,
                          uint8_t* xq, const WispSegment* segs, int nseg, int sk_rows,
                          cudaStream_t st, WispErrCtx* err);
int grouped_sk_rows(int n_segs, int n_entries);
uint8_t* grouped_xq(void* d_workspace, int n_segs, int rows_capacity, int M, int I);
WispError grouped_ffn_impl(const WispMoeConfig* cfg, const void* d_prepared,
                           const WispInt4Expert* d_experts, int n_entries,
                           const WispSegment* d_segs, int n_segs, int rows_capacity,
                           const uint16_t* d_xp, uint16_t* d_h, int mode, const int* d_row_token,
                           const float* d_row_weight, float* d_out, void* d_workspace,
                           size_t workspace_bytes, int* d_error_flag, bool xq_ready,
                           int max_seg_rows, cudaStream_t stream, WispErrCtx* err,
                           bool plans_ready = false);
void decode_units(const WispMoeConfig* cfg, int n_segs, int n_entries, int rows_capacity, int mode,
                  void* d_workspace, DecodeUnits* du);
WispError launch_router_gemv(const WispMoeConfig* c, const uint16_t* x, const uint16_t* W,
                             float* logits, cudaStream_t st, WispErrCtx* err);
bool decode_plan_fits(const WispMoeConfig* c, int sk_rows);
WispError launch_decode_plan(const WispMoeConfig* c, const float* logits, const float* bias,
                             int* idx, float* w, int* counts, WispSegment* segs, int* row_token,
                             float* row_weight, const uint16_t* x, float* out, int* error_flag,
                             const DecodeUnits& du, cudaStream_t st, WispErrCtx* err);
}  // namespace wb

namespace {

struct Carve {
  size_t off = 0;
  template <typename T>
  T* take(void* base, size_t count) {
    off = (off + 255) & ~(size_t)255;
    T* p = base ? reinterpret_cast<T*>(static_cast<uint8_t*>(base) + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

struct Workspace {
  float* part;
  int* plan_scratch;
  int* idx;
  float* w;
  int* counts;
  WispSegment* segs;
  int* row_token;
  float* row_weight;
  void* grouped;
  size_t grouped_bytes;
  int* error_flag;
  uint16_t* xp;
  uint16_t* h;
  // deterministic layers only: the expert outputs, one fp32 row per routed
  // row, and each token's rows
  float* y;
  int* tok_cnt;
  int* tok_list;
  int lanes;   // rows per token: top_k (+ 1 with a shared expert)
  size_t bytes;
  size_t splits;
  int rows;
};

Workspace carve(const WispMoeConfig* c, void* base) {
  Workspace ws;
  Carve cv;
  const int T = c->tokens, E = c->n_experts, k = c->top_k, M = c->hidden, I = c->inter;
  const int V = E + (c->has_shared ? 1 : 0);
  ws.rows = T * k + (c->has_shared ? T : 0);
  ws.splits = wb::router_splits(T, E, M);
  ws.part = cv.take<float>(base, ws.splits * (size_t)T * E);
  ws.plan_scratch = cv.take<int>(base, std::max<size_t>(1, wb::plan_scratch_ints(c)));
  ws.idx = cv.take<int>(base, (size_t)T * k);
  ws.w = cv.take<float>(base, (size_t)T * k);
  ws.counts = cv.take<int>(base, V);
  ws.segs = cv.take<WispSegment>(base, V);
  ws.row_token = cv.take<int>(base, ws.rows);
  ws.row_weight = cv.take<float>(base, ws.rows);
  ws.grouped_bytes = wisp_b200_grouped_workspace_bytes(c, V, ws.rows);
  ws.grouped = cv.take<uint8_t>(base, ws.grouped_bytes);
  ws.error_flag = cv.take<int>(base, 1);
  ws.xp = cv.take<uint16_t>(base, (size_t)ws.rows * M);
  ws.h = cv.take<uint16_t>(base, (size_t)ws.rows * I);
  ws.lanes = k + (c->has_shared ? 1 : 0);
  ws.y = nullptr;
  ws.tok_cnt = ws.tok_list = nullptr;
  if (c->deterministic) {
    ws.y = cv.take<float>(base, (size_t)ws.rows * M);
    ws.tok_cnt = cv.take<int>(base, T);
    ws.tok_list = cv.take<int>(base, (size_t)T * ws.lanes);
  }
  ws.bytes = (cv.off + 255) & ~(size_t)255;
  return ws;
}

// Deterministic combine (WispMoeConfig.deterministic). The expert outputs
// arrive as plain fp32 rows (grouped FFN mode 1: no weights, no atomics, no
// K split of the down projection); each token's output is then the sum of
// its rows in ascending row order -- routed experts by index, then the
// shared expert -- so every run produces the same bits, where the atomics
// of the fused combine add in whatever order the hardware picks.
// Step 1: each token's rows into a per-token list (in any order).
__global__ void token_rows_kernel(const int* __restrict__ row_token,
                                  const WispSegment* __restrict__ segs, int V, int cap, int lanes,
                                  int* __restrict__ cnt, int* __restrict__ list) {
  const int total = min(cap, segs[V - 1].row_begin + segs[V - 1].rows);
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < total; p += gridDim.x * blockDim.x) {
    const int t = row_token[p];
    const int j = atomicAdd(cnt + t, 1);
    if (j < lanes) list[(size_t)t * lanes + j] = p;
  }
}

// Step 2: one block per (token, 1024 columns): the token's rows sorted by
// position, then out[t][m] = sum over them, in that order, of weight * y.
constexpr int kDetMaxLanes = 64;
__global__ void combine_ordered_kernel(const float* __restrict__ y,
                                       const float* __restrict__ row_weight,
                                       const int* __restrict__ cnt, const int* __restrict__ list,
                                       int lanes, int M, float* __restrict__ out) {
  __shared__ int s_p[kDetMaxLanes];
  __shared__ float s_w[kDetMaxLanes];
  __shared__ int s_n;
  const int t = blockIdx.x;
  if (threadIdx.x == 0) {
    const int n = min(cnt[t], lanes);
    for (int i = 0; i < n; i++) {   // insertion sort of at most 33 positions
      const int v = list[(size_t)t * lanes + i];
      int j = i;
      while (j > 0 && s_p[j - 1] > v) {
        s_p[j] = s_p[j - 1];
        j--;
      }
      s_p[j] = v;
    }
    for (int i = 0; i < n; i++) s_w[i] = row_weight[s_p[i]];
    s_n = n;
  }
  __syncthreads();
  const int n = s_n;
  const int m1 = min(M, (int)(blockIdx.y + 1) * 1024);
  for (int m = (int)blockIdx.y * 1024 + threadIdx.x; m < m1; m += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < n; i++) acc = fmaf(s_w[i], y[(size_t)s_p[i] * M + m], acc);
    out[(size_t)t * M + m] = acc;
  }
}

WispError validate(const WispMoeConfig* c, WispErrCtx* err) {
  if (!c) return WB_FAIL(WISP_ERR_INVALID_ARG, "moe: null config");
  if (c->tokens <= 0 || c->n_experts <= 0 || c->n_experts > 1024)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "moe: tokens=%d n_experts=%d (1..1024)", c->tokens, c->n_experts);
  if (c->top_k <= 0 || c->top_k > 32 || c->top_k > c->n_experts)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "moe: top_k=%d (1..min(32, n_experts))", c->top_k);
  if (c->hidden <= 0 || c->inter <= 0 || c->hidden % 128 || c->inter % 128)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "moe: hidden=%d inter=%d must be multiples of 128", c->hidden, c->inter);
  if (c->group_size != 64 && c->group_size != 128)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "moe: group_size=%d (64 or 128)", c->group_size);
  if (c->scoring == WISP_SCORE_SIGMOID_GROUPED) {
    if (c->n_groups <= 0 || c->n_groups > 32 || c->n_experts % c->n_groups ||
        c->topk_groups <= 0 || c->topk_groups > c->n_groups ||
        c->top_k > c->topk_groups * (c->n_experts / c->n_groups))
      return WB_FAIL(WISP_ERR_INVALID_ARG, "moe: bad group routing (E=%d groups=%d keep=%d k=%d)",
                     c->n_experts, c->n_groups, c->topk_groups, c->top_k);
  } else if (c->scoring != WISP_SCORE_SOFTMAX) {
    return WB_FAIL(WISP_ERR_INVALID_ARG, "moe: unknown scoring %d", c->scoring);
  }
  return WISP_OK;
}

}  // namespace

extern "C" size_t wisp_b200_moe_workspace_bytes(const WispMoeConfig* cfg) {
  if (validate(cfg, nullptr) != WISP_OK) return 0;
  return carve(cfg, nullptr).bytes;
}

extern "C" WispError wisp_b200_route(const WispMoeConfig* cfg, const WispMoeWeights* w,
                                     const uint16_t* d_x, float* d_logits, int* d_idx, float* d_w,
                                     cudaStream_t stream, WispErrCtx* err) {
  WispError e = validate(cfg, err);
  if (e != WISP_OK) return e;
  if (!w || !w->router_w || !d_x || !d_logits || !d_idx || !d_w)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "route: null pointer argument");
  // d_logits serves as the (single-split) partial buffer and then receives
  // the final logits (bias included); each token's row is read before it
  // is rewritten by the same thread.
  return wb::launch_route(cfg, d_x, w->router_w, w->router_bias, d_logits, 1, d_logits, d_idx, d_w,
                          stream, err);
}

namespace {
// wisp_b200_route_ws workspace: the split partial sums.
size_t route_part_bytes(const WispMoeConfig* cfg) {
  const size_t n = wb::router_splits(cfg->tokens, cfg->n_experts, cfg->hidden) *
                   (size_t)cfg->tokens * cfg->n_experts * sizeof(float);
  return (n + 255) & ~(size_t)255;
}
}  // namespace

extern "C" size_t wisp_b200_route_workspace_bytes(const WispMoeConfig* cfg) {
  if (validate(cfg, nullptr) != WISP_OK) return 0;
  return route_part_bytes(cfg);
}

extern "C" WispError wisp_b200_route_ws(const WispMoeConfig* cfg, const WispMoeWeights* w,
                                        const uint16_t* d_x, float* d_logits, int* d_idx,
                                        float* d_w, void* d_workspace, size_t workspace_bytes,
                                        cudaStream_t stream, WispErrCtx* err) {
  WispError e = validate(cfg, err);
  if (e != WISP_OK) return e;
  if (!w || !w->router_w || !d_x || !d_idx || !d_w || !d_workspace)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "route_ws: null pointer argument");
  const size_t splits = wb::router_splits(cfg->tokens, cfg->n_experts, cfg->hidden);
  const size_t need = wisp_b200_route_workspace_bytes(cfg);
  if (workspace_bytes < need)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "route_ws: workspace %zu < required %zu", workspace_bytes,
                   need);
  if (((uintptr_t)d_x | (uintptr_t)w->router_w | (uintptr_t)d_workspace) & 15)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "route_ws: x, router_w and workspace must be 16-byte aligned");
  return wb::launch_route(cfg, d_x, w->router_w, w->router_bias, static_cast<float*>(d_workspace),
                          splits, d_logits, d_idx, d_w, stream, err);
}

extern "C" WispError wisp_b200_moe_forward(const WispMoeConfig* cfg, const WispMoeWeights* w,
                                           const uint16_t* d_x, float* d_out, int* d_topk_idx,
                                           float* d_topk_w, void* d_workspace,
                                           size_t workspace_bytes, cudaStream_t stream,
                                           WispErrCtx* err) {
  WispError e = validate(cfg, err);
  if (e != WISP_OK) return e;
  if (!w || !w->router_w || !w->prepared || !d_x || !d_out || !d_workspace)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "moe_forward: null pointer argument (router_w, prepared, x, out, workspace)");
  if (((uintptr_t)d_x | (uintptr_t)w->router_w | (uintptr_t)d_workspace) & 15)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "moe_forward: x, router_w and workspace must be 16-byte aligned");
  Workspace ws = carve(cfg, d_workspace);
  if (workspace_bytes < ws.bytes)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "moe_forward: workspace %zu < required %zu", workspace_bytes, ws.bytes);
  int* idx = d_topk_idx ? d_topk_idx : ws.idx;
  float* wt = d_topk_w ? d_topk_w : ws.w;
  const int V = cfg->n_experts + (cfg->has_shared ? 1 : 0);
  if (!w->experts) return WB_FAIL(WISP_ERR_INVALID_ARG, "moe_forward: null expert table");

  // Decode batches (T <= 4): router logits, then one planner launch for
  // top-k, dispatch plan, q16 rows, output zeroing and the register path's
  // unit plans, then the register-path gate/up and down launches.
  const bool det = cfg->deterministic != 0;
  if (!det && wb::decode_plan_fits(cfg, wb::grouped_sk_rows(V, V))) {
    // ws.part holds splits * T * E floats, splits >= 1: room for the logits
    e = wb::launch_router_gemv(cfg, d_x, w->router_w, ws.part, stream, err);
    if (e != WISP_OK) return e;
    wb::DecodeUnits du;
    wb::decode_units(cfg, V, V, ws.rows, 0, ws.grouped, &du);
    e = wb::launch_decode_plan(cfg, ws.part, w->router_bias, idx, wt, ws.counts, ws.segs,
                               ws.row_token, ws.row_weight, d_x, d_out, ws.error_flag, du, stream,
                               err);
    if (e != WISP_OK) return e;
    return wb::grouped_ffn_impl(cfg, w->prepared, w->experts, V, ws.segs, V, ws.rows, ws.xp, ws.h,
                                0, ws.row_token, ws.row_weight, d_out, ws.grouped,
                                ws.grouped_bytes, ws.error_flag, true, cfg->tokens, stream, err,
                                true);
  }

  e = wb::launch_route(cfg, d_x, w->router_w, w->router_bias, ws.part, ws.splits, nullptr, idx, wt,
                       stream, err);
  if (e != WISP_OK) return e;
  e = wb::launch_plan(cfg, idx, wt, ws.counts, ws.segs, ws.row_token, ws.row_weight, stream, err,
                      ws.plan_scratch);
  if (e != WISP_OK) return e;
  // The gathered rows in the operand form of the kernel their segment runs
  // on: fp16 for the tensor-core kernel, q16 (into the grouped workspace) for
  // the register path.
  e = wb::launch_pack_q16(d_x, ws.row_token, ws.rows, cfg->hidden, ws.xp,
                          wb::grouped_xq(ws.grouped, V, ws.rows, cfg->hidden, cfg->inter), ws.segs,
                          V, wb::grouped_sk_rows(V, V), stream, err);
  if (e != WISP_OK) return e;
  WB_CUDA_CHECK(cudaMemsetAsync(ws.error_flag, 0, sizeof(int), stream));
  if (det) {
    // expert outputs as rows, then the fixed-order combine
    e = wb::grouped_ffn_impl(cfg, w->prepared, w->experts, V, ws.segs, V, ws.rows, ws.xp, ws.h, 1,
                             ws.row_token, ws.row_weight, ws.y, ws.grouped, ws.grouped_bytes,
                             ws.error_flag, true, cfg->tokens, stream, err);
    if (e != WISP_OK) return e;
    WB_CUDA_CHECK(cudaMemsetAsync(ws.tok_cnt, 0, (size_t)cfg->tokens * sizeof(int), stream));
    wb::launch_k(token_rows_kernel, (ws.rows + 255) / 256, 256, 0, stream, ws.row_token, ws.segs, V,
                 ws.rows, ws.lanes, ws.tok_cnt, ws.tok_list);
    wb::launch_k(combine_ordered_kernel, dim3(cfg->tokens, (cfg->hidden + 1023) / 1024), 256, 0,
                 stream, ws.y, ws.row_weight, ws.tok_cnt, ws.tok_list, ws.lanes, cfg->hidden, d_out);
    WB_CUDA_CHECK(cudaGetLastError());
    return WISP_OK;
  }
  WB_CUDA_CHECK(cudaMemsetAsync(d_out, 0, (size_t)cfg->tokens * cfg->hidden * sizeof(float), stream));
  // A routed expert gets at most one row per token and the shared expert T
  // rows, so no segment exceeds T rows.
  return wb::grouped_ffn_impl(cfg, w->prepared, w->experts, V, ws.segs, V, ws.rows, ws.xp, ws.h, 0,
                              ws.row_token, ws.row_weight, d_out, ws.grouped, ws.grouped_bytes,
                              ws.error_flag, true, cfg->tokens, stream, err);
}

// ---------------------------------------------------------------------------
// Dense int4 MLP: the MLP as the one segment of a one-entry weight set, run
// through the grouped kernels in mode 1 (plain fp32 row stores, no weights,
// no atomics). The reference runs this MLP in fp16 through op_swiglu_ffn +
// op_gemv (csrc/core/wisp_engine.c:1676-1686).
// ---------------------------------------------------------------------------
namespace {

__global__ void one_segment_kernel(WispSegment* s, int rows) {
  WispSegment v;
  v.expert = 0;
  v.row_begin = 0;
  v.rows = rows;
  v.reserved = 0;
  *s = v;
}

struct DenseWs {
  WispSegment* seg;
  void* grouped;
  size_t grouped_bytes;
  uint16_t* xp;
  uint16_t* h;
  size_t bytes;
};

DenseWs carve_dense(const WispMoeConfig* c, void* base) {
  DenseWs ws;
  Carve cv;
  const int T = c->tokens;
  ws.seg = cv.take<WispSegment>(base, 1);
  ws.grouped_bytes = wisp_b200_grouped_workspace_bytes(c, 1, T);
  ws.grouped = cv.take<uint8_t>(base, ws.grouped_bytes);
  ws.xp = cv.take<uint16_t>(base, (size_t)T * c->hidden);
  ws.h = cv.take<uint16_t>(base, (size_t)T * c->inter);
  ws.bytes = (cv.off + 255) & ~(size_t)255;
  return ws;
}

WispError validate_dense(const WispMoeConfig* c, WispErrCtx* err) {
  if (!c) return WB_FAIL(WISP_ERR_INVALID_ARG, "dense_mlp: null config");
  if (c->tokens <= 0 || c->hidden <= 0 || c->inter <= 0 || c->hidden % 128 || c->inter % 128)
    return WB_FAIL(WISP_ERR_INVALID_ARG,
                   "dense_mlp: tokens=%d hidden=%d inter=%d (hidden, inter multiples of 128)",
                   c->tokens, c->hidden, c->inter);
  if (c->group_size != 64 && c->group_size != 128)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "dense_mlp: group_size=%d (64 or 128)", c->group_size);
  return WISP_OK;
}

}  // namespace

extern "C" size_t wisp_b200_dense_mlp_workspace_bytes(const WispMoeConfig* cfg) {
  if (validate_dense(cfg, nullptr) != WISP_OK) return 0;
  return carve_dense(cfg, nullptr).bytes;
}

extern "C" WispError wisp_b200_dense_mlp(const WispMoeConfig* cfg, const void* d_prepared,
                                         const WispInt4Expert* d_mlp, const uint16_t* d_x,
                                         float* d_out, void* d_workspace, size_t workspace_bytes,
                                         int* d_error_flag, cudaStream_t stream, WispErrCtx* err) {
  WispError e = validate_dense(cfg, err);
  if (e != WISP_OK) return e;
  if (!d_prepared || !d_mlp || !d_x || !d_out || !d_workspace)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "dense_mlp: null pointer argument");
  if (((uintptr_t)d_x | (uintptr_t)d_workspace) & 15)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "dense_mlp: x and workspace must be 16-byte aligned");
  const DenseWs ws = carve_dense(cfg, d_workspace);
  if (workspace_bytes < ws.bytes)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "dense_mlp: workspace %zu < required %zu",
                   workspace_bytes, ws.bytes);
  const int T = cfg->tokens;
  one_segment_kernel<<<1, 1, 0, stream>>>(ws.seg, T);
  WB_CUDA_CHECK(cudaGetLastError());
  e = wb::launch_pack_q16(d_x, nullptr, T, cfg->hidden, ws.xp,
                          wb::grouped_xq(ws.grouped, 1, T, cfg->hidden, cfg->inter), ws.seg, 1,
                          wb::grouped_sk_rows(1, 1), stream, err);
  if (e != WISP_OK) return e;
  return wb::grouped_ffn_impl(cfg, d_prepared, d_mlp, 1, ws.seg, 1, T, ws.xp, ws.h, 1, nullptr,
                              nullptr, d_out, ws.grouped, ws.grouped_bytes, d_error_flag, true, T,
                              stream, err);
}

// Pointers into a reference blob (header at offset 0) from its parsed meta.
extern "C" WispError wisp_b200_blob_expert(const WispExpertMeta* meta, const void* d_blob,
                                           WispInt4Expert* out, WispErrCtx* err) {
  if (!meta || !d_blob || !out) return WB_FAIL(WISP_ERR_INVALID_ARG, "blob_expert: null pointer");
  if (!meta->valid) return WB_FAIL(WISP_ERR_INVALID_ARG, "blob_expert: meta not valid");
  const uint8_t* base = static_cast<const uint8_t*>(d_blob);
  WispInt4Mat* mats[3] = {&out->gate, &out->up, &out->down};
  for (int m = 0; m < 3; m++) {
    const uint8_t* packed = base + meta->packed_off[m];
    const uint8_t* scales = base + meta->scales_off[m];
    // Zero points are present when bytes remain between zeros_off and the
    // next matrix's packed data (the end of the blob for down).
    const size_t end = m < 2 ? meta->packed_off[m + 1] : meta->total_bytes;
    const uint8_t* zeros = end > meta->zeros_off[m] ? base + meta->zeros_off[m] : nullptr;
    if (((uintptr_t)packed | (uintptr_t)scales | (uintptr_t)zeros) & 15)
      return WB_FAIL(WISP_ERR_INVALID_ARG,
                     "blob_expert: matrix %d data not 16-byte aligned (place the blob at an "
                     "address = 8 mod 16)", m);
    mats[m]->packed = packed;
    mats[m]->scales = reinterpret_cast<const wisp_half*>(scales);
    mats[m]->zeros = reinterpret_cast<const wisp_half*>(zeros);
  }
  return WISP_OK;
}

extern "C" int* wisp_b200_moe_error_word(const WispMoeConfig* cfg, void* d_workspace) {
  if (validate(cfg, nullptr) != WISP_OK || !d_workspace) return nullptr;
  return carve(cfg, d_workspace).error_flag;
}

extern "C" WispError wisp_b200_check_error_flag(const int* d_error_flag, cudaStream_t stream,
                                                WispErrCtx* err) {
  if (!d_error_flag) return WB_FAIL(WISP_ERR_INVALID_ARG, "check_error_flag: null pointer");
  int h = 0;
  WB_CUDA_CHECK(cudaMemcpyAsync(&h, d_error_flag, sizeof(int), cudaMemcpyDeviceToHost, stream));
  WB_CUDA_CHECK(cudaStreamSynchronize(stream));
  if (h) return WB_FAIL(WISP_ERR_TIMEOUT, "a tensor-core kernel gave up waiting (device error word %d)", h);
  return WISP_OK;
}

// Header parse on host memory; semantics of csrc/core/wisp_engine.c:268-303.
extern "C" WispError wisp_b200_parse_expert_header(const void* blob, size_t blob_size,
                                                   WispExpertMeta* meta, WispErrCtx* err) {
  if (!blob || !meta) return WB_FAIL(WISP_ERR_OOM, "NULL pointer: expert_parse_header: blob");
  if (blob_size < sizeof(WispExpertHeader))
    return WB_FAIL(WISP_ERR_MODEL, "expert blob too small: %zu bytes", blob_size);
  WispExpertHeader h;
  memcpy(&h, blob, sizeof h);
  if (h.magic != WISP_EXPERT_MAGIC || h.version != WISP_EXPERT_VERSION || h.n_mats != WISP_EXPERT_NMATS)
    return WB_FAIL(WISP_ERR_MODEL, "expert blob corrupt: magic=%08x version=%u n_mats=%u", h.magic,
                   h.version, h.n_mats);
  size_t off = sizeof(WispExpertHeader);
  for (int m = 0; m < WISP_EXPERT_NMATS; m++) {
    meta->rows[m] = h.mats[m].rows;
    meta->cols[m] = h.mats[m].cols;
    meta->packed_off[m] = off;
    off += h.mats[m].packed_bytes;
    meta->scales_off[m] = off;
    off += h.mats[m].scales_bytes;
    meta->zeros_off[m] = off;
    off += h.mats[m].zeros_bytes;
  }
  meta->group_size = h.group_size;
  meta->total_bytes = off;
  meta->valid = 1;
  if (off > blob_size) {
    meta->valid = 0;
    return WB_FAIL(WISP_ERR_MODEL, "expert blob truncated: needs %zu, have %zu", off, blob_size);
  }
  return WISP_OK;
}

extern "C" const char* wisp_b200_version(void) { return "wisp_b200 0.1.0 (sm_100a)"; }
