/*
 * ref_harness.c -- TEST INFRASTRUCTURE ONLY (never linked into the product).
 *
 * Compiles the reference engine's own CPU hot-path functions in place (the
 * Makefile beside this file adds the reference's csrc/core directory to the
 * include path) and exports them under ref_* names so the parity tests and
 * the bench's CPU-baseline / reference arm can call them through ctypes.
 *
 * Functions exported and the reference code they run (file:line within the
 * reference project):
 *   ref_gemv_int4       -> cpu_gemv_int4        csrc/core/wisp_engine.c:822-845
 *   ref_gemv_f16        -> cpu_gemv_f16         csrc/core/wisp_engine.c:630-645
 *   ref_swiglu          -> cpu_swiglu           csrc/core/wisp_engine.c:677-686
 *   ref_scale_accum     -> cpu_scale_accum      csrc/core/wisp_engine.c:688-690
 *   ref_router_topk     -> cpu_router_topk      csrc/core/wisp_engine.c:782-818
 *   ref_parse_header    -> wisp_expert_parse_header  csrc/core/wisp_engine.c:268-303
 *   ref_expert_ffn      -> cpu_expert_ffn       csrc/core/wisp_engine.c:1535-1561
 *   ref_moe_token       -> the CPU branch of run_moe (csrc/core/wisp_engine.c:1563-1645):
 *                          router, zeroed accumulator, shared expert with weight 1.0,
 *                          then every selected routed expert.
 *
 * Two builds are made from the same harness: the scalar/OpenMP build (the
 * numerically correct path and parity oracle) and the reference's own AVX-512
 * flags (timed only; its AVX-512 branches produce wrong results).
 */
#include "wisp_engine.c"

#include <stdlib.h>

void ref_gemv_int4(const uint8_t* packed, const uint16_t* scales,
                   const uint16_t* zeros, const float* x, float* y,
                   int rows, int cols, int gs) {
    cpu_gemv_int4(packed, scales, zeros, x, y, rows, cols, gs);
}

void ref_gemv_f16(const uint16_t* W, const float* x, float* y, int rows,
                  int cols) {
    cpu_gemv_f16((const wisp_half*)W, x, y, rows, cols);
}

void ref_swiglu(const float* g, const float* u, float* o, int n) {
    cpu_swiglu(g, u, o, n);
}

void ref_scale_accum(float* acc, const float* x, float w, int n) {
    cpu_scale_accum(acc, x, w, n);
}

void ref_router_topk(const uint16_t* W, const uint16_t* bias, const float* x,
                     float* logits, int n_experts, int hidden, int top_k,
                     int* out_idx, float* out_w) {
    cpu_router_topk((const wisp_half*)W, (const wisp_half*)bias, x, logits,
                    n_experts, hidden, top_k, out_idx, out_w);
}

/* Returns WispError; fills meta_out[0..] with packed/scales/zeros offsets,
 * rows, cols (3 each), group_size and total_bytes as int64 values. */
int ref_parse_header(const void* blob, size_t size, int64_t* meta_out) {
    WispExpertMeta m;
    WispErrCtx err;
    memset(&m, 0, sizeof m);
    memset(&err, 0, sizeof err);
    WispError e = wisp_expert_parse_header(blob, size, &m, &err);
    if (e != WISP_OK) return (int)e;
    for (int i = 0; i < 3; i++) {
        meta_out[i] = (int64_t)m.packed_off[i];
        meta_out[3 + i] = (int64_t)m.scales_off[i];
        meta_out[6 + i] = (int64_t)m.zeros_off[i];
        meta_out[9 + i] = (int64_t)m.rows[i];
        meta_out[12 + i] = (int64_t)m.cols[i];
    }
    meta_out[15] = (int64_t)m.group_size;
    meta_out[16] = (int64_t)m.total_bytes;
    return 0;
}

/* A minimal engine object that carries exactly the fields cpu_expert_ffn
 * reads: the layer's expert meta and the host scratch vectors. */
typedef struct {
    WispEngine eng;
    WispExpertMeta meta;
    int inter, hidden;
} RefCtx;

static RefCtx* ref_ctx_make(const void* blob, size_t size) {
    RefCtx* c = (RefCtx*)calloc(1, sizeof(RefCtx));
    if (!c) return NULL;
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    if (wisp_expert_parse_header(blob, size, &c->meta, &err) != WISP_OK) {
        free(c);
        return NULL;
    }
    c->inter = (int)c->meta.rows[0];
    c->hidden = (int)c->meta.cols[0];
    c->eng.expert_meta = &c->meta;
    c->eng.hs_gate = (float*)calloc((size_t)c->inter, 4);
    c->eng.hs_up = (float*)calloc((size_t)c->inter, 4);
    c->eng.hs_h = (float*)calloc((size_t)c->inter, 4);
    c->eng.hs_y = (float*)calloc((size_t)c->hidden, 4);
    return c;
}

static void ref_ctx_free(RefCtx* c) {
    if (!c) return;
    free(c->eng.hs_gate);
    free(c->eng.hs_up);
    free(c->eng.hs_h);
    free(c->eng.hs_y);
    free(c);
}

/* acc[hidden] += weight * expert(x) for one expert blob (header included). */
int ref_expert_ffn(const void* blob, size_t size, const float* x, float* acc,
                   float weight) {
    RefCtx* c = ref_ctx_make(blob, size);
    if (!c) return (int)WISP_ERR_MODEL;
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    WispError e = cpu_expert_ffn(&c->eng, 0, (void*)blob, x, acc, weight, &err);
    ref_ctx_free(c);
    return (int)e;
}

/* One token through the CPU branch of run_moe: route, zero, shared expert
 * (weight 1.0; the blob pointer may be NULL for no shared expert), then the
 * top_k routed experts. `blobs[e]` points at routed expert e's blob. All
 * blobs share one shape (one layer). */
int ref_moe_token(const uint16_t* router_w, const uint16_t* router_bias,
                  const float* x, int n_experts, int top_k,
                  const void* const* blobs, size_t blob_size,
                  const void* shared_blob, float* out, int* out_idx,
                  float* out_w) {
    RefCtx* c = ref_ctx_make(blobs[0], blob_size);
    if (!c) return (int)WISP_ERR_MODEL;
    float* logits = (float*)calloc((size_t)n_experts, 4);
    cpu_router_topk((const wisp_half*)router_w, (const wisp_half*)router_bias,
                    x, logits, n_experts, c->hidden, top_k, out_idx, out_w);
    memset(out, 0, (size_t)c->hidden * 4);
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    WispError e = WISP_OK;
    if (shared_blob)
        e = cpu_expert_ffn(&c->eng, 0, (void*)shared_blob, x, out, 1.0f, &err);
    for (int k = 0; k < top_k && e == WISP_OK; k++) {
        if (out_idx[k] < 0) continue;
        e = cpu_expert_ffn(&c->eng, 0, (void*)blobs[out_idx[k]], x, out,
                           out_w[k], &err);
    }
    free(logits);
    ref_ctx_free(c);
    return (int)e;
}

/* Host fp16 conversion exactly as the reference engine does it. */
float ref_half_to_float(uint16_t h) { return wisp_half_to_float(h); }

int ref_omp_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Thread count of the OpenMP regions the calling thread starts next. A
 * launcher such as torch.distributed.run exports OMP_NUM_THREADS=1, which
 * the OpenMP runtime reads once when it loads; the timed CPU paths call
 * this so they use the host cores they were given whatever the launcher
 * set. */
void ref_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
