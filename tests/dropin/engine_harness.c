/*
 * engine_harness.c -- TEST INFRASTRUCTURE ONLY: the drop-in proof.
 *
 * Compiles the reference engine's own csrc/core/wisp_engine.c in place WITH
 * its CUDA branches (no WISP_NO_CUDA) and links it against libwisp_b200.so,
 * which supplies every MoE launcher the engine calls (launch_dequant_expert,
 * wisp_gpu_router_topk, wisp_gpu_swiglu_ffn, wisp_gpu_gemv_f16,
 * wisp_gpu_scale_accum). The launchers outside the MoE path come from
 * dropin_stubs.c and abort if reached.
 *
 * Exported for tests/test_dropin_engine.py (ctypes):
 *   eh_create / eh_destroy      a minimal single-layer engine: config, router,
 *                               optional dense fp16 shared expert, device
 *                               scratch buffers and streams, and a VRAM-tier
 *                               LRU cache holding the routed experts' blobs
 *   eh_put_expert               copy a blob to the device (at 8 mod 16, so its
 *                               packed data is 16-byte aligned) and insert it
 *                               into the VRAM tier under (layer 0, expert e)
 *   eh_run_moe                  the reference's own run_moe (wisp_engine.c:
 *                               1563-1674), full-GPU branch: router on the
 *                               GPU, dense shared expert, then gpu_expert_ffn
 *                               per fetched expert -- the stock chain running
 *                               on this library's drop-in launchers
 *   eh_run_moe_fused            the same layer with the per-expert chain
 *                               replaced by one wisp_b200_expert_ffn call, as
 *                               INTEGRATION.md section 2 describes
 *   eh_prefill_moe              one MoE layer over T prompt tokens at once
 *                               (the batched form of wisp_prefill's per-token
 *                               loop, wisp_engine.c:2292-2307): GPU routing,
 *                               expert residency through the engine's own
 *                               wisp_expert_fetch, slot-wise preparation of
 *                               the layer's weight set whenever a slot's blob
 *                               address changes (promotion / move), then the
 *                               grouped int4 FFN
 *   eh_move_expert              moves a blob to a new VRAM address (as after
 *                               an eviction and a later promotion)
 *   eh_batched_state /          the prepared set, for comparison with a
 *   eh_copy_prepared            whole-table wisp_b200_prepare_experts
 *   eh_dense_mlp_int4           run_dense_mlp (wisp_engine.c:1676-1686) with
 *                               the MLP quantised to int4: one
 *                               wisp_b200_expert_ffn call with weight 1.0
 */
#include "wisp_engine.c"

#define WISP_B200_NO_ENGINE_TYPES
#include "wisp_b200.h"

typedef struct {
    WispEngine eng;
    LRUCache vram, ram;
    void* blob_mem[1024];
    /* batched (prefill) state: the layer's device expert table and its
     * prepared set, kept in step with the VRAM tier slot by slot */
    WispInt4Expert* d_table;
    WispInt4Expert h_table[1024];
    const void* slot_blob[1024];     /* blob address each slot was prepared from */
    void* d_prepared;
    size_t prepared_bytes;
    float* d_bias_f32;
    int slot_prepares;               /* slots (re)prepared so far */
} EngineHarness;

#define EH_CK(call)                                                   \
    do {                                                              \
        if ((call) != cudaSuccess) { eh_destroy(h); return NULL; }    \
    } while (0)

void eh_destroy(EngineHarness* h);

EngineHarness* eh_create(int hidden, int moe_inter, int n_experts, int top_k,
                         int group_size, int shared_inter,
                         const uint16_t* router_w, const uint16_t* router_bias,
                         const uint16_t* sh_gate, const uint16_t* sh_up,
                         const uint16_t* sh_down) {
    EngineHarness* h = (EngineHarness*)calloc(1, sizeof(EngineHarness));
    if (!h) return NULL;
    WispEngine* e = &h->eng;
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    e->cfg.hidden = hidden;
    e->cfg.moe_inter = moe_inter;
    e->cfg.n_experts = n_experts;
    e->cfg.top_k = top_k;
    e->cfg.group_size = group_size;
    e->cfg.shared_inter = shared_inter;
    e->cfg.num_layers = 1;
    e->use_gpu = 1;
    e->experts_on_gpu = 1;
    wisp_mutex_init(&e->stats_mutex);
    if (lru_init(&h->vram, (uint64_t)1 << 40, TIER_VRAM, &err) != WISP_OK ||
        lru_init(&h->ram, (uint64_t)1 << 40, TIER_RAM, &err) != WISP_OK) {
        free(h);
        return NULL;
    }
    e->vram_cache = &h->vram;
    e->ram_cache = &h->ram;
    e->layers = (WispLayerWeights*)calloc(1, sizeof(WispLayerWeights));
    e->expert_meta = (WispExpertMeta*)calloc(1, sizeof(WispExpertMeta));
    if (!e->layers || !e->expert_meta) { eh_destroy(h); return NULL; }
    EH_CK(cudaStreamCreate(&e->compute_stream));
    EH_CK(cudaStreamCreate(&e->transfer_stream));
    const size_t rb = (size_t)n_experts * hidden * 2;
    WispLayerWeights* w = &e->layers[0];
    EH_CK(cudaMalloc((void**)&w->router, rb));
    EH_CK(cudaMemcpy(w->router, router_w, rb, cudaMemcpyHostToDevice));
    if (router_bias) {
        EH_CK(cudaMalloc((void**)&w->router_bias, (size_t)n_experts * 2));
        EH_CK(cudaMemcpy(w->router_bias, router_bias, (size_t)n_experts * 2,
                         cudaMemcpyHostToDevice));
    }
    if (shared_inter > 0) {
        const size_t sb = (size_t)shared_inter * hidden * 2;
        EH_CK(cudaMalloc((void**)&w->shared_gate, sb));
        EH_CK(cudaMalloc((void**)&w->shared_up, sb));
        EH_CK(cudaMalloc((void**)&w->shared_down, sb));
        EH_CK(cudaMemcpy(w->shared_gate, sh_gate, sb, cudaMemcpyHostToDevice));
        EH_CK(cudaMemcpy(w->shared_up, sh_up, sb, cudaMemcpyHostToDevice));
        EH_CK(cudaMemcpy(w->shared_down, sh_down, sb, cudaMemcpyHostToDevice));
        w->shared_inter = shared_inter;
    }
    const int inter_max = moe_inter > shared_inter ? moe_inter : shared_inter;
    EH_CK(cudaMalloc((void**)&e->buf_norm, (size_t)hidden * 4));
    EH_CK(cudaMalloc((void**)&e->buf_ffn, (size_t)hidden * 4));
    EH_CK(cudaMalloc((void**)&e->buf_attn_a, (size_t)hidden * 4));
    EH_CK(cudaMalloc((void**)&e->buf_h, (size_t)inter_max * 4));
    EH_CK(cudaMalloc((void**)&e->buf_router_logits, (size_t)n_experts * 4));
    EH_CK(cudaMalloc((void**)&e->buf_dq_gate, (size_t)moe_inter * hidden * 2));
    EH_CK(cudaMalloc((void**)&e->buf_dq_up, (size_t)moe_inter * hidden * 2));
    EH_CK(cudaMalloc((void**)&e->buf_dq_down, (size_t)moe_inter * hidden * 2));
    EH_CK(cudaHostAlloc((void**)&e->host_topk_idx, 64 * sizeof(int), cudaHostAllocDefault));
    EH_CK(cudaHostAlloc((void**)&e->host_topk_w, 64 * sizeof(float), cudaHostAllocDefault));
    return h;
}

/* Routed expert e's blob into the VRAM tier (its header also fills the
 * layer's expert meta, as the engine does on the first fetch). */
int eh_put_expert(EngineHarness* h, int expert, const void* blob, size_t size) {
    WispEngine* e = &h->eng;
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    if (expert < 0 || expert >= 1024) return WISP_ERR_INVALID_ARG;
    if (!e->expert_meta[0].valid &&
        wisp_expert_parse_header(blob, size, &e->expert_meta[0], &err) != WISP_OK)
        return err.code;
    uint8_t* mem = NULL;
    if (cudaMalloc((void**)&mem, size + 16) != cudaSuccess) return WISP_ERR_CUDA;
    h->blob_mem[expert] = mem;
    uint8_t* dst = mem + ((8 - ((uintptr_t)mem & 15)) & 15);   /* 8 mod 16 */
    if (cudaMemcpy(dst, blob, size, cudaMemcpyHostToDevice) != cudaSuccess) return WISP_ERR_CUDA;
    return lru_put(e->vram_cache, 0, (uint32_t)expert, dst, size, &err);
}

static int eh_io(EngineHarness* h, const float* x, float* out, int* idx, float* wts, int dir) {
    WispEngine* e = &h->eng;
    const size_t n = (size_t)e->cfg.hidden * 4;
    if (dir == 0)
        return cudaMemcpy(e->buf_norm, x, n, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : WISP_ERR_CUDA;
    if (cudaStreamSynchronize(e->compute_stream) != cudaSuccess) return WISP_ERR_CUDA;
    if (cudaMemcpy(out, e->buf_ffn, n, cudaMemcpyDeviceToHost) != cudaSuccess) return WISP_ERR_CUDA;
    for (int k = 0; k < e->cfg.top_k; k++) {
        idx[k] = e->host_topk_idx[k];
        wts[k] = e->host_topk_w[k];
    }
    return 0;
}

/* The reference's run_moe, unmodified, on the drop-in launchers. */
int eh_run_moe(EngineHarness* h, const float* x, float* out, int* idx, float* wts) {
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    int rc = eh_io(h, x, out, idx, wts, 0);
    if (rc) return rc;
    WispError e = run_moe(&h->eng, 0, &err);
    if (e != WISP_OK) return (int)e;
    return eh_io(h, x, out, idx, wts, 1);
}

/* The same layer with the per-expert dequant -> GEMV chain replaced by one
 * fused call: router and shared expert through the engine's own ops, the
 * routed experts fetched from the VRAM tier, then wisp_b200_expert_ffn over
 * all of them with buf_dq_gate as its scratch. */
int eh_run_moe_fused(EngineHarness* h, const float* x, float* out, int* idx, float* wts) {
    WispEngine* eng = &h->eng;
    WispModelConfig* c = &eng->cfg;
    WispLayerWeights* w = &eng->layers[0];
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    int rc = eh_io(h, x, out, idx, wts, 0);
    if (rc) return rc;
    wisp_gpu_router_topk(w->router, w->router_bias, eng->buf_norm, eng->buf_router_logits,
                         c->n_experts, c->hidden, c->top_k, eng->host_topk_idx,
                         eng->host_topk_w, eng->compute_stream);
    if (cudaStreamSynchronize(eng->compute_stream) != cudaSuccess) return WISP_ERR_CUDA;
    cudaMemsetAsync(eng->buf_ffn, 0, (size_t)c->hidden * 4, eng->compute_stream);
    if (w->shared_gate) {
        op_swiglu_ffn(eng, w->shared_gate, w->shared_up, eng->buf_norm, eng->buf_h,
                      w->shared_inter, c->hidden);
        op_gemv(eng, w->shared_down, eng->buf_h, eng->buf_attn_a, c->hidden, w->shared_inter);
        op_scale_accum(eng, eng->buf_ffn, eng->buf_attn_a, 1.0f, c->hidden);
    }
    const void* blobs[64];
    float wsel[64];
    int nb = 0;
    for (int k = 0; k < c->top_k && k < 64; k++) {
        const int e = eng->host_topk_idx[k];
        if (e < 0) continue;
        void* b = wisp_expert_fetch(eng, 0, (uint32_t)e, &err);
        if (!b) return err.code ? (int)err.code : WISP_ERR_EXPERT_MISS;
        blobs[nb] = b;
        wsel[nb] = eng->host_topk_w[k];
        nb++;
    }
    if (nb > 0) {
        WispError e = wisp_b200_expert_ffn(&eng->expert_meta[0], blobs, wsel, nb, eng->buf_norm,
                                           eng->buf_ffn, eng->buf_dq_gate,
                                           (size_t)c->moe_inter * c->hidden * 2,
                                           eng->compute_stream, &err);
        if (e != WISP_OK) return (int)e;
    }
    return eh_io(h, x, out, idx, wts, 1);
}

/* Moves routed expert e's blob to a new device address (another VRAM slot,
 * as after an eviction and a later promotion): new allocation at 8 mod 16,
 * device-to-device copy, the tier's node replaced, the old memory freed. */
int eh_move_expert(EngineHarness* h, int expert) {
    WispEngine* e = &h->eng;
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    if (expert < 0 || expert >= 1024 || !h->blob_mem[expert]) return WISP_ERR_INVALID_ARG;
    LRUNode* node = lru_get(e->vram_cache, 0, (uint32_t)expert);
    if (!node) return WISP_ERR_EXPERT_MISS;
    const size_t size = node->size_bytes;
    uint8_t* mem = NULL;
    if (cudaMalloc((void**)&mem, size + 16) != cudaSuccess) return WISP_ERR_CUDA;
    uint8_t* dst = mem + ((8 - ((uintptr_t)mem & 15)) & 15);
    if (cudaMemcpy(dst, node->data_ptr, size, cudaMemcpyDeviceToDevice) != cudaSuccess)
        return WISP_ERR_CUDA;
    lru_remove(e->vram_cache, node);
    lru_node_free(node);
    cudaFree(h->blob_mem[expert]);
    h->blob_mem[expert] = mem;
    return lru_put(e->vram_cache, 0, (uint32_t)expert, dst, size, &err);
}

/* The batched layer's configuration for T tokens: the engine's softmax
 * router over fp16 weights (the reference's router ABI). */
static WispMoeConfig eh_cfg(EngineHarness* h, int T) {
    WispModelConfig* c = &h->eng.cfg;
    WispMoeConfig cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.tokens = T;
    cfg.hidden = c->hidden;
    cfg.inter = c->moe_inter;
    cfg.n_experts = c->n_experts;
    cfg.top_k = c->top_k;
    cfg.group_size = c->group_size;
    cfg.scoring = WISP_SCORE_SOFTMAX;
    cfg.router_fp16 = 1;
    return cfg;
}

static int eh_batched_init(EngineHarness* h) {
    if (h->d_table) return 0;
    WispEngine* e = &h->eng;
    WispModelConfig* c = &e->cfg;
    WispMoeConfig cfg = eh_cfg(h, 1);
    const int E = c->n_experts;
    h->prepared_bytes = wisp_b200_prepared_bytes(&cfg, E);
    if (!h->prepared_bytes) return WISP_ERR_INVALID_ARG;
    if (cudaMalloc((void**)&h->d_table, sizeof(WispInt4Expert) * E) != cudaSuccess ||
        cudaMalloc(&h->d_prepared, h->prepared_bytes) != cudaSuccess ||
        cudaMemset(h->d_table, 0, sizeof(WispInt4Expert) * E) != cudaSuccess ||
        cudaMemset(h->d_prepared, 0, h->prepared_bytes) != cudaSuccess)
        return WISP_ERR_CUDA;
    /* The batched router adds an fp32 bias; the engine holds fp16. */
    WispLayerWeights* w = &e->layers[0];
    if (w->router_bias) {
        uint16_t hb[1024];
        float fb[1024];
        if (cudaMemcpy(hb, w->router_bias, (size_t)E * 2, cudaMemcpyDeviceToHost) != cudaSuccess)
            return WISP_ERR_CUDA;
        for (int i = 0; i < E; i++) fb[i] = wisp_half_to_float(hb[i]);
        if (cudaMalloc((void**)&h->d_bias_f32, (size_t)E * 4) != cudaSuccess ||
            cudaMemcpy(h->d_bias_f32, fb, (size_t)E * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return WISP_ERR_CUDA;
    }
    return 0;
}

/* One MoE layer over T prompt tokens at once -- the batched replacement of
 * the per-token loop of wisp_prefill (wisp_engine.c:2292-2307) for the MoE
 * part of a layer. x: T x hidden fp32 values that bf16 represents exactly
 * (the batched entry takes bf16 rows). Steps:
 *   1. route all T tokens on the GPU (wisp_b200_route), one host sync;
 *   2. fetch every touched expert through the engine's own tier path
 *      (wisp_expert_fetch); a slot whose blob address changed since it was
 *      last prepared (a promotion into VRAM, or a move after an eviction)
 *      is re-prepared in place (wisp_b200_blob_expert +
 *      wisp_b200_prepare_expert_slot) and its table entry updated;
 *   3. dispatch plan, row pack and the grouped int4 FFN with the weighted
 *      combine (mode 0) into out.
 * idx / wts receive the routing (T x top_k). */
int eh_prefill_moe(EngineHarness* h, const float* x, int T, float* out, int* idx, float* wts) {
    WispEngine* e = &h->eng;
    WispModelConfig* c = &e->cfg;
    WispLayerWeights* w = &e->layers[0];
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    int rc = eh_batched_init(h);
    if (rc) return rc;
    const int M = c->hidden, I = c->moe_inter, E = c->n_experts, k = c->top_k;
    WispMoeConfig cfg = eh_cfg(h, T);
    cudaStream_t st = e->compute_stream;
    const size_t R = (size_t)T * k;
    uint16_t* xb = (uint16_t*)malloc((size_t)T * M * 2);
    uint16_t *d_x = NULL, *d_xp = NULL, *d_h = NULL;
    float *d_logits = NULL, *d_w = NULL, *d_rw = NULL, *d_out = NULL;
    int *d_idx = NULL, *d_counts = NULL, *d_rt = NULL, *d_flag = NULL;
    WispSegment* d_segs = NULL;
    void* d_ws = NULL;
    const size_t wsb = wisp_b200_grouped_workspace_bytes(&cfg, E, (int)R);
    rc = WISP_ERR_CUDA;
    if (!xb || !wsb) { rc = WISP_ERR_INVALID_ARG; goto done; }
    for (size_t i = 0; i < (size_t)T * M; i++) {
        uint32_t u;
        memcpy(&u, &x[i], 4);
        xb[i] = (uint16_t)(u >> 16);   /* exact for bf16-representable values */
    }
    if (cudaMalloc((void**)&d_x, (size_t)T * M * 2) || cudaMalloc((void**)&d_logits, (size_t)T * E * 4) ||
        cudaMalloc((void**)&d_idx, R * 4) || cudaMalloc((void**)&d_w, R * 4) ||
        cudaMalloc((void**)&d_counts, (size_t)E * 4) ||
        cudaMalloc((void**)&d_segs, sizeof(WispSegment) * E) || cudaMalloc((void**)&d_rt, R * 4) ||
        cudaMalloc((void**)&d_rw, R * 4) || cudaMalloc((void**)&d_xp, R * M * 2) ||
        cudaMalloc((void**)&d_h, R * I * 2) || cudaMalloc((void**)&d_out, (size_t)T * M * 4) ||
        cudaMalloc((void**)&d_flag, 4) || cudaMalloc(&d_ws, wsb))
        goto done;
    if (cudaMemcpy(d_x, xb, (size_t)T * M * 2, cudaMemcpyHostToDevice) || cudaMemset(d_flag, 0, 4))
        goto done;
    /* 1. routing */
    WispMoeWeights mw;
    mw.router_w = (const uint16_t*)w->router;
    mw.router_bias = h->d_bias_f32;
    mw.experts = h->d_table;
    mw.prepared = h->d_prepared;
    if ((rc = wisp_b200_route(&cfg, &mw, d_x, d_logits, d_idx, d_w, st, &err))) goto done;
    if (cudaMemcpyAsync(idx, d_idx, R * 4, cudaMemcpyDeviceToHost, st) ||
        cudaMemcpyAsync(wts, d_w, R * 4, cudaMemcpyDeviceToHost, st) || cudaStreamSynchronize(st)) {
        rc = WISP_ERR_CUDA;
        goto done;
    }
    /* 2. residency through the engine's tiers; slots follow the blobs */
    {
        unsigned char touched[1024] = {0};
        for (size_t i = 0; i < R; i++)
            if (idx[i] >= 0 && idx[i] < E) touched[idx[i]] = 1;
        for (int x_e = 0; x_e < E; x_e++) {
            if (!touched[x_e]) continue;
            void* b = wisp_expert_fetch(e, 0, (uint32_t)x_e, &err);
            if (!b) { rc = err.code ? (int)err.code : WISP_ERR_EXPERT_MISS; goto done; }
            if (b == h->slot_blob[x_e]) continue;
            WispInt4Expert ent;
            if ((rc = wisp_b200_blob_expert(&e->expert_meta[0], b, &ent, &err))) goto done;
            if ((rc = wisp_b200_prepare_expert_slot(&cfg, E, x_e, &ent, h->d_prepared,
                                                    h->prepared_bytes, st, &err)))
                goto done;
            h->h_table[x_e] = ent;
            if (cudaMemcpyAsync(h->d_table + x_e, &h->h_table[x_e], sizeof ent,
                                cudaMemcpyHostToDevice, st)) {
                rc = WISP_ERR_CUDA;
                goto done;
            }
            h->slot_blob[x_e] = b;
            h->slot_prepares++;
        }
    }
    /* 3. dispatch plan, row pack, grouped FFN with the weighted combine */
    if ((rc = wisp_b200_dispatch_plan(&cfg, d_idx, d_w, d_counts, d_segs, d_rt, d_rw, st, &err)))
        goto done;
    if ((rc = wisp_b200_pack_rows(d_x, d_rt, (int)R, M, d_xp, st, &err))) goto done;
    if (cudaMemsetAsync(d_out, 0, (size_t)T * M * 4, st)) { rc = WISP_ERR_CUDA; goto done; }
    if ((rc = wisp_b200_grouped_ffn(&cfg, h->d_prepared, h->d_table, E, d_segs, E, (int)R, d_xp,
                                    d_h, 0, d_rt, d_rw, d_out, d_ws, wsb, d_flag, st, &err)))
        goto done;
    if ((rc = wisp_b200_check_error_flag(d_flag, st, &err))) goto done;
    rc = cudaMemcpy(out, d_out, (size_t)T * M * 4, cudaMemcpyDeviceToHost) ? WISP_ERR_CUDA : 0;
done:
    if (rc)   /* the failing step, for the test log */
        fprintf(stderr, "eh_prefill_moe: error %d: %s (last CUDA error: %s)\n", rc, err.message,
                cudaGetErrorString(cudaGetLastError()));
    cudaStreamSynchronize(st);
    free(xb);
    cudaFree(d_x); cudaFree(d_logits); cudaFree(d_idx); cudaFree(d_w); cudaFree(d_counts);
    cudaFree(d_segs); cudaFree(d_rt); cudaFree(d_rw); cudaFree(d_xp); cudaFree(d_h);
    cudaFree(d_out); cudaFree(d_flag); cudaFree(d_ws);
    return rc;
}

/* The batched state for the tests: device table, prepared set and its size,
 * and how many slot preparations have run. */
int eh_batched_state(EngineHarness* h, void** d_table, void** d_prepared, size_t* bytes) {
    *d_table = h->d_table;
    *d_prepared = h->d_prepared;
    *bytes = h->prepared_bytes;
    return h->slot_prepares;
}

/* Copies the prepared set to host memory (bytes from eh_batched_state). */
int eh_copy_prepared(EngineHarness* h, void* host_dst) {
    if (!h->d_prepared) return WISP_ERR_INVALID_ARG;
    return cudaMemcpy(host_dst, h->d_prepared, h->prepared_bytes, cudaMemcpyDeviceToHost)
               ? WISP_ERR_CUDA : 0;
}

/* An int4 dense MLP (or int4 shared expert) for one token at reference
 * precision: out = mlp(x) through wisp_b200_expert_ffn with the MLP's blob
 * as the one expert and weight 1.0 -- the int4 form of run_dense_mlp
 * (wisp_engine.c:1676-1686), whose stock form runs fp16 weights through
 * op_swiglu_ffn + op_gemv. */
int eh_dense_mlp_int4(EngineHarness* h, const void* blob, size_t size, const float* x, float* out) {
    WispEngine* e = &h->eng;
    WispErrCtx err;
    memset(&err, 0, sizeof err);
    WispExpertMeta meta;
    memset(&meta, 0, sizeof meta);
    if (wisp_expert_parse_header(blob, size, &meta, &err) != WISP_OK) return err.code;
    uint8_t* mem = NULL;
    int rc = WISP_ERR_CUDA;
    if (cudaMalloc((void**)&mem, size + 16) != cudaSuccess) return WISP_ERR_CUDA;
    uint8_t* dst = mem + ((8 - ((uintptr_t)mem & 15)) & 15);
    const void* blobs[1] = {dst};
    const float one = 1.0f;
    const size_t n = (size_t)meta.cols[0] * 4;   /* hidden */
    if (cudaMemcpy(dst, blob, size, cudaMemcpyHostToDevice) ||
        cudaMemcpy(e->buf_norm, x, n, cudaMemcpyHostToDevice) ||
        cudaMemsetAsync(e->buf_ffn, 0, n, e->compute_stream))
        goto done;
    rc = wisp_b200_expert_ffn(&meta, blobs, &one, 1, e->buf_norm, e->buf_ffn, e->buf_dq_gate,
                              (size_t)e->cfg.moe_inter * e->cfg.hidden * 2, e->compute_stream, &err);
    if (rc) goto done;
    rc = (cudaStreamSynchronize(e->compute_stream) ||
          cudaMemcpy(out, e->buf_ffn, n, cudaMemcpyDeviceToHost)) ? WISP_ERR_CUDA : 0;
done:
    cudaStreamSynchronize(e->compute_stream);
    cudaFree(mem);
    return rc;
}

void eh_destroy(EngineHarness* h) {
    if (!h) return;
    WispEngine* e = &h->eng;
    if (e->compute_stream) cudaStreamSynchronize(e->compute_stream);
    cudaFree(h->d_table);
    cudaFree(h->d_prepared);
    cudaFree(h->d_bias_f32);
    for (int i = 0; i < 1024; i++)
        if (h->blob_mem[i]) cudaFree(h->blob_mem[i]);
    if (e->layers) {
        WispLayerWeights* w = &e->layers[0];
        cudaFree(w->router);
        cudaFree(w->router_bias);
        cudaFree(w->shared_gate);
        cudaFree(w->shared_up);
        cudaFree(w->shared_down);
        free(e->layers);
    }
    free(e->expert_meta);
    cudaFree(e->buf_norm);
    cudaFree(e->buf_ffn);
    cudaFree(e->buf_attn_a);
    cudaFree(e->buf_h);
    cudaFree(e->buf_router_logits);
    cudaFree(e->buf_dq_gate);
    cudaFree(e->buf_dq_up);
    cudaFree(e->buf_dq_down);
    if (e->host_topk_idx) cudaFreeHost(e->host_topk_idx);
    if (e->host_topk_w) cudaFreeHost(e->host_topk_w);
    if (e->compute_stream) cudaStreamDestroy(e->compute_stream);
    if (e->transfer_stream) cudaStreamDestroy(e->transfer_stream);
    lru_destroy(&h->vram);
    lru_destroy(&h->ram);
    free(h);
}
