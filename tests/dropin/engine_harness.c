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
 */
#include "wisp_engine.c"

#define WISP_B200_NO_ENGINE_TYPES
#include "wisp_b200.h"

typedef struct {
    WispEngine eng;
    LRUCache vram, ram;
    void* blob_mem[1024];
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

void eh_destroy(EngineHarness* h) {
    if (!h) return;
    WispEngine* e = &h->eng;
    if (e->compute_stream) cudaStreamSynchronize(e->compute_stream);
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
