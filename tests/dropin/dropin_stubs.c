/*
 * dropin_stubs.c -- TEST INFRASTRUCTURE ONLY. The reference engine's GPU
 * launchers outside the routed-expert path (attention, MLA, KV append,
 * RoPE, RMSNorm, residual, embedding) are not part of libwisp_b200.so; the
 * drop-in harness never reaches them, so each stub stops the process if it
 * is called. Only their names matter to the linker.
 */
#include <stdio.h>
#include <stdlib.h>

#define STUB(name)                                                          \
    void name(void) {                                                       \
        fprintf(stderr, "engine harness: %s is outside the MoE path\n", #name); \
        abort();                                                            \
    }

STUB(wisp_gpu_attention)
STUB(wisp_gpu_embed_lookup)
STUB(wisp_gpu_kv_append)
STUB(wisp_gpu_mla_absorb_q)
STUB(wisp_gpu_mla_out)
STUB(wisp_gpu_residual_add)
STUB(wisp_gpu_rmsnorm)
STUB(wisp_gpu_rope)
