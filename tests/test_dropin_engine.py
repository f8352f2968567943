"""The drop-in proof: the reference engine's own GPU code linked against
libwisp_b200.so.

tests/dropin/engine_harness.c compiles the reference's csrc/core/wisp_engine.c
in place with its CUDA branches, so its run_moe (wisp_engine.c:1563-1674)
runs unmodified on this library's drop-in launchers: the router
(wisp_gpu_router_topk), the dense fp16 shared expert (wisp_gpu_swiglu_ffn,
wisp_gpu_gemv_f16, wisp_gpu_scale_accum) and, per routed expert fetched from
the engine's VRAM-tier LRU, gpu_expert_ffn's dequant -> SwiGLU GEMV -> GEMV ->
scale-accumulate chain (launch_dequant_expert and the same launchers). A
second run replaces that per-expert chain with one wisp_b200_expert_ffn call
over all fetched experts, as INTEGRATION.md section 2 describes.

Both runs are checked against the reference's own compiled CPU code on the
same inputs: routing indices from its cpu_router_topk exactly, and outputs
against its cpu_expert_ffn for the routed experts plus an fp64 dense shared
expert. The stock chain rounds each dequantised weight to fp16 (as the
reference's dequant kernel does), so it is held to the parity tolerance; the
fused path keeps the weights exact and is held to 1e-5.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from helpers import assert_close
from wisp_b200.blob import Int4Matrix, pack_blob

pytestmark = pytest.mark.gpu

HARNESS = Path(__file__).resolve().parent / "dropin" / "_build" / "libengine_harness.so"

_P = C.c_void_p


def _load():
    if not HARNESS.exists():
        pytest.skip(f"{HARNESS} not built (needs the reference sources at build time)")
    L = C.CDLL(str(HARNESS))
    L.eh_create.restype = _P
    L.eh_create.argtypes = [C.c_int] * 6 + [_P] * 5
    L.eh_put_expert.restype = C.c_int
    L.eh_put_expert.argtypes = [_P, C.c_int, _P, C.c_size_t]
    for f in (L.eh_run_moe, L.eh_run_moe_fused):
        f.restype = C.c_int
        f.argtypes = [_P] * 5
    L.eh_destroy.argtypes = [_P]
    return L


def _ptr(a):
    return a.ctypes.data


def test_reference_run_moe_on_dropin_launchers_and_fused_entry(orc):
    import torch  # noqa: F401  (initialises the CUDA runtime the same way the other tests do)
    from oracle.oracle import RefCPU

    L = _load()
    ref = RefCPU()
    rng = np.random.default_rng(31)
    M, I, E, k, gs, SI = 256, 128, 8, 2, 64, 64

    def mat(rows, cols):
        n = rows * cols
        return Int4Matrix(rng.integers(0, 256, n // 2, dtype=np.uint8),
                          np.float16(rng.uniform(0.004, 0.02, n // gs)).view(np.uint16),
                          np.float16(rng.uniform(-0.01, 0.01, n // gs)).view(np.uint16), rows, cols)

    mats = [[mat(I, M), mat(I, M), mat(M, I)] for _ in range(E)]
    blobs = [np.frombuffer(pack_blob(*m, group_size=gs), np.uint8).copy() for m in mats]
    router = np.float16(rng.standard_normal((E, M)) * 0.05).view(np.uint16)
    bias = np.float16(rng.standard_normal(E) * 0.1).view(np.uint16)
    sg = np.float16(rng.standard_normal((SI, M)) * 0.05)
    su = np.float16(rng.standard_normal((SI, M)) * 0.05)
    sd = np.float16(rng.standard_normal((M, SI)) * 0.05)

    h = L.eh_create(M, I, E, k, gs, SI, _ptr(router), _ptr(bias), _ptr(sg.view(np.uint16)),
                    _ptr(su.view(np.uint16)), _ptr(sd.view(np.uint16)))
    assert h, "engine harness set-up failed"
    try:
        for e in range(E):
            assert L.eh_put_expert(h, e, _ptr(blobs[e]), blobs[e].size) == 0
        for t in range(6):
            x = rng.standard_normal(M).astype(np.float32)
            # the reference's own CPU results for this token
            idx_ref, w_ref = ref.router_topk(router, bias, x, k)
            want = np.zeros(M, np.float32)
            for j in range(k):
                ref.expert_ffn(blobs[idx_ref[j]].tobytes(), x, want, float(w_ref[j]))
            xs = x.astype(np.float64)
            g = sg.astype(np.float64) @ xs
            u = su.astype(np.float64) @ xs
            want = want.astype(np.float64) + sd.astype(np.float64) @ (g / (1 + np.exp(-g)) * u)

            for name, fn, tol in (("stock run_moe", L.eh_run_moe, None),
                                  ("fused entry", L.eh_run_moe_fused, 1e-5)):
                out = np.empty(M, np.float32)
                idx = np.empty(k, np.int32)
                w = np.empty(k, np.float32)
                assert fn(h, _ptr(x), _ptr(out), _ptr(idx), _ptr(w)) == 0, name
                np.testing.assert_array_equal(idx, idx_ref, err_msg=f"{name} token {t}")
                np.testing.assert_allclose(w, w_ref, rtol=1e-5, err_msg=f"{name} token {t}")
                if tol is None:
                    assert_close(out, want, what=f"{name} token {t}")
                else:
                    assert_close(out, want, tol, tol, what=f"{name} token {t}")
    finally:
        L.eh_destroy(h)
