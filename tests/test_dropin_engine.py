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
    L.eh_prefill_moe.restype = C.c_int
    L.eh_prefill_moe.argtypes = [_P, _P, C.c_int, _P, _P, _P]
    L.eh_move_expert.restype = C.c_int
    L.eh_move_expert.argtypes = [_P, C.c_int]
    L.eh_batched_state.restype = C.c_int
    L.eh_batched_state.argtypes = [_P, C.POINTER(_P), C.POINTER(_P), C.POINTER(C.c_size_t)]
    L.eh_copy_prepared.restype = C.c_int
    L.eh_copy_prepared.argtypes = [_P, _P]
    L.eh_dense_mlp_int4.restype = C.c_int
    L.eh_dense_mlp_int4.argtypes = [_P, _P, C.c_size_t, _P, _P]
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


def _bf16_exact(rng, shape):
    """float32 values that bf16 represents exactly (the batched entry's input
    format), so the per-token reference sees the same activations."""
    v = rng.standard_normal(shape).astype(np.float32)
    return (v.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


def _ref_margins(router16, bias16, x, k):
    """Gap between the k-th and (k+1)-th logit per token (fp64)."""
    W = router16.view(np.float16).astype(np.float64)
    lg = x.astype(np.float64) @ W.T + bias16.view(np.float16).astype(np.float64)
    s = -np.sort(-lg, axis=1)
    return s[:, k - 1] - s[:, k]


def test_batched_prefill_layer_through_engine_tiers():
    """The batched replacement of wisp_prefill's per-token loop for one MoE
    layer, run inside the reference engine: routing of all prompt tokens at
    once, expert residency through the engine's own tier fetch, slot-wise
    preparation that follows each blob's VRAM address, the grouped int4 FFN.
    Checked per token against the reference's own CPU router and expert FFN
    (reference blobs with zero points), at a prompt length that keeps every
    segment on the register path (48 tokens) and one that puts them on
    tcgen05 (300); then the prepared set against a whole-table preparation,
    and again after two blobs moved to new VRAM addresses."""
    import torch
    from oracle.oracle import RefCPU
    from wisp_b200 import abi

    L = _load()
    ref = RefCPU()
    rng = np.random.default_rng(57)
    M, I, E, k, gs = 512, 256, 16, 4, 128

    def mat(rows, cols):
        n = rows * cols
        return Int4Matrix(rng.integers(0, 256, n // 2, dtype=np.uint8),
                          np.float16(rng.uniform(0.004, 0.02, n // gs)).view(np.uint16),
                          np.float16(rng.uniform(-0.01, 0.01, n // gs)).view(np.uint16), rows, cols)

    blobs = [np.frombuffer(pack_blob(mat(I, M), mat(I, M), mat(M, I), group_size=gs), np.uint8).copy()
             for _ in range(E)]
    router = np.float16(rng.standard_normal((E, M)) * 0.05).view(np.uint16)
    bias = np.float16(rng.standard_normal(E) * 0.1).view(np.uint16)
    h = L.eh_create(M, I, E, k, gs, 0, _ptr(router), _ptr(bias), None, None, None)
    assert h, "engine harness set-up failed"
    d_tab, d_prep, nbytes = _P(), _P(), C.c_size_t()
    try:
        for e in range(E):
            assert L.eh_put_expert(h, e, _ptr(blobs[e]), blobs[e].size) == 0

        def prefill(x):
            T = x.shape[0]
            out = np.empty((T, M), np.float32)
            idx = np.empty((T, k), np.int32)
            w = np.empty((T, k), np.float32)
            assert L.eh_prefill_moe(h, _ptr(x), T, _ptr(out), _ptr(idx), _ptr(w)) == 0
            return out, idx, w

        for T in (48, 300):
            x = _bf16_exact(rng, (T, M))
            out, idx, w = prefill(x)
            margin = _ref_margins(router, bias, x, k)
            tokens = range(T) if T <= 48 else range(0, T, 7)
            for t in tokens:
                idx_ref, w_ref = ref.router_topk(router, bias, x[t], k)
                if margin[t] >= 1e-4:
                    np.testing.assert_array_equal(idx[t], idx_ref, err_msg=f"T={T} token {t}")
                    np.testing.assert_allclose(w[t], w_ref, rtol=1e-4, err_msg=f"T={T} token {t}")
                want = np.zeros(M, np.float32)
                for j in range(k):   # the reference CPU FFN under the batched routing
                    ref.expert_ffn(blobs[idx[t, j]].tobytes(), x[t], want, float(w[t, j]))
                assert_close(out[t], want, what=f"prefill T={T} token {t}")
            prepares = L.eh_batched_state(h, C.byref(d_tab), C.byref(d_prep), C.byref(nbytes))
            assert prepares == len(np.unique(idx)) or T > 48

        # every expert is resident and prepared: the slot-built set equals a
        # whole-table preparation over the same table
        def check_whole_set():
            got = np.empty(nbytes.value, np.uint8)
            assert L.eh_copy_prepared(h, _ptr(got)) == 0
            cfg = abi.WispMoeConfig(tokens=1, hidden=M, inter=I, n_experts=E, top_k=k,
                                    group_size=gs, router_fp16=1)
            fresh = torch.zeros(nbytes.value, dtype=torch.uint8, device="cuda")
            abi.call("wisp_b200_prepare_experts", C.byref(cfg), d_tab.value, E, fresh.data_ptr(),
                     nbytes.value, torch.cuda.current_stream().cuda_stream)
            np.testing.assert_array_equal(got, fresh.cpu().numpy())

        prepares = L.eh_batched_state(h, C.byref(d_tab), C.byref(d_prep), C.byref(nbytes))
        assert prepares == E
        check_whole_set()
        out1, idx1, _ = prefill(x)
        assert L.eh_batched_state(h, C.byref(d_tab), C.byref(d_prep), C.byref(nbytes)) == E
        for e in (3, 11):
            assert L.eh_move_expert(h, e) == 0
        out2, idx2, _ = prefill(x)
        assert L.eh_batched_state(h, C.byref(d_tab), C.byref(d_prep), C.byref(nbytes)) == E + 2
        check_whole_set()
        np.testing.assert_array_equal(idx2, idx1)
        assert_close(out2, out1, 1e-5, 1e-6, "after two blobs moved")
    finally:
        L.eh_destroy(h)


def test_int4_dense_mlp_on_engine():
    """run_dense_mlp with the MLP quantised to int4 (a reference blob with zero
    points), through wisp_b200_expert_ffn with weight 1.0 inside the engine,
    against the reference's own CPU expert FFN on the same blob."""
    import torch  # noqa: F401
    from oracle.oracle import RefCPU

    L = _load()
    ref = RefCPU()
    rng = np.random.default_rng(8)
    M, I, E, k, gs, DI = 512, 256, 4, 2, 64, 384

    def mat(rows, cols):
        n = rows * cols
        return Int4Matrix(rng.integers(0, 256, n // 2, dtype=np.uint8),
                          np.float16(rng.uniform(0.004, 0.02, n // gs)).view(np.uint16),
                          np.float16(rng.uniform(-0.01, 0.01, n // gs)).view(np.uint16), rows, cols)

    dense = np.frombuffer(pack_blob(mat(DI, M), mat(DI, M), mat(M, DI), group_size=gs),
                          np.uint8).copy()
    router = np.float16(rng.standard_normal((E, M)) * 0.05).view(np.uint16)
    h = L.eh_create(M, DI, E, k, gs, 0, _ptr(router), None, None, None, None)
    assert h, "engine harness set-up failed"
    try:
        for t in range(3):
            x = rng.standard_normal(M).astype(np.float32)
            out = np.empty(M, np.float32)
            assert L.eh_dense_mlp_int4(h, _ptr(dense), dense.size, _ptr(x), _ptr(out)) == 0
            want = np.zeros(M, np.float32)
            ref.expert_ffn(dense.tobytes(), x, want, 1.0)
            assert_close(out, want, 1e-5, 1e-5, what=f"dense int4 token {t}")
    finally:
        L.eh_destroy(h)
