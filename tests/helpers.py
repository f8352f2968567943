"""Shared checks for the parity tests.

Tolerances: router expert indices bit-exact (ties to
the lower index); outputs within max relative error 1e-2 and mean absolute
error 1e-3, both normalised by the reference output's magnitude:
    max|got - ref| / max|ref|   <= 1e-2
    mean|got - ref| / mean|ref| <= 1e-3
A token whose oracle routing margin (gap between the k-th pick and the best
non-pick, fp64) is below NEAR_TIE is a near-tie: fp32 summation order may
legitimately flip it, so its indices are reported, not asserted. Routing
weights agree within ROUTE_W_RTOL: the batched router sums bf16 products on
the tensor cores with fp32 accumulation, whose logits differ from fp64 by
~1e-5 relative (the weights of a softmax follow the logit differences).
"""
from __future__ import annotations

import os

import numpy as np
import torch

MAX_REL = 1e-2
MEAN_REL = 1e-3
NEAR_TIE = 1e-4           # softmax routing: margin in logit units
NEAR_TIE_SIGMOID = 5e-5   # sigmoid routing: margin in score units (tensor-core logits: ~1e-5)
ROUTE_W_RTOL = 1e-4


def bf16_to_f64(x: torch.Tensor) -> np.ndarray:
    return x.float().cpu().numpy().astype(np.float64)


def rel_errors(got: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.abs(got - ref)
    return float(d.max() / max(np.abs(ref).max(), 1e-30)), float(d.mean() / max(np.abs(ref).mean(), 1e-30))


def assert_close(got, ref, max_rel=MAX_REL, mean_rel=MEAN_REL, what=""):
    mr, me = rel_errors(got, ref)
    if os.environ.get("WB_REPORT_ERRORS"):
        # the measured errors, for the record (run pytest with -s)
        print(f"[errors] {what}: max_rel={mr:.3e} mean_rel={me:.3e}")
    assert mr <= max_rel and me <= mean_rel, f"{what}: max_rel={mr:.3e} (<= {max_rel}) mean_rel={me:.3e} (<= {mean_rel})"
    return mr, me


def router_weight_host(lw):
    """(uint16 bits, wtype) of a layer's router weight for the oracle."""
    w = lw.router_w.cpu()
    bits = w.view(torch.int16).numpy().view(np.uint16)
    return bits, (1 if w.dtype == torch.float16 else 2)


def oracle_route(orc, lw, x: torch.Tensor):
    spec = lw.spec
    W, wt = router_weight_host(lw)
    bias = None if lw.router_bias is None else lw.router_bias.float().cpu().numpy().astype(np.float64)
    logits = orc.router_logits(W, wt, bias, bf16_to_f64(x))
    return orc.topk(logits, spec.top_k, 0 if spec.scoring == 0 else 1, spec.n_groups,
                    spec.topk_groups, spec.routed_scaling)


def check_routing(idx_gpu, w_gpu, idx_ref, w_ref, margin, scoring_w_tol=ROUTE_W_RTOL, near_tie=NEAR_TIE):
    """Indices exact except near-ties; weights close where indices agree.
    Returns the list of near-tie tokens."""
    idx_gpu = np.asarray(idx_gpu)
    near = [t for t in range(idx_ref.shape[0]) if margin[t] < near_tie]
    for t in range(idx_ref.shape[0]):
        if t in near:
            continue
        assert np.array_equal(idx_gpu[t], idx_ref[t]), f"token {t}: gpu {idx_gpu[t]} ref {idx_ref[t]} margin {margin[t]:.2e}"
        np.testing.assert_allclose(w_gpu[t], w_ref[t], rtol=scoring_w_tol, atol=1e-7)
    return near


def oracle_outputs(orc, lw, x: torch.Tensor, idx: np.ndarray, w: np.ndarray, tokens):
    """fp64 oracle outputs for the listed tokens under the given routing."""
    spec = lw.spec
    need = sorted({int(e) for t in tokens for e in idx[t] if e >= 0})
    experts = [None] * spec.n_experts
    for e in need:
        experts[e] = lw.expert_host(e)
    shared = lw.expert_host(spec.n_experts) if spec.has_shared else None
    return orc.moe_tokens(spec.hidden, spec.group_size, bf16_to_f64(x), idx, w, experts, shared,
                          list(tokens))
