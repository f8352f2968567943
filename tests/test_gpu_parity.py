"""GPU parity: every CUDA entry point against the oracle (and the reference's
golden outputs), called through the C ABI. Tolerances: see helpers.py."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from wisp_b200 import abi
from wisp_b200.blob import Int4Matrix, pack_blob, parse_blob
from wisp_b200.moe import MoeLayer, expert_ffn_decode, parse_header
from wisp_b200 import synth

from helpers import (NEAR_TIE, NEAR_TIE_SIGMOID, assert_close, bf16_to_f64, check_routing,
                     oracle_outputs, oracle_route, rel_errors)

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(params=["mixed", "tcgen05"])
def path(request):
    """mixed: segments of <= 32 rows on the register-fed kernel, larger ones
    on tcgen05 (the library default); tcgen05: every segment on tcgen05."""
    abi.lib().wisp_b200_set_skinny_max_rows(0 if request.param == "tcgen05" else -1)
    yield request.param
    abi.lib().wisp_b200_set_skinny_max_rows(-1)


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _dev_u16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(DEV)


def _rand_mat(rng, rows, cols, gs, zeros=True):
    n = rows * cols
    return Int4Matrix(rng.integers(0, 256, n // 2, dtype=np.uint8),
                      np.float16(rng.uniform(0.004, 0.02, n // gs)).view(np.uint16),
                      np.float16(rng.uniform(-0.01, 0.01, n // gs)).view(np.uint16) if zeros else None,
                      rows, cols)


def _blob_on_device(blob: bytes, packed_align16: bool) -> tuple[torch.Tensor, int]:
    """Copy a blob to device memory. packed_align16: place it at 8 mod 16 so
    the packed data (at +120) is 16-byte aligned; else at a 16-byte boundary
    (packed 8 bytes off) as the reference's own buffers are."""
    buf = torch.empty(len(blob) + 64, dtype=torch.uint8, device=DEV)
    base = buf.data_ptr()
    off = 0
    while (base + off) % 16 != (8 if packed_align16 else 0):
        off += 1
    buf[off:off + len(blob)] = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(DEV)
    return buf, base + off


# ---------------------------------------------------------------------------
# Reference launcher ABI
# ---------------------------------------------------------------------------

def test_launch_dequant_expert_bitexact(orc):
    rng = np.random.default_rng(0)
    L = abi.lib()
    for rows, cols, gs in [(64, 128, 64), (33, 64, 16), (7, 9, 3)]:
        n = rows * cols
        m = _rand_mat(rng, rows, cols, gs)
        nb = (n + 1) // 2
        ng = (n + gs - 1) // gs
        m.packed = m.packed[:nb] if m.packed.size >= nb else np.pad(m.packed, (0, nb - m.packed.size))
        m.scales = np.float16(rng.uniform(0.004, 0.02, ng)).view(np.uint16)
        m.zeros = np.float16(rng.uniform(-0.01, 0.01, ng)).view(np.uint16)
        p = torch.from_numpy(m.packed).to(DEV)
        s = _dev_u16(m.scales)
        z = _dev_u16(m.zeros)
        out = torch.empty(n, dtype=torch.float16, device=DEV)
        rc = L.launch_dequant_expert(p.data_ptr(), s.data_ptr(), z.data_ptr(), out.data_ptr(), n, gs, _stream())
        assert rc == 0
        ref = orc.dequant(m, n, gs).astype(np.float16)
        np.testing.assert_array_equal(out.cpu().numpy(), ref)
    assert L.launch_dequant_expert(None, None, None, None, 0, 64, None) != 0   # invalid value
    assert L.launch_dequant_expert(None, None, None, None, 10, 0, None) != 0


def test_gemv_swiglu_scale_accum_launchers():
    L = abi.lib()
    torch.manual_seed(0)
    for rows, cols in [(256, 512), (37, 100), (1, 8)]:
        W = (torch.randn(rows, cols, device=DEV) * 0.05).half()
        x = torch.randn(cols, device=DEV)
        y = torch.empty(rows, device=DEV)
        L.wisp_gpu_gemv_f16(W.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, _stream())
        ref = W.double() @ x.double()
        assert_close(y.cpu().numpy(), ref.cpu().numpy(), 1e-5, 1e-5, "gemv_f16")
        Wu = (torch.randn(rows, cols, device=DEV) * 0.05).half()
        h = torch.empty(rows, device=DEV)
        L.wisp_gpu_swiglu_ffn(W.data_ptr(), Wu.data_ptr(), x.data_ptr(), h.data_ptr(), rows, cols, _stream())
        g = W.double() @ x.double()
        u = Wu.double() @ x.double()
        assert_close(h.cpu().numpy(), (g / (1 + torch.exp(-g)) * u).cpu().numpy(), 1e-5, 1e-5, "swiglu_ffn")
    g = torch.randn(1000, device=DEV)
    u = torch.randn(1000, device=DEV)
    o = torch.empty(1000, device=DEV)
    L.wisp_gpu_swiglu(g.data_ptr(), u.data_ptr(), o.data_ptr(), 1000, _stream())
    assert_close(o.cpu().numpy(), (g.double() / (1 + torch.exp(-g.double())) * u.double()).cpu().numpy(), 1e-6, 1e-6)
    acc = torch.randn(1000, device=DEV)
    a0 = acc.clone()
    L.wisp_gpu_scale_accum(acc.data_ptr(), g.data_ptr(), 0.25, 1000, _stream())
    assert torch.allclose(acc, a0 + 0.25 * g)
    L.wisp_gpu_scale_accum(acc.data_ptr(), g.data_ptr(), 0.25, 0, _stream())   # silently ignored
    torch.cuda.synchronize()


@pytest.mark.parametrize("E,M,k", [(8, 4096, 2), (256, 7168, 8), (384, 7168, 8), (5, 64, 5),
                                   (1500, 512, 8), (2048, 256, 64)])
def test_router_topk_launcher(orc, E, M, k):
    """The reference launcher ABI for any expert count (more than 1024
    experts take the scratch-row selection)."""
    L = abi.lib()
    g = torch.Generator().manual_seed(E * 7 + M)
    W = (torch.randn(E, M, generator=g) * 0.02).half()
    bias = (torch.randn(E, generator=g) * 0.1).half()
    x = torch.randn(M, generator=g)
    Wd, bd, xd = W.to(DEV), bias.to(DEV), x.to(DEV)
    logits = torch.empty(E, device=DEV)
    idx = torch.empty(k, dtype=torch.int32).pin_memory()
    w = torch.empty(k, dtype=torch.float32).pin_memory()
    L.wisp_gpu_router_topk(Wd.data_ptr(), bd.data_ptr(), xd.data_ptr(), logits.data_ptr(), E, M, k,
                           idx.data_ptr(), w.data_ptr(), _stream())
    torch.cuda.synchronize()
    lg = orc.router_logits(W.view(torch.int16).numpy().view(np.uint16), 1,
                           bias.float().numpy().astype(np.float64), x.numpy()[None, :].astype(np.float64))
    i_ref, w_ref, mg = orc.topk(lg, k)
    check_routing(idx.numpy()[None, :], w.numpy()[None, :], i_ref, w_ref, mg)


@pytest.mark.parametrize("T,E,k,shared,skew", [(1, 8, 2, False, False), (300, 8, 2, True, False),
                                               (4096, 256, 8, True, True), (2048, 1024, 8, True, True),
                                               (5000, 64, 8, False, True), (64, 1100, 4, True, False)])
def test_dispatch_plan_layout(T, E, k, shared, skew):
    """wisp_b200_dispatch_plan: each expert's rows are its (token, slot)
    pairs in order, the shared expert holds every token with weight 1 --
    exactly, for the one-block count and the chunked fill (up to 1024 routed
    experts, chunks larger than one block's above 32k slots) and for the
    per-expert kernels beyond that. Expert-parallel dispatch relies on this
    order. Indices out of range (a malformed caller table) match no expert."""
    rng = np.random.default_rng(T * 7 + E)
    p = rng.gamma(0.3, size=E) if skew else np.ones(E)
    p = p / p.sum()
    idx = np.stack([rng.choice(E, size=k, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    if T > 1:
        idx[0, 0] = E + 3          # out of range
    w = rng.random((T, k)).astype(np.float32)
    cfg = abi.WispMoeConfig(tokens=T, hidden=128, inter=128, n_experts=E, top_k=k, group_size=128,
                            has_shared=int(shared))
    V = E + int(shared)
    d_idx = torch.from_numpy(idx).to(DEV)
    d_w = torch.from_numpy(w).to(DEV)
    counts = torch.full((V,), -1, dtype=torch.int32, device=DEV)
    segs = torch.zeros((V, 4), dtype=torch.int32, device=DEV)
    rows = T * k + (T if shared else 0)
    row_token = torch.full((rows,), -1, dtype=torch.int32, device=DEV)
    row_weight = torch.zeros((rows,), dtype=torch.float32, device=DEV)
    abi.call("wisp_b200_dispatch_plan", C.byref(cfg), d_idx.data_ptr(), d_w.data_ptr(),
             counts.data_ptr(), segs.data_ptr(), row_token.data_ptr(), row_weight.data_ptr(),
             _stream())
    torch.cuda.synchronize()
    flat_i, flat_w = idx.reshape(-1), w.reshape(-1)
    want_tok, want_w, want_segs = [], [], []
    for e in range(E):
        sel = np.nonzero(flat_i == e)[0]
        want_segs.append((e, len(want_tok), len(sel)))
        want_tok += list(sel // k)
        want_w += list(flat_w[sel])
    if shared:
        want_segs.append((E, len(want_tok), T))
        want_tok += list(range(T))
        want_w += [1.0] * T
    n = len(want_tok)
    got_segs = segs.cpu().numpy()[:, :3]
    np.testing.assert_array_equal(got_segs, np.array(want_segs, dtype=np.int32))
    np.testing.assert_array_equal(counts.cpu().numpy(), np.array([sg[2] for sg in want_segs]))
    np.testing.assert_array_equal(row_token.cpu().numpy()[:n], np.array(want_tok, dtype=np.int32))
    np.testing.assert_array_equal(row_weight.cpu().numpy()[:n], np.array(want_w, dtype=np.float32))


@pytest.mark.parametrize("T", [1, 2, 4, 5, 70])
@pytest.mark.parametrize("E,M,k,fp16,scoring", [(5, 128, 5, True, 0), (8, 4096, 2, False, 0),
                                                (256, 7168, 8, False, 1), (64, 2048, 6, True, 1),
                                                (300, 2048, 8, False, 0), (384, 7168, 8, False, 0),
                                                (512, 1024, 8, True, 0), (600, 1024, 8, False, 0),
                                                (1024, 512, 16, False, 0)])
def test_route_logits(orc, T, E, M, k, fp16, scoring):
    """Batched router through wisp_b200_route: logits within fp32 summation
    error of the fp64 oracle (|err| <= 1e-5 * sum|x w|), indices exact away
    from near-ties. T <= 4 runs the GEMV form, larger T the tiled split-K
    form."""
    g = torch.Generator().manual_seed(E * 31 + M + T)
    dt = torch.float16 if fp16 else torch.bfloat16
    W = (torch.randn(E, M, generator=g) * 0.02).to(dt)
    bias = (torch.randn(E, generator=g) * 0.1).float() if scoring else None
    x = torch.randn(T, M, generator=g).to(torch.bfloat16)
    cfg = abi.WispMoeConfig(tokens=T, hidden=M, inter=128, n_experts=E, top_k=k, group_size=128,
                            scoring=scoring, n_groups=8 if scoring else 1,
                            topk_groups=4 if scoring else 1, routed_scaling=2.5 if scoring else 1.0,
                            has_shared=0, router_fp16=1 if fp16 else 0)
    Wd, xd = W.to(DEV), x.to(DEV)
    bd = bias.to(DEV) if bias is not None else None
    ws = abi.WispMoeWeights()
    ws.router_w = Wd.data_ptr()
    ws.router_bias = bd.data_ptr() if bd is not None else None
    logits = torch.empty((T, E), device=DEV)
    idx = torch.empty((T, k), dtype=torch.int32, device=DEV)
    w = torch.empty((T, k), dtype=torch.float32, device=DEV)
    abi.call("wisp_b200_route", C.byref(cfg), C.byref(ws), xd.data_ptr(), logits.data_ptr(),
             idx.data_ptr(), w.data_ptr(), _stream())
    torch.cuda.synchronize()
    Wb = W.view(torch.int16).numpy().view(np.uint16)
    b64 = bias.numpy().astype(np.float64) if bias is not None else None
    xf = bf16_to_f64(x)
    lg = orc.router_logits(Wb, 1 if fp16 else 2, b64, xf)
    bound = np.abs(xf) @ np.abs(W.double().numpy()).T
    np.testing.assert_array_less(np.abs(logits.cpu().numpy() - lg), 1e-5 * bound + 1e-7)
    i_ref, w_ref, mg = orc.topk(lg, k, scoring, cfg.n_groups, cfg.topk_groups, cfg.routed_scaling)
    check_routing(idx.cpu().numpy(), w.cpu().numpy(), i_ref, w_ref, mg,
                  near_tie=NEAR_TIE if scoring == 0 else NEAR_TIE_SIGMOID)


# ---------------------------------------------------------------------------
# Fused decode entry (fp32 activations, reference blobs)
# ---------------------------------------------------------------------------

def _golden(golden_dir):
    return np.load(golden_dir / "moe_small.npz")


@pytest.mark.parametrize("packed_align16", [True, False])
def test_expert_ffn_decode_matches_reference_golden(golden_dir, packed_align16):
    g = _golden(golden_dir)
    M, I, E, k, gs, T = (int(v) for v in g["dims"])
    blobs = [b.tobytes() for b in g["blobs"]]
    meta = parse_header(blobs[0])
    dev = [_blob_on_device(b, packed_align16) for b in blobs]
    scratch = torch.empty(abi.lib().wisp_b200_expert_ffn_scratch_bytes(C.byref(meta), k + 1) // 4,
                          dtype=torch.float32, device=DEV)
    for t in range(T):
        x = torch.from_numpy(g["x"][t]).float().to(DEV)
        acc = torch.zeros(M, device=DEV)
        ptrs = [dev[int(e)][1] for e in g["idx"][t]] + [dev[E][1]]
        wts = [float(v) for v in g["w"][t]] + [1.0]
        expert_ffn_decode(meta, ptrs, wts, x, acc, scratch)
        torch.cuda.synchronize()
        mr, me = rel_errors(acc.cpu().numpy(), g["out"][t])
        assert mr < 1e-4 and me < 1e-4, (t, mr, me)


@pytest.mark.slow
@pytest.mark.parametrize("name", ["mixtral_b1", "ds_b1"])
def test_expert_ffn_decode_full_size(orc, name):
    spec = synth.CONFIGS[name]
    rng = np.random.default_rng(11)
    M, I, gs = spec.hidden, spec.inter, spec.group_size
    n = spec.top_k + (1 if spec.has_shared else 0)
    experts = [[_rand_mat(rng, I, M, gs, zeros=False), _rand_mat(rng, I, M, gs, zeros=False),
                _rand_mat(rng, M, I, gs, zeros=False)] for _ in range(n)]
    blobs = [pack_blob(*e, group_size=gs) for e in experts]
    meta = parse_header(blobs[0])
    dev = [_blob_on_device(b, True) for b in blobs]
    x = torch.randn(M, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).float()
    w = list(rng.uniform(0.05, 0.5, n))
    scratch = torch.empty(n * I, dtype=torch.float32, device=DEV)
    acc = torch.zeros(M, device=DEV)
    expert_ffn_decode(meta, [d[1] for d in dev], w, x.to(DEV), acc, scratch)
    torch.cuda.synchronize()
    ref = np.zeros(M)
    for e, wt in zip(experts, w):
        orc.expert_ffn(e, gs, x.numpy().astype(np.float64), wt, ref)
    assert_close(acc.cpu().numpy(), ref, 1e-4, 1e-4, name)


# ---------------------------------------------------------------------------
# Batched MoE layer (router + dispatch + tcgen05 grouped FFN + combine)
# ---------------------------------------------------------------------------

def _layer_from_golden(g):
    """LayerWeights from the golden reference blobs (fp16 router)."""
    M, I, E, k, gs, T = (int(v) for v in g["dims"])
    spec = synth.MoeSpec("golden", M, I, E, k, group_size=gs, has_shared=True, tokens=T)
    arenas = []
    for mi, (rows, cols) in enumerate([(I, M), (I, M), (M, I)]):
        packed = torch.empty((E + 1, rows, cols // 2), dtype=torch.uint8)
        scales = torch.empty((E + 1, rows, cols // gs), dtype=torch.float16)
        zeros = torch.empty_like(scales)
        for v in range(E + 1):
            b = g["blobs"][v]
            pm = parse_blob(b.tobytes())
            nn = rows * cols
            packed[v] = torch.from_numpy(b[pm.packed_off[mi]:pm.packed_off[mi] + nn // 2].copy()).view(rows, cols // 2)
            scales[v] = torch.from_numpy(b[pm.scales_off[mi]:pm.scales_off[mi] + 2 * nn // gs].copy()
                                         .view(np.int16)).view(torch.float16).view(rows, cols // gs)
            zeros[v] = torch.from_numpy(b[pm.zeros_off[mi]:pm.zeros_off[mi] + 2 * nn // gs].copy()
                                        .view(np.int16)).view(torch.float16).view(rows, cols // gs)
        arenas.append(synth.Int4Arena(packed.to(DEV), scales.to(DEV), zeros.to(DEV)))
    rw = torch.from_numpy(g["router_w16"].copy()).view(torch.float16).to(DEV)
    lw = synth.LayerWeights(spec, rw, None, *arenas)
    lw.build_table()
    return lw


def test_moe_forward_matches_reference_golden(golden_dir, path):
    g = _golden(golden_dir)
    M, I, E, k, gs, T = (int(v) for v in g["dims"])
    lw = _layer_from_golden(g)
    layer = MoeLayer(lw, T)
    layer.cfg.router_fp16 = 1
    x = torch.from_numpy(g["x"]).to(torch.bfloat16).to(DEV)
    out = layer.forward(x)
    torch.cuda.synchronize()
    layer.check()
    np.testing.assert_array_equal(layer.idx.cpu().numpy(), g["idx"])
    np.testing.assert_allclose(layer.wt.cpu().numpy(), g["w"], rtol=1e-5)
    assert_close(out.cpu().numpy(), g["out"], what="golden moe")


SMALL = [
    dict(hidden=512, inter=256, n_experts=16, top_k=4, group_size=128),
    dict(hidden=256, inter=384, n_experts=8, top_k=2, group_size=64, has_shared=True),
    dict(hidden=768, inter=256, n_experts=64, top_k=8, group_size=128, has_shared=True,
         scoring=abi.WISP_SCORE_SIGMOID_GROUPED, n_groups=8, topk_groups=4, routed_scaling=2.5),
    dict(hidden=256, inter=256, n_experts=32, top_k=6, group_size=64, skew=True),
    dict(hidden=256, inter=384, n_experts=64, top_k=32, group_size=128, has_shared=True),
]


@pytest.mark.parametrize("zeros", [False, True])
@pytest.mark.parametrize("T", [1, 5, 37, 300])
@pytest.mark.parametrize("si", range(len(SMALL)))
def test_moe_forward_small(orc, si, T, zeros, path):
    """Ragged token counts, both group sizes, both scoring rules, with and
    without zero points and a shared expert."""
    spec = synth.MoeSpec(f"small{si}", tokens=T, seed=100 + si, **SMALL[si])
    layers, x = synth.make_model(spec, DEV, zeros=zeros)
    lw = layers[0]
    layer = MoeLayer(lw, T)
    out = layer.forward(x)
    torch.cuda.synchronize()
    layer.check()
    idx = layer.idx.cpu().numpy()
    w = layer.wt.cpu().numpy()
    i_ref, w_ref, mg = oracle_route(orc, lw, x)
    check_routing(idx, w, i_ref, w_ref, mg,
                  near_tie=NEAR_TIE if spec.scoring == abi.WISP_SCORE_SOFTMAX else NEAR_TIE_SIGMOID)
    tokens = list(range(T)) if T <= 40 else list(range(0, T, 13))
    ref = oracle_outputs(orc, lw, x, idx, w.astype(np.float64), tokens)
    assert_close(out.cpu().numpy()[tokens], ref, what=spec.name)


@pytest.mark.parametrize("T", [1, 3, 300])
@pytest.mark.parametrize("si", [1, 2, 4])
def test_moe_forward_deterministic(orc, si, T, path):
    """WispMoeConfig.deterministic: the expert outputs as rows, then each
    token's rows summed in a fixed order. Two calls give the same bits, the
    outputs match the oracle, and they agree with the default (atomic)
    combine within the parity tolerance; top_k 32 + shared is 33 rows a token."""
    spec = synth.MoeSpec(f"det{si}", tokens=T, seed=500 + si, **SMALL[si])
    layers, x = synth.make_model(spec, DEV)
    lw = layers[0]
    det = MoeLayer(lw, T, deterministic=True)
    outs = []
    for _ in range(2):
        outs.append(det.forward(x).clone())
        torch.cuda.synchronize()
        det.check()
    assert torch.equal(outs[0], outs[1]), "deterministic layer: two calls differ"
    idx = det.idx.cpu().numpy()
    w = det.wt.cpu().numpy()
    i_ref, w_ref, mg = oracle_route(orc, lw, x)
    check_routing(idx, w, i_ref, w_ref, mg,
                  near_tie=NEAR_TIE if spec.scoring == abi.WISP_SCORE_SOFTMAX else NEAR_TIE_SIGMOID)
    tokens = list(range(T)) if T <= 40 else list(range(0, T, 13))
    ref = oracle_outputs(orc, lw, x, idx, w.astype(np.float64), tokens)
    got = outs[0].cpu().numpy()
    assert_close(got[tokens], ref, what=f"{spec.name} deterministic")
    fused = MoeLayer(lw, T).forward(x)
    torch.cuda.synchronize()
    assert_close(got, fused.cpu().numpy().astype(np.float64), what=f"{spec.name} vs fused combine")


DECODE = [
    dict(hidden=256, inter=256, n_experts=8, top_k=2, group_size=128),
    dict(hidden=512, inter=256, n_experts=256, top_k=8, group_size=128, has_shared=True,
         scoring=abi.WISP_SCORE_SIGMOID_GROUPED, n_groups=8, topk_groups=4, routed_scaling=2.5),
    dict(hidden=256, inter=128, n_experts=384, top_k=8, group_size=64, has_shared=True),
    dict(hidden=256, inter=128, n_experts=1024, top_k=32, group_size=128, has_shared=True),
]


@pytest.mark.parametrize("zeros", [False, True])
@pytest.mark.parametrize("T", [1, 2, 3, 4])
@pytest.mark.parametrize("di", range(len(DECODE)))
def test_moe_forward_decode_batches(orc, di, T, zeros):
    """Batches of 1-4 tokens take the decode chain (router logits, one
    planner launch, register-path gate/up and down): routing and every
    token's output against the oracle, twice over the same workspace, for
    softmax and sigmoid scoring and expert counts from 8 to 1024 (+ shared)."""
    spec = synth.MoeSpec(f"decode{di}", tokens=T, seed=300 + di, **DECODE[di])
    layers, x = synth.make_model(spec, DEV, zeros=zeros)
    lw = layers[0]
    layer = MoeLayer(lw, T)
    out = torch.full((T, spec.hidden), float("nan"), dtype=torch.float32, device=DEV)
    for _ in range(2):   # the second call reuses the workspace (plans, rows, output)
        layer.forward(x, out)
        torch.cuda.synchronize()
        layer.check()
        idx = layer.idx.cpu().numpy()
        w = layer.wt.cpu().numpy()
        i_ref, w_ref, mg = oracle_route(orc, lw, x)
        check_routing(idx, w, i_ref, w_ref, mg,
                      near_tie=NEAR_TIE if spec.scoring == abi.WISP_SCORE_SOFTMAX else NEAR_TIE_SIGMOID)
        ref = oracle_outputs(orc, lw, x, idx, w.astype(np.float64), list(range(T)))
        assert_close(out.cpu().numpy(), ref, what=f"{spec.name} T={T}")


def _segments_device(segs):
    arr = (abi.WispSegment * len(segs))()
    for i, (e, b, r) in enumerate(segs):
        arr[i].expert, arr[i].row_begin, arr[i].rows = e, b, r
    return torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(DEV)


@pytest.mark.parametrize("mode", [0, 1])
def test_grouped_ffn_tile_boundaries(orc, mode, path):
    """Segments of 0, 1, 15, 16, 17, 32, 33, 64, 65, 128, 129 and 300 rows
    (every BN choice and its ragged edge) through the grouped kernels."""
    counts = [0, 1, 15, 16, 17, 32, 33, 64, 65, 128, 129, 300]
    spec = synth.MoeSpec("tiles", 256, 256, len(counts), 1, group_size=128, tokens=1, seed=7)
    lw = synth.make_model(spec, DEV)[0][0]
    R = sum(counts)
    T = R
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn((T, spec.hidden), generator=g, device=DEV).to(torch.bfloat16)
    segs, b = [], 0
    for e, c in enumerate(counts):
        segs.append((e, b, c))
        b += c
    row_token = torch.arange(R, dtype=torch.int32, device=DEV)   # row p holds token p
    row_w = torch.rand(R, generator=g, device=DEV) + 0.5
    xp = torch.empty((R, spec.hidden), dtype=torch.float16, device=DEV)
    h = torch.empty((R, spec.inter), dtype=torch.float16, device=DEV)
    out = torch.zeros((R, spec.hidden), dtype=torch.float32, device=DEV)
    cfg = spec.cfg(T)
    ws = torch.empty(abi.lib().wisp_b200_grouped_workspace_bytes(C.byref(cfg), len(segs), R),
                     dtype=torch.uint8, device=DEV)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    dsegs = _segments_device(segs)
    abi.call("wisp_b200_pack_rows", x.data_ptr(), None, R, spec.hidden, xp.data_ptr(), _stream())
    abi.call("wisp_b200_grouped_ffn", C.byref(cfg), lw.prepare().data_ptr(), lw.table.data_ptr(),
             lw.n_entries,
             dsegs.data_ptr(), len(segs), R,
             xp.data_ptr(), h.data_ptr(), mode, row_token.data_ptr(), row_w.data_ptr(), out.data_ptr(),
             ws.data_ptr(), ws.numel(), flag.data_ptr(), _stream())
    abi.call("wisp_b200_check_error_flag", flag.data_ptr(), _stream())
    got = out.cpu().numpy()
    xs = bf16_to_f64(x)
    wv = row_w.cpu().numpy()
    for e, b0, c in segs:
        if c == 0:
            continue
        mats = lw.expert_host(e)
        for p in sorted({b0, b0 + c - 1, b0 + c // 2}):
            ref = orc.expert_ffn(mats, spec.group_size, xs[p], wv[p] if mode == 0 else 1.0)
            assert_close(got[p], ref, what=f"seg {e} rows {c} row {p}")


@pytest.mark.slow
@pytest.mark.parametrize("name", ["mixtral_b1", "mixtral_b64", "ds_b1", "ds_b128", "ds_prefill"])
def test_moe_forward_full_size(orc, name):
    spec = synth.CONFIGS[name]
    layers, x = synth.make_model(spec, DEV)
    lw = layers[0]
    layer = MoeLayer(lw, spec.tokens)
    out = layer.forward(x)
    torch.cuda.synchronize()
    layer.check()
    idx = layer.idx.cpu().numpy()
    w = layer.wt.cpu().numpy()
    T = spec.tokens
    # routing of every token (oracle router in fp64)
    i_ref, w_ref, mg = oracle_route(orc, lw, x)
    tie = NEAR_TIE if spec.scoring == abi.WISP_SCORE_SOFTMAX else NEAR_TIE_SIGMOID
    near = check_routing(idx, w, i_ref, w_ref, mg, near_tie=tie)
    print(f"{name}: {len(near)} near-tie tokens of {T} (margin < {tie})")
    assert len(near) <= max(2, T // 20)
    # expert outputs of sampled tokens under the GPU's routing
    tokens = sorted({0, T - 1, T // 2, T // 3})
    ref = oracle_outputs(orc, lw, x, idx, w.astype(np.float64), tokens)
    assert_close(out.cpu().numpy()[tokens], ref, what=name)
    # size-independent property: permuting the tokens permutes the outputs
    if T > 1:
        perm = torch.randperm(T, generator=torch.Generator().manual_seed(0)).to(DEV)
        out2 = layer.forward(x[perm].contiguous())
        torch.cuda.synchronize()
        assert_close(out2.cpu().numpy(), out[perm].cpu().numpy(), 1e-5, 1e-6, "permutation")


def test_rms_rescale_matches_fp64():
    """d_out[t] = bf16(d_in[t] / sqrt(mean(d_in[t]^2) + eps)): within one bf16
    rounding of the fp64 value (fp32 sum of squares and rsqrt)."""
    g = torch.Generator(device=DEV).manual_seed(9)
    for T, M in [(1, 7168), (7, 4096), (256, 7168), (3, 256)]:
        x = torch.randn((T, M), generator=g, device=DEV) * torch.rand((T, 1), generator=g, device=DEV) * 30
        y = torch.empty((T, M), dtype=torch.bfloat16, device=DEV)
        abi.call("wisp_b200_rms_rescale", x.data_ptr(), y.data_ptr(), T, M, 1e-6, _stream())
        torch.cuda.synchronize()
        xd = x.double()
        ref = xd / torch.sqrt((xd * xd).mean(dim=1, keepdim=True) + 1e-6)
        got = y.double()
        # bf16 keeps 8 significant bits: |err| <= 2^-8 |ref| (rounding plus the
        # fp32 reduction's last bits)
        assert torch.all((got - ref).abs() <= 2.0 ** -8 * ref.abs() + 1e-30), (T, M)


@pytest.mark.slow
def test_ep_stack_headline_config(orc):
    """The benchmark's own workload: 4 stacked layers, 384 routed
    experts + 1 shared, softmax top-8, 256 tokens, int4 group 128, with the
    rms_rescale step between layers exactly as bench.py chains them. Every
    layer: the routing of all 256 tokens against the fp64 oracle router
    (indices exact away from near-ties), sampled token outputs against the
    oracle under the GPU's routing, and the rescale against fp64."""
    spec = synth.CONFIGS["ep_stack"]
    layers_w, x0 = synth.make_model(spec, DEV)
    T, M = spec.tokens, spec.hidden
    x = x0
    for l, lw in enumerate(layers_w):
        layer = MoeLayer(lw, T)
        out = layer.forward(x)
        torch.cuda.synchronize()
        layer.check()
        idx = layer.idx.cpu().numpy()
        w = layer.wt.cpu().numpy()
        i_ref, w_ref, mg = oracle_route(orc, lw, x)
        near = check_routing(idx, w, i_ref, w_ref, mg, near_tie=NEAR_TIE)
        # Layers after the first take the previous layer's rescaled output,
        # which concentrates the router logits: more tokens fall inside the
        # near-tie band there (excluded from the exact check, never more
        # than a tenth of the tokens).
        print(f"ep_stack layer {l}: {len(near)} near-tie tokens of {T}")
        assert len(near) <= T // 10, f"layer {l}: {len(near)} near-ties"
        tokens = [0, 97, 181, T - 1]
        ref = oracle_outputs(orc, lw, x, idx, w.astype(np.float64), tokens)
        assert_close(out.cpu().numpy()[tokens], ref, what=f"ep_stack layer {l}")
        if l + 1 < len(layers_w):
            nxt = torch.empty((T, M), dtype=torch.bfloat16, device=DEV)
            abi.call("wisp_b200_rms_rescale", out.data_ptr(), nxt.data_ptr(), T, M, 1e-6, _stream())
            torch.cuda.synchronize()
            od = out.double()
            want = od / torch.sqrt((od * od).mean(dim=1, keepdim=True) + 1e-6)
            assert torch.all((nxt.double() - want).abs() <= 2.0 ** -8 * want.abs() + 1e-30)
            x = nxt
