"""The oracle (oracle/oracle.c) pinned against the reference's golden vectors
and against the reference's own compiled CPU functions (oracle/_ref)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import RefCPU
from wisp_b200.blob import Int4Matrix, pack_blob, parse_blob

from helpers import rel_errors


def _fv(golden_dir):
    return np.load(golden_dir / "format_vectors.npz")


def _u16(a):
    return np.asarray(a).view(np.uint16)


def test_constant_group_packs_to_0x88_and_dequantises_exactly(orc, golden_dir):
    # Reference known answer: tests/test_adapters.py:262-267.
    fv = _fv(golden_dir)
    assert fv["const_packed"][0] == 0x88
    m = Int4Matrix(fv["const_packed"], _u16(fv["const_scales"]), _u16(fv["const_zeros"]), 2, 64)
    got = orc.dequant(m, 128, 64)
    np.testing.assert_array_equal(got.astype(np.float16), fv["const_dequant"].reshape(-1).astype(np.float16))


def test_roundtrip_dequant_matches_reference_python(orc, golden_dir):
    # Reference: tests/test_adapters.py:250-259 and quantizer.py:89-105.
    fv = _fv(golden_dir)
    m = Int4Matrix(fv["rt_packed"], _u16(fv["rt_scales"]), _u16(fv["rt_zeros"]), 64, 128)
    got = orc.dequant(m, 64 * 128, 64)
    ref = fv["rt_dequant"].reshape(-1)
    # The reference rounds its result to fp16; ours is the fp32 value.
    np.testing.assert_array_equal(got.astype(np.float16), ref.astype(np.float16))
    # Round-trip error bound of the reference test: <= 0.51 quantisation step.
    w = fv["rt_weight"].reshape(-1, 64)
    step = (w.max(1) - w.min(1)) / 15
    assert np.abs(fv["rt_weight"].reshape(-1) - got).max() <= step.max() * 0.51 + 1e-6


def test_small_blob_header_and_dequant(orc, golden_dir):
    # Reference: tests/test_adapters.py:281-345 (120-byte header, blobs tile
    # the file, C dequant == Python dequant within 5e-3).
    fv = _fv(golden_dir)
    blob = fv["small_blob"].tobytes()
    meta = orc.parse_header(blob)
    assert meta is not None
    assert meta["packed_off"][0] == 120
    assert meta["rows"] == [16, 16, 32] and meta["cols"] == [32, 32, 16]
    assert meta["group_size"] == 16 and meta["total_bytes"] == len(blob)
    pm = parse_blob(blob)
    assert list(pm.packed_off) == meta["packed_off"] and pm.total_bytes == len(blob)
    raw = np.frombuffer(blob, np.uint8)
    for i in range(3):
        r, c = meta["rows"][i], meta["cols"][i]
        n = r * c
        p0, s0, z0 = meta["packed_off"][i], meta["scales_off"][i], meta["zeros_off"][i]
        m = Int4Matrix(raw[p0:p0 + n // 2], raw[s0:s0 + n // 16 * 2].view(np.uint16),
                       raw[z0:z0 + n // 16 * 2].view(np.uint16), r, c)
        got = orc.dequant(m, n, 16)
        ref = fv[f"small_dequant_{i}"]
        assert np.abs(got - ref).max() <= 5e-3
        np.testing.assert_array_equal(got.astype(np.float16), ref.astype(np.float16))


def test_truncated_or_corrupt_header_rejected(orc, golden_dir):
    blob = _fv(golden_dir)["small_blob"].tobytes()
    assert orc.parse_header(blob[:-1]) is None           # truncated
    assert orc.parse_header(blob[:100]) is None          # shorter than the header
    bad = bytearray(blob)
    bad[0] ^= 0xff
    assert orc.parse_header(bytes(bad)) is None          # magic
    bad = bytearray(blob)
    bad[20] = 2
    assert orc.parse_header(bytes(bad)) is None          # n_mats


def _experts_from_blobs(blobs):
    out = []
    for b in blobs:
        b = np.asarray(b, np.uint8)
        pm = parse_blob(b.tobytes())
        mats = []
        for i in range(3):
            r, c = pm.rows[i], pm.cols[i]
            n = r * c
            ng = n // pm.group_size
            mats.append(Int4Matrix(b[pm.packed_off[i]:pm.packed_off[i] + n // 2],
                                   b[pm.scales_off[i]:pm.scales_off[i] + 2 * ng].view(np.uint16),
                                   b[pm.zeros_off[i]:pm.zeros_off[i] + 2 * ng].view(np.uint16), r, c))
        out.append(mats)
    return out, pm.group_size


def test_oracle_matches_reference_moe_golden(orc, golden_dir):
    """Router indices, weights and per-token outputs of the reference's CPU
    run_moe branch (golden) against the fp64 restatement."""
    g = np.load(golden_dir / "moe_small.npz")
    M, I, E, k, gs, T = (int(v) for v in g["dims"])
    experts, gs2 = _experts_from_blobs(g["blobs"])
    assert gs2 == gs
    W16 = g["router_w16"].view(np.uint16)
    x = g["x"].astype(np.float64)
    logits = orc.router_logits(W16, 1, None, x)
    idx, w, margin = orc.topk(logits, k)
    assert (margin > 1e-6).all()
    np.testing.assert_array_equal(idx, g["idx"])
    np.testing.assert_allclose(w, g["w"], rtol=1e-5)
    out = orc.moe_tokens(M, gs, x, idx, w, experts[:E], experts[E], list(range(T)))
    mr, me = rel_errors(out, g["out"])
    assert mr < 1e-5 and me < 1e-5, (mr, me)
    out2 = orc.moe_tokens(M, gs, x, idx, w, experts[:E], None, list(range(T)))
    mr, me = rel_errors(out2, g["out_noshared"])
    assert mr < 1e-5 and me < 1e-5, (mr, me)


ref_missing = not RefCPU.available()


@pytest.mark.skipif(ref_missing, reason="oracle/_ref/libwisp_ref.so not built")
def test_oracle_matches_live_reference_functions(orc):
    """Random shapes through the reference's compiled cpu_gemv_int4 and
    cpu_router_topk versus the restatement."""
    ref = RefCPU()
    rng = np.random.default_rng(5)
    for rows, cols, gs in [(64, 256, 64), (96, 512, 128), (33, 64, 32)]:
        n = rows * cols
        m = Int4Matrix(rng.integers(0, 256, n // 2, dtype=np.uint8),
                       np.float16(rng.uniform(0.004, 0.02, n // gs)).view(np.uint16),
                       np.float16(rng.uniform(-0.01, 0.01, n // gs)).view(np.uint16), rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        y_ref = ref.gemv_int4(m, gs, x)
        y_orc = orc.gemv(m, gs, x.astype(np.float64))
        mr, me = rel_errors(y_ref, y_orc)
        assert mr < 1e-5 and me < 1e-5
    for E, M, k in [(8, 256, 2), (64, 512, 8), (256, 128, 8)]:
        W = np.float16(rng.standard_normal((E, M)) * 0.05).view(np.uint16)
        x = rng.standard_normal(M).astype(np.float32)
        i_ref, w_ref = ref.router_topk(W, None, x, k)
        logits = orc.router_logits(W, 1, None, x[None, :].astype(np.float64))
        i_orc, w_orc, mg = orc.topk(logits, k)
        if mg[0] > 1e-5:
            np.testing.assert_array_equal(i_ref, i_orc[0])
            np.testing.assert_allclose(w_ref, w_orc[0], rtol=1e-5)


@pytest.mark.skipif(not RefCPU.available(avx512=True), reason="AVX-512 reference build or CPU support missing")
def test_reference_avx512_build_is_numerically_wrong(orc):
    """The reference's own AVX-512 flags produce a wrong int4 GEMV (its
    vector branch double counts; csrc/core/wisp_engine.c:445-456). This is why
    the AVX-512 CPU number is reported but never used as a parity oracle."""
    ref = RefCPU(avx512=True)
    rng = np.random.default_rng(3)
    rows, cols, gs = 64, 512, 128
    n = rows * cols
    m = Int4Matrix(rng.integers(0, 256, n // 2, dtype=np.uint8),
                   np.float16(rng.uniform(0.004, 0.02, n // gs)).view(np.uint16),
                   np.zeros(n // gs, np.uint16), rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    mr, _ = rel_errors(ref.gemv_int4(m, gs, x), orc.gemv(m, gs, x.astype(np.float64)))
    assert mr > 0.5


def test_sigmoid_grouped_known_answer(orc):
    # 8 experts, 4 groups of 2, keep 2 groups, pick 2 experts, scaling 2.5.
    s = np.array([0.9, 0.1, 0.5, 0.45, 0.95, 0.2, 0.3, 0.3])
    logits = np.log(s / (1 - s))[None, :]
    idx, w, mg = orc.topk(logits, 2, scoring=1, n_groups=4, topk_groups=2, scaling=2.5)
    # group scores: g0 1.0, g1 0.95, g2 1.15, g3 0.6 -> keep g2, g0 -> experts 4 (0.95), 0 (0.9)
    assert idx[0].tolist() == [4, 0]
    np.testing.assert_allclose(w[0], np.array([0.95, 0.9]) / 1.85 * 2.5, rtol=1e-12)
    # tie: equal scores go to the lower index
    s = np.array([0.5, 0.5, 0.5, 0.5])
    idx, w, mg = orc.topk(np.log(s / (1 - s))[None, :], 2, scoring=1, n_groups=2, topk_groups=1, scaling=1.0)
    assert idx[0].tolist() == [0, 1] and mg[0] == 0.0


def test_softmax_tie_goes_to_lower_index(orc):
    idx, w, mg = orc.topk(np.array([[1.0, 3.0, 3.0, 2.0]]), 2)
    assert idx[0].tolist() == [1, 2]
    idx, w, mg = orc.topk(np.array([[1.0, 3.0, 3.0, 3.0]]), 2)
    assert idx[0].tolist() == [1, 2] and mg[0] == 0.0


def test_blob_writer_roundtrip(orc):
    rng = np.random.default_rng(0)
    mats = []
    for r, c in [(128, 256), (128, 256), (256, 128)]:
        n = r * c
        mats.append(Int4Matrix(rng.integers(0, 256, n // 2, dtype=np.uint8),
                               np.float16(rng.uniform(0.004, 0.02, n // 64)).view(np.uint16),
                               None, r, c))
    blob = pack_blob(*mats, group_size=64, layer=3, expert=9)
    meta = orc.parse_header(blob)
    assert meta["total_bytes"] == len(blob) and meta["group_size"] == 64
    assert meta["packed_off"][0] == 120
