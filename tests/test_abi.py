"""The C ABI library loads and exports every declared entry point; host-side
validation and blob parsing behave like the reference (no GPU needed)."""
from __future__ import annotations

import ctypes as C
import subprocess

import numpy as np
import pytest

from wisp_b200 import abi
from wisp_b200.blob import Int4Matrix, pack_blob


def test_library_loads_and_reports_version():
    v = abi.lib().wisp_b200_version().decode()
    assert "sm_100a" in v


def test_every_declared_function_is_exported():
    L = abi.lib()
    declared = abi.header_functions()
    assert len(declared) >= 19
    for name in declared:
        assert hasattr(L, name), f"{name} declared in include/wisp_b200.h but not exported"
    assert set(declared) == set(abi.SIGNATURES)
    out = subprocess.run(["nm", "-D", "--defined-only", str(abi.LIB_PATH)], capture_output=True,
                         text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert set(declared) <= exported


def test_reference_launcher_symbols_present():
    # Same names as csrc/core/wisp_engine.h:496-583 of the reference.
    for name in ["launch_dequant_expert", "async_load_expert", "wisp_gpu_gemv_f16",
                 "wisp_gpu_swiglu", "wisp_gpu_swiglu_ffn", "wisp_gpu_scale_accum",
                 "wisp_gpu_router_topk"]:
        assert hasattr(abi.lib(), name)


def _golden_blob(golden_dir):
    return np.load(golden_dir / "format_vectors.npz")["small_blob"].tobytes()


def test_parse_header_matches_oracle(orc, golden_dir):
    blob = _golden_blob(golden_dir)
    meta = abi.WispExpertMeta()
    err = abi.WispErrCtx()
    rc = abi.lib().wisp_b200_parse_expert_header(blob, len(blob), C.byref(meta), C.byref(err))
    assert rc == abi.WISP_OK and meta.valid == 1
    o = orc.parse_header(blob)
    assert list(meta.packed_off) == o["packed_off"]
    assert list(meta.scales_off) == o["scales_off"]
    assert list(meta.zeros_off) == o["zeros_off"]
    assert list(meta.rows) == o["rows"] and list(meta.cols) == o["cols"]
    assert meta.group_size == o["group_size"] and meta.total_bytes == o["total_bytes"]


@pytest.mark.parametrize("mutate,code", [
    (lambda b: b[:-1], abi.WISP_ERR_MODEL),                         # truncated
    (lambda b: b[:64], abi.WISP_ERR_MODEL),                         # shorter than header
    (lambda b: b"\x00" + b[1:], abi.WISP_ERR_MODEL),                # bad magic
    (lambda b: b[:4] + b"\x02" + b[5:], abi.WISP_ERR_MODEL),        # bad version
])
def test_parse_header_rejects_bad_blobs(golden_dir, mutate, code):
    blob = mutate(_golden_blob(golden_dir))
    meta = abi.WispExpertMeta()
    err = abi.WispErrCtx()
    rc = abi.lib().wisp_b200_parse_expert_header(blob, len(blob), C.byref(meta), C.byref(err))
    assert rc == code
    assert err.code == code and err.message


def _cfg(**kw):
    c = abi.WispMoeConfig()
    c.tokens, c.hidden, c.inter, c.n_experts, c.top_k = 4, 256, 128, 8, 2
    c.group_size, c.scoring, c.n_groups, c.topk_groups = 64, 0, 1, 1
    c.routed_scaling, c.has_shared, c.router_fp16 = 1.0, 0, 0
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def test_deterministic_layer_workspace_holds_its_rows():
    """A deterministic layer's workspace adds one fp32 row per routed row
    (tokens x (top_k + shared) x hidden) and the per-token row lists."""
    for shared in (0, 1):
        base = abi.lib().wisp_b200_moe_workspace_bytes(C.byref(_cfg(has_shared=shared)))
        det = abi.lib().wisp_b200_moe_workspace_bytes(C.byref(_cfg(has_shared=shared, deterministic=1)))
        rows = 4 * (2 + shared)
        assert base > 0 and det >= base + rows * 256 * 4 + 4 * 4 + 4 * rows


@pytest.mark.parametrize("kw", [
    dict(hidden=200), dict(inter=100), dict(group_size=32), dict(top_k=0), dict(top_k=9),
    dict(n_experts=2000), dict(tokens=0), dict(scoring=5),
    dict(scoring=1, n_groups=3), dict(scoring=1, n_groups=4, topk_groups=5),
])
def test_invalid_configs_are_rejected_before_any_launch(kw):
    c = _cfg(**kw)
    assert abi.lib().wisp_b200_moe_workspace_bytes(C.byref(c)) == 0
    w = abi.WispMoeWeights()
    w.router_w = 16
    w.experts = 16
    err = abi.WispErrCtx()
    rc = abi.lib().wisp_b200_moe_forward(C.byref(c), C.byref(w), 16, 16, None, None, 16, 1 << 30,
                                         None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
    with pytest.raises(RuntimeError, match=r"wisp engine error \[4\]"):
        abi.check(rc, err)


def test_valid_config_workspace_is_sized():
    c = _cfg()
    n = abi.lib().wisp_b200_moe_workspace_bytes(C.byref(c))
    rows = 4 * 2
    assert n >= rows * (256 + 128) * 2


def test_expert_ffn_argument_checks(golden_dir):
    blob = _golden_blob(golden_dir)
    meta = abi.WispExpertMeta()
    err = abi.WispErrCtx()
    abi.lib().wisp_b200_parse_expert_header(blob, len(blob), C.byref(meta), C.byref(err))
    ptrs = (C.c_void_p * 1)(16)
    ws = (C.c_float * 1)(1.0)
    # n_blobs out of range
    rc = abi.lib().wisp_b200_expert_ffn(C.byref(meta), ptrs, ws, 0, 16, 16, 16, 1 << 20, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
    # golden blob has gs=16 with hidden 32: accepted shapes, but scratch too small
    rc = abi.lib().wisp_b200_expert_ffn(C.byref(meta), ptrs, ws, 1, 16, 16, 16, 4, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"scratch" in err.message
    # inconsistent shapes
    bad = abi.WispExpertMeta.from_buffer_copy(meta)
    bad.rows[2] = 48
    rc = abi.lib().wisp_b200_expert_ffn(C.byref(bad), ptrs, ws, 1, 16, 16, 16, 1 << 20, None, C.byref(err))
    assert rc == abi.WISP_ERR_MODEL


def test_grouped_ffn_argument_checks():
    L, err = abi.lib(), abi.WispErrCtx()
    c = _cfg(group_size=32)
    assert L.wisp_b200_grouped_workspace_bytes(C.byref(c), 4, 8) == 0
    rc = L.wisp_b200_grouped_ffn(C.byref(c), 256, 16, 4, 16, 1, 8, 16, 16, 0, 16, 16, 16, 256,
                                 1 << 30, None, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"group_size" in err.message
    c = _cfg()
    need = L.wisp_b200_grouped_workspace_bytes(C.byref(c), 4, 8)
    # tile plans, ~25 MB of split partial sums (256 items x 192 columns x 128
    # rows), q16 rows and their metadata
    assert need >= 256 * 192 * 128 * 4 + 8 * 2 * c.hidden
    assert L.wisp_b200_grouped_workspace_bytes(C.byref(c), 4, 800) > need
    rc = L.wisp_b200_grouped_ffn(C.byref(c), 256, 16, 4, 16, 1, 8, 16, 16, 0, None, None, 16, 256,
                                 need, None, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"mode 0" in err.message
    rc = L.wisp_b200_grouped_ffn(C.byref(c), 264, 16, 4, 16, 1, 8, 16, 16, 1, None, None, 16, 256,
                                 need, None, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"256-byte" in err.message
    rc = L.wisp_b200_grouped_ffn(C.byref(c), 256, 16, 4, 16, 4, 8, 16, 16, 1, None, None, 16, 256,
                                 need - 1, None, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"workspace" in err.message


def test_prepared_size_and_checks():
    c = _cfg()
    n = abi.lib().wisp_b200_prepared_bytes(C.byref(c), 9)
    # 27 descriptors + flags + transposed scales and zeros for 27 matrices
    assert n >= 27 * 128 + 27 * 4 + 2 * 27 * (256 * 128 // 64) * 2
    assert abi.lib().wisp_b200_prepared_bytes(C.byref(_cfg(group_size=32)), 9) == 0
    err = abi.WispErrCtx()
    rc = abi.lib().wisp_b200_prepare_experts(C.byref(c), 16, 9, 256, n - 1, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"required" in err.message


def test_ep_exchange_argument_checks():
    """The exchange entry points reject bad shapes before any launch."""
    L, err = abi.lib(), abi.WispErrCtx()
    P = 256  # a non-null, 16-byte-aligned stand-in pointer; never dereferenced here
    assert L.wisp_b200_ep_block_bytes(7168, 48, 32, 8) > 32 * 7168 * 2
    assert L.wisp_b200_ep_block_bytes(7168, 48, 32, 33) == 0       # top_k > 32
    assert L.wisp_b200_ep_block_bytes(100, 48, 32, 8) == 0          # hidden % 8
    # experts do not split over the ranks
    rc = L.wisp_b200_ep_dispatch(P, 4, 256, P, 2, P, P, P, 8, 3, 4, P, P, None, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"ep_dispatch" in err.message
    # more tokens than the block capacity
    rc = L.wisp_b200_ep_dispatch(P, 5, 256, P, 2, P, P, P, 8, 2, 4, P, P, None, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
    # misaligned send buffer
    rc = L.wisp_b200_ep_dispatch(P, 4, 256, P, 2, P, P, P, 8, 2, 4, P + 8, P, None, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"16-byte" in err.message
    # null pointer
    rc = L.wisp_b200_ep_dispatch(None, 4, 256, P, 2, P, P, P, 8, 2, 4, P, P, None, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
    # too many (rank, local expert) pairs for the single-block receive plan
    rc = L.wisp_b200_ep_recv_plan(P, 8, 200, 4, 2, 256, 0, P, P, P, P, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"1024" in err.message
    # own rows beyond the block capacity
    rc = L.wisp_b200_ep_recv_plan(P, 2, 4, 4, 2, 256, 5, P, P, P, P, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"own_rows" in err.message
    rc = L.wisp_b200_ep_gather_rows(P, 2, 4, 4, 2, 260, P, P, None, 0, 16, P, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
    # own rows without their buffer
    rc = L.wisp_b200_ep_gather_rows(P, 2, 4, 4, 2, 256, P, P, None, 3, 16, P, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
    rc = L.wisp_b200_ep_combine(P, P, 5, 2, 4, 256, P, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
    rc = L.wisp_b200_ep_combine(P, P, 4, 2, 4, 258, P, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
