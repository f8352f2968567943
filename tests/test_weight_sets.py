"""Weight-set entry points: the int4 dense MLP, expert-table entries made
from reference blobs, and one-slot preparation (the VRAM-promotion hook).

* wisp_b200_dense_mlp -- the MLP of a dense layer (csrc/core/wisp_engine.c:
  1676-1686, fp16 there) quantised to int4 and run through the grouped
  kernels as one segment: checked against the fp64 oracle at token counts
  that put the segment on the register path (<= 32 rows) and on tcgen05.
* wisp_b200_blob_expert -- table entries pointing into reference blobs
  (wisp/converter/partitioner.py layout), used by the batched layer directly:
  a layer whose experts are reference blobs (with zero points) at 8 mod 16
  equals the oracle on the same blobs.
* wisp_b200_prepare_expert_slot -- a prepared set built one slot at a time,
  in any order, is byte-identical to wisp_b200_prepare_experts over the
  whole table; re-preparing a slot after its blob moved gives the set of
  the new table.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from wisp_b200 import abi, synth
from wisp_b200.blob import pack_blob, parse_blob
from wisp_b200.moe import parse_header

from helpers import assert_close, bf16_to_f64

DEV = "cuda"


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _rand_mats(rng, M, I, gs, zeros):
    from wisp_b200.blob import Int4Matrix

    def mat(rows, cols):
        n = rows * cols
        return Int4Matrix(rng.integers(0, 256, n // 2, dtype=np.uint8),
                          np.float16(rng.uniform(0.004, 0.02, n // gs)).view(np.uint16),
                          np.float16(rng.uniform(-0.01, 0.01, n // gs)).view(np.uint16)
                          if zeros else None, rows, cols)
    return [mat(I, M), mat(I, M), mat(M, I)]


def _blobs_on_device(blobs: list[bytes]) -> tuple[torch.Tensor, list[int]]:
    """All blobs in one device buffer, each at an address = 8 mod 16."""
    size = max(len(b) for b in blobs)
    stride = (size + 16 + 255) // 256 * 256
    buf = torch.zeros(stride * len(blobs) + 256, dtype=torch.uint8, device=DEV)
    base = buf.data_ptr()
    first = (8 - base) % 16
    addrs = []
    for i, b in enumerate(blobs):
        off = first + i * stride
        buf[off:off + len(b)] = torch.frombuffer(bytearray(b), dtype=torch.uint8).to(DEV)
        addrs.append(base + off)
    return buf, addrs


def _entry(meta, addr) -> abi.WispInt4Expert:
    ent = abi.WispInt4Expert()
    abi.call("wisp_b200_blob_expert", C.byref(meta), C.c_void_p(addr), C.byref(ent))
    return ent


def _table(entries) -> torch.Tensor:
    arr = (abi.WispInt4Expert * len(entries))(*entries)
    return torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(DEV)


def _prepare_all(cfg, table, n) -> torch.Tensor:
    nb = abi.lib().wisp_b200_prepared_bytes(C.byref(cfg), n)
    prep = torch.zeros(nb, dtype=torch.uint8, device=DEV)
    abi.call("wisp_b200_prepare_experts", C.byref(cfg), table.data_ptr(), n, prep.data_ptr(), nb,
             _stream())
    return prep


def _prepare_slots(cfg, entries, order) -> torch.Tensor:
    n = len(entries)
    nb = abi.lib().wisp_b200_prepared_bytes(C.byref(cfg), n)
    prep = torch.zeros(nb, dtype=torch.uint8, device=DEV)
    for v in order:
        abi.call("wisp_b200_prepare_expert_slot", C.byref(cfg), n, int(v), C.byref(entries[v]),
                 prep.data_ptr(), nb, _stream())
    return prep


# ---------------------------------------------------------------------------
# Dense int4 MLP
# ---------------------------------------------------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("zeros", [False, True])
@pytest.mark.parametrize("T", [1, 7, 32, 33, 200])
def test_dense_mlp_matches_oracle(orc, T, zeros):
    spec = synth.MoeSpec("dense", 512, 384, 1, 1, group_size=128, tokens=T, seed=41)
    lw = synth.make_model(spec, DEV, zeros=zeros)[0][0]
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn((T, spec.hidden), generator=g, device=DEV).to(torch.bfloat16)
    cfg = spec.cfg(T)
    nb = abi.lib().wisp_b200_dense_mlp_workspace_bytes(C.byref(cfg))
    assert nb > 0
    ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
    out = torch.full((T, spec.hidden), float("nan"), dtype=torch.float32, device=DEV)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(2):   # a second call over the same workspace gives the same rows
        abi.call("wisp_b200_dense_mlp", C.byref(cfg), lw.prepare().data_ptr(), lw.table.data_ptr(),
                 x.data_ptr(), out.data_ptr(), ws.data_ptr(), nb, flag.data_ptr(), _stream())
        abi.call("wisp_b200_check_error_flag", flag.data_ptr(), _stream())
        got = out.cpu().numpy()
        mats = lw.expert_host(0)
        xs = bf16_to_f64(x)
        rows = range(T) if T <= 40 else range(0, T, 7)
        ref = np.stack([orc.expert_ffn(mats, spec.group_size, xs[t]) for t in rows])
        assert_close(got[list(rows)], ref, what=f"dense T={T}")


def test_dense_mlp_rejects_bad_shapes():
    """Shape checks run before any launch (no GPU needed)."""
    cfg = synth.MoeSpec("dense", 500, 384, 1, 1, tokens=4).cfg(4)
    assert abi.lib().wisp_b200_dense_mlp_workspace_bytes(C.byref(cfg)) == 0
    err = abi.WispErrCtx()
    rc = abi.lib().wisp_b200_dense_mlp(C.byref(cfg), 256, 256, 256, 256, 256, 1 << 20, None, None,
                                       C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG and b"multiples of 128" in err.message


# ---------------------------------------------------------------------------
# Reference blobs as table entries; one-slot preparation
# ---------------------------------------------------------------------------

def test_blob_expert_entry_offsets():
    """Host-only pointer arithmetic (no GPU): the entry points at the blob's
    matrices; zero points only when the blob carries them; misplaced blobs
    are rejected."""
    rng = np.random.default_rng(2)
    M, I, gs = 256, 128, 64
    for zeros in (True, False):
        blob = pack_blob(*_rand_mats(rng, M, I, gs, zeros), group_size=gs, write_zeros=zeros)
        meta = parse_header(blob)
        bm = parse_blob(blob)
        base = 0x10000008   # = 8 mod 16: packed data at +120 is 16-byte aligned
        ent = _entry(meta, base)
        for m, mat in enumerate((ent.gate, ent.up, ent.down)):
            assert mat.packed == base + bm.packed_off[m]
            assert mat.scales == base + bm.scales_off[m]
            assert mat.zeros == (base + bm.zeros_off[m] if zeros else None)
        err = abi.WispErrCtx()
        rc = abi.lib().wisp_b200_blob_expert(C.byref(meta), C.c_void_p(0x10000000), C.byref(ent),
                                             C.byref(err))
        assert rc == abi.WISP_ERR_INVALID_ARG and b"8 mod 16" in err.message


@pytest.mark.gpu
def test_slot_prepared_set_equals_whole_set_and_follows_moved_blobs(orc):
    rng = np.random.default_rng(11)
    M, I, E, k, gs, T = 512, 256, 12, 3, 128, 70
    mats = [_rand_mats(rng, M, I, gs, zeros=True) for _ in range(E)]
    blobs = [pack_blob(*m, group_size=gs) for m in mats]
    buf, addrs = _blobs_on_device(blobs)
    meta = parse_header(blobs[0])
    entries = [_entry(meta, a) for a in addrs]
    spec = synth.MoeSpec("blobs", M, I, E, k, group_size=gs, tokens=T, seed=3)
    cfg = spec.cfg(T)
    table = _table(entries)
    whole = _prepare_all(cfg, table, E)
    slots = _prepare_slots(cfg, entries, rng.permutation(E))
    torch.cuda.synchronize()
    assert torch.equal(whole, slots), "slot-by-slot preparation differs from the whole set"

    # the batched layer on those blobs equals the oracle on the same blobs
    router = (torch.randn((E, M), generator=torch.Generator().manual_seed(4)) * 0.05).to(
        torch.bfloat16).to(DEV)
    x = torch.randn((T, M), generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).to(DEV)

    def forward(tab, prep):
        w = abi.WispMoeWeights()
        w.router_w, w.router_bias = router.data_ptr(), None
        w.experts, w.prepared = tab.data_ptr(), prep.data_ptr()
        nb = abi.lib().wisp_b200_moe_workspace_bytes(C.byref(cfg))
        ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
        out = torch.empty((T, M), dtype=torch.float32, device=DEV)
        idx = torch.empty((T, k), dtype=torch.int32, device=DEV)
        wt = torch.empty((T, k), dtype=torch.float32, device=DEV)
        abi.call("wisp_b200_moe_forward", C.byref(cfg), C.byref(w), x.data_ptr(), out.data_ptr(),
                 idx.data_ptr(), wt.data_ptr(), ws.data_ptr(), nb, _stream())
        abi.call("wisp_b200_check_error_flag",
                 abi.lib().wisp_b200_moe_error_word(C.byref(cfg), ws.data_ptr()), _stream())
        return out.cpu().numpy(), idx.cpu().numpy(), wt.cpu().numpy().astype(np.float64)

    out, idx, wt = forward(table, slots)
    experts = [[m for m in e] for e in mats]
    tokens = list(range(0, T, 3))
    ref = orc.moe_tokens(M, gs, bf16_to_f64(x), idx, wt, experts, None, tokens)
    assert_close(out[tokens], ref, what="reference blobs via slot-prepared set")

    # three blobs move (an eviction and a later promotion elsewhere): only
    # their slots are re-prepared, and the set equals the new whole set
    buf2, addrs2 = _blobs_on_device(blobs)
    moved = [1, 5, 9]
    for v in moved:
        entries[v] = _entry(meta, addrs2[v])
        abi.call("wisp_b200_prepare_expert_slot", C.byref(cfg), E, v, C.byref(entries[v]),
                 slots.data_ptr(), slots.numel(), _stream())
    table2 = _table(entries)
    whole2 = _prepare_all(cfg, table2, E)
    torch.cuda.synchronize()
    assert torch.equal(whole2, slots)
    out2, idx2, _ = forward(table2, slots)
    np.testing.assert_array_equal(idx2, idx)
    assert_close(out2, out, 1e-5, 1e-6, "after the blobs moved")
