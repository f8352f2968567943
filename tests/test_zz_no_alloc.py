"""The allocation-free decode entry point (wisp_b200_expert_ffn_noalloc).

It serves callers that cannot allocate device memory -- an engine whose
VRAM budget is entirely given to the expert cache, or a host callback where
a cudaMalloc would synchronise the device -- by keeping the intermediate
activations in a fixed 227 KB array inside the library. These tests call it
through the C ABI and check it against the regular entry point (which takes
a caller buffer) on two calls in a row, so the second call runs on the
array the first one left behind. This file is collected last on purpose and
is self-contained, so it passes alone in a fresh process too.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from wisp_b200 import abi

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "moe_small.npz"
# the decode tests' tolerance (fp32 path): relative to the output magnitude
MAX_REL = 1e-4
MEAN_REL = 1e-4


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _blob_on_device(blob: bytes):
    buf = torch.empty(len(blob) + 64, dtype=torch.uint8, device="cuda")
    off = (8 - buf.data_ptr()) % 16          # packed data at +120 lands 16-byte aligned
    buf[off:off + len(blob)] = torch.frombuffer(bytearray(blob), dtype=torch.uint8).cuda()
    return buf, buf.data_ptr() + off


def _meta(blob: bytes) -> abi.WispExpertMeta:
    meta = abi.WispExpertMeta()
    abi.call("wisp_b200_parse_expert_header", blob, len(blob), C.byref(meta))
    return meta


def _rel(a, b):
    d = np.abs(a - b)
    return d.max() / np.abs(b).max(), d.mean() / np.abs(b).mean()


def test_noalloc_matches_regular_entry_on_consecutive_calls():
    g = np.load(GOLDEN)
    M, I, E, k, gs, T = (int(v) for v in g["dims"])
    blobs = [b.tobytes() for b in g["blobs"]]
    meta = _meta(blobs[0])
    dev = [_blob_on_device(b) for b in blobs]
    n = k + 1
    scratch = torch.empty(n * I, dtype=torch.float32, device="cuda")
    for t in (0, 1):   # two calls in a row, different tokens and experts
        ptrs = (C.c_void_p * n)(*([dev[int(e)][1] for e in g["idx"][t]] + [dev[E][1]]))
        wts = (C.c_float * n)(*([float(v) for v in g["w"][t]] + [1.0]))
        x = torch.from_numpy(g["x"][t]).float().cuda()
        ref = torch.zeros(M, device="cuda")
        got = torch.zeros(M, device="cuda")
        abi.call("wisp_b200_expert_ffn", C.byref(meta), ptrs, wts, n, x.data_ptr(), ref.data_ptr(),
                 scratch.data_ptr(), scratch.numel() * 4, _stream())
        abi.call("wisp_b200_expert_ffn_noalloc", C.byref(meta), ptrs, wts, n, x.data_ptr(),
                 got.data_ptr(), _stream())
        torch.cuda.synchronize()
        mr, me = _rel(got.cpu().numpy(), ref.cpu().numpy())
        assert mr <= MAX_REL and me <= MEAN_REL, (t, mr, me)
        # and against the reference engine's own CPU output for this token
        mr, me = _rel(got.cpu().numpy(), g["out"][t])
        assert mr <= MAX_REL and me <= MEAN_REL, (t, mr, me)


def test_noalloc_full_size_deepseek_decode_twice():
    """Nine DeepSeek-V3-shaped experts (8 routed + shared): 9 x 2048 floats
    of intermediate activations fit the built-in array."""
    rng = np.random.default_rng(5)
    M, I, gs = 7168, 2048, 128
    from wisp_b200.blob import Int4Matrix, pack_blob

    def mat(r, c):
        nn = r * c
        return Int4Matrix(rng.integers(0, 256, nn // 2, dtype=np.uint8),
                          np.float16(rng.uniform(0.004, 0.02, nn // gs)).view(np.uint16), None, r, c)

    blobs = [pack_blob(mat(I, M), mat(I, M), mat(M, I), gs) for _ in range(9)]
    meta = _meta(blobs[0])
    dev = [_blob_on_device(b) for b in blobs]
    ptrs = (C.c_void_p * 9)(*[d[1] for d in dev])
    wts = (C.c_float * 9)(*[float(v) for v in rng.uniform(0.05, 0.4, 9)])
    scratch = torch.empty(9 * I, dtype=torch.float32, device="cuda")
    for seed in (1, 2):
        x = torch.randn(M, generator=torch.Generator().manual_seed(seed)).cuda()
        ref = torch.zeros(M, device="cuda")
        got = torch.zeros(M, device="cuda")
        abi.call("wisp_b200_expert_ffn", C.byref(meta), ptrs, wts, 9, x.data_ptr(), ref.data_ptr(),
                 scratch.data_ptr(), scratch.numel() * 4, _stream())
        abi.call("wisp_b200_expert_ffn_noalloc", C.byref(meta), ptrs, wts, 9, x.data_ptr(),
                 got.data_ptr(), _stream())
        torch.cuda.synchronize()
        mr, me = _rel(got.cpu().numpy(), ref.cpu().numpy())
        assert mr <= MAX_REL and me <= MEAN_REL, (seed, mr, me)


def test_noalloc_rejects_sizes_beyond_the_array():
    # Mixtral-shaped: 5 x 14336 = 71680 floats > 58112
    meta = abi.WispExpertMeta()
    meta.rows[:] = [14336, 14336, 4096]
    meta.cols[:] = [4096, 4096, 14336]
    meta.group_size, meta.valid = 128, 1
    ptrs = (C.c_void_p * 5)(*([16] * 5))
    wts = (C.c_float * 5)(*([0.2] * 5))
    err = abi.WispErrCtx()
    rc = abi.lib().wisp_b200_expert_ffn_noalloc(C.byref(meta), ptrs, wts, 5, 16, 16, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
    assert b"exceeds the built-in scratch" in err.message


def test_noalloc_size_boundary():
    """The largest call the built-in array takes (16 experts x 3632 = 58112
    floats, the down kernel's shared-memory limit too) runs and matches the
    caller-buffer entry on two calls in a row; one more row block (16 x 3648)
    is rejected before any launch."""
    rng = np.random.default_rng(8)
    M, I, gs, n = 64, 3632, 16, 16
    from wisp_b200.blob import Int4Matrix, pack_blob

    def mat(r, c):
        nn = r * c
        return Int4Matrix(rng.integers(0, 256, nn // 2, dtype=np.uint8),
                          np.float16(rng.uniform(0.004, 0.02, nn // gs)).view(np.uint16), None, r, c)

    blobs = [pack_blob(mat(I, M), mat(I, M), mat(M, I), gs) for _ in range(n)]
    meta = _meta(blobs[0])
    dev = [_blob_on_device(b) for b in blobs]
    ptrs = (C.c_void_p * n)(*[d[1] for d in dev])
    wts = (C.c_float * n)(*[float(v) for v in rng.uniform(0.05, 0.4, n)])
    scratch = torch.empty(n * I, dtype=torch.float32, device="cuda")
    for seed in (3, 4):
        x = torch.randn(M, generator=torch.Generator().manual_seed(seed)).cuda()
        ref = torch.zeros(M, device="cuda")
        got = torch.zeros(M, device="cuda")
        abi.call("wisp_b200_expert_ffn", C.byref(meta), ptrs, wts, n, x.data_ptr(), ref.data_ptr(),
                 scratch.data_ptr(), scratch.numel() * 4, _stream())
        abi.call("wisp_b200_expert_ffn_noalloc", C.byref(meta), ptrs, wts, n, x.data_ptr(),
                 got.data_ptr(), _stream())
        torch.cuda.synchronize()
        mr, me = _rel(got.cpu().numpy(), ref.cpu().numpy())
        assert mr <= MAX_REL and me <= MEAN_REL, (seed, mr, me)
    big = abi.WispExpertMeta.from_buffer_copy(meta)
    big.rows[0] = big.rows[1] = 3648
    big.cols[2] = 3648
    err = abi.WispErrCtx()
    rc = abi.lib().wisp_b200_expert_ffn_noalloc(C.byref(big), ptrs, wts, n, 16, 16, None, C.byref(err))
    assert rc == abi.WISP_ERR_INVALID_ARG
    assert b"exceeds the built-in scratch" in err.message
