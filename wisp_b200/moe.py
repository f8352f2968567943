"""Python face of the batched MoE layer and the fused decode entry.

Thin wrappers over the C ABI (include/wisp_b200.h): tensors are PyTorch CUDA
tensors used as device memory; every launch goes on the current torch
stream. The work itself runs in libwisp_b200.so.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import abi
from .synth import LayerWeights, MoeSpec


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class MoeLayer:
    """One routed-expert MoE layer over int4 weights (router, dispatch,
    grouped gate/up + SwiGLU, grouped down + weighted combine)."""

    def __init__(self, weights: LayerWeights, tokens: int, deterministic: bool = False):
        """deterministic: sum each token's expert outputs in a fixed order, so
        that repeated calls give the same bits (WispMoeConfig.deterministic)."""
        self.w = weights
        self.spec: MoeSpec = weights.spec
        self.cfg = self.spec.cfg(tokens)
        self.cfg.deterministic = 1 if deterministic else 0
        weights.prepare()
        self._wstruct = weights.weights_struct()
        nbytes = abi.lib().wisp_b200_moe_workspace_bytes(C.byref(self.cfg))
        if nbytes == 0:
            raise RuntimeError(f"wisp engine error [{abi.WISP_ERR_INVALID_ARG}]: invalid MoE config")
        dev = weights.router_w.device
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        T, k = tokens, self.spec.top_k
        self.idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        self.wt = torch.empty((T, k), dtype=torch.float32, device=dev)

    @property
    def tokens(self) -> int:
        return self.cfg.tokens

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        assert x.dtype == torch.bfloat16 and x.is_contiguous() and x.shape == (self.tokens, self.spec.hidden)
        if out is None:
            out = torch.empty((self.tokens, self.spec.hidden), dtype=torch.float32, device=x.device)
        abi.call("wisp_b200_moe_forward", C.byref(self.cfg), C.byref(self._wstruct), x.data_ptr(),
                 out.data_ptr(), self.idx.data_ptr(), self.wt.data_ptr(), self.workspace.data_ptr(),
                 self.workspace.numel(), _stream())
        return out

    def error_flag_ptr(self) -> int:
        """Device error word inside the workspace (see wisp_b200_check_error_flag)."""
        return abi.lib().wisp_b200_moe_error_word(C.byref(self.cfg), self.workspace.data_ptr())

    def check(self) -> None:
        """Raise if a tensor-core kernel of the last forward gave up waiting."""
        abi.call("wisp_b200_check_error_flag", self.error_flag_ptr(), _stream())


def expert_ffn_decode(meta: abi.WispExpertMeta, blob_ptrs: list[int], weights: list[float],
                      x: torch.Tensor, acc: torch.Tensor, scratch: torch.Tensor) -> None:
    """acc += sum_j weights[j] * expert_j(x) for one token at fp32 (the fused
    replacement of the reference's gpu_expert_ffn loop)."""
    n = len(blob_ptrs)
    ptrs = (C.c_void_p * n)(*blob_ptrs)
    ws = (C.c_float * n)(*weights)
    abi.call("wisp_b200_expert_ffn", C.byref(meta), ptrs, ws, n, x.data_ptr(), acc.data_ptr(),
             scratch.data_ptr(), scratch.numel() * scratch.element_size(), _stream())


def parse_header(blob: bytes) -> abi.WispExpertMeta:
    meta = abi.WispExpertMeta()
    buf = C.create_string_buffer(blob, len(blob))
    abi.call("wisp_b200_parse_expert_header", buf, len(blob), C.byref(meta))
    return meta
