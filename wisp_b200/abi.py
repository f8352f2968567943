"""ctypes view of include/wisp_b200.h.

Loads ``libwisp_b200.so`` from the package directory and declares every
entry point's argument types. Errors from the fused entry points are raised
as ``RuntimeError("wisp engine error [code]: message (file:line)")``, the
same form the reference's pybind layer uses (csrc/bindings/wisp_bindings.cpp:
53-60). There is no fallback: if the library is missing the import fails.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libwisp_b200.so"
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "wisp_b200.h"

WISP_OK = 0
WISP_ERR_OOM = 1
WISP_ERR_IO = 2
WISP_ERR_CUDA = 3
WISP_ERR_INVALID_ARG = 4
WISP_ERR_EXPERT_MISS = 5
WISP_ERR_MODEL = 6
WISP_ERR_TIMEOUT = 7

WISP_SCORE_SOFTMAX = 0
WISP_SCORE_SIGMOID_GROUPED = 1


class WispErrCtx(C.Structure):
    _fields_ = [("code", C.c_int), ("message", C.c_char * 512), ("file", C.c_char_p),
                ("line", C.c_int)]


class WispExpertMeta(C.Structure):
    _fields_ = [("packed_off", C.c_size_t * 3), ("scales_off", C.c_size_t * 3),
                ("zeros_off", C.c_size_t * 3), ("rows", C.c_uint32 * 3),
                ("cols", C.c_uint32 * 3), ("group_size", C.c_uint32),
                ("total_bytes", C.c_size_t), ("valid", C.c_int)]


class WispMoeConfig(C.Structure):
    _fields_ = [("tokens", C.c_int), ("hidden", C.c_int), ("inter", C.c_int),
                ("n_experts", C.c_int), ("top_k", C.c_int), ("group_size", C.c_int),
                ("scoring", C.c_int), ("n_groups", C.c_int), ("topk_groups", C.c_int),
                ("routed_scaling", C.c_float), ("has_shared", C.c_int),
                ("router_fp16", C.c_int), ("deterministic", C.c_int)]


class WispInt4Mat(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("zeros", C.c_void_p)]


class WispInt4Expert(C.Structure):
    _fields_ = [("gate", WispInt4Mat), ("up", WispInt4Mat), ("down", WispInt4Mat)]


class WispMoeWeights(C.Structure):
    _fields_ = [("router_w", C.c_void_p), ("router_bias", C.c_void_p), ("experts", C.c_void_p),
                ("prepared", C.c_void_p)]


class WispSegment(C.Structure):
    _fields_ = [("expert", C.c_int32), ("row_begin", C.c_int32), ("rows", C.c_int32),
                ("reserved", C.c_int32)]


assert C.sizeof(WispInt4Expert) == 72 and C.sizeof(WispSegment) == 16

_P = C.c_void_p
_I = C.c_int
_F = C.c_float
_SZ = C.c_size_t
_E = C.POINTER(WispErrCtx)

# name -> (restype, argtypes)
SIGNATURES = {
    "launch_dequant_expert": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "async_load_expert": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _P]),
    "wisp_gpu_gemv_f16": (None, [_P, _P, _P, _I, _I, _P]),
    "wisp_gpu_swiglu": (None, [_P, _P, _P, _I, _P]),
    "wisp_gpu_swiglu_ffn": (None, [_P, _P, _P, _P, _I, _I, _P]),
    "wisp_gpu_scale_accum": (None, [_P, _P, _F, _I, _P]),
    "wisp_gpu_router_topk": (None, [_P, _P, _P, _P, _I, _I, _I, _P, _P, _P]),
    "wisp_b200_parse_expert_header": (_I, [_P, _SZ, C.POINTER(WispExpertMeta), _E]),
    "wisp_b200_expert_ffn_scratch_bytes": (_SZ, [C.POINTER(WispExpertMeta), _I]),
    "wisp_b200_expert_ffn": (_I, [C.POINTER(WispExpertMeta), C.POINTER(_P), C.POINTER(_F), _I,
                                  _P, _P, _P, _SZ, _P, _E]),
    "wisp_b200_expert_ffn_noalloc": (_I, [C.POINTER(WispExpertMeta), C.POINTER(_P), C.POINTER(_F),
                                          _I, _P, _P, _P, _E]),
    "wisp_b200_moe_workspace_bytes": (_SZ, [C.POINTER(WispMoeConfig)]),
    "wisp_b200_moe_forward": (_I, [C.POINTER(WispMoeConfig), C.POINTER(WispMoeWeights), _P, _P,
                                   _P, _P, _P, _SZ, _P, _E]),
    "wisp_b200_route": (_I, [C.POINTER(WispMoeConfig), C.POINTER(WispMoeWeights), _P, _P, _P,
                             _P, _P, _E]),
    "wisp_b200_route_workspace_bytes": (_SZ, [C.POINTER(WispMoeConfig)]),
    "wisp_b200_route_ws": (_I, [C.POINTER(WispMoeConfig), C.POINTER(WispMoeWeights), _P, _P, _P,
                                _P, _P, _SZ, _P, _E]),
    "wisp_b200_grouped_workspace_bytes": (_SZ, [C.POINTER(WispMoeConfig), _I, _I]),
    "wisp_b200_grouped_ffn": (_I, [C.POINTER(WispMoeConfig), _P, _P, _I, _P, _I, _I, _P, _P, _I,
                                   _P, _P, _P, _P, _SZ, _P, _P, _E]),
    "wisp_b200_set_skinny_max_rows": (None, [_I]),
    "wisp_b200_prepared_bytes": (_SZ, [C.POINTER(WispMoeConfig), _I]),
    "wisp_b200_prepare_experts": (_I, [C.POINTER(WispMoeConfig), _P, _I, _P, _SZ, _P, _E]),
    "wisp_b200_prepare_expert_slot": (_I, [C.POINTER(WispMoeConfig), _I, _I,
                                           C.POINTER(WispInt4Expert), _P, _SZ, _P, _E]),
    "wisp_b200_blob_expert": (_I, [C.POINTER(WispExpertMeta), _P, C.POINTER(WispInt4Expert), _E]),
    "wisp_b200_dense_mlp_workspace_bytes": (_SZ, [C.POINTER(WispMoeConfig)]),
    "wisp_b200_dense_mlp": (_I, [C.POINTER(WispMoeConfig), _P, _P, _P, _P, _P, _SZ, _P, _P, _E]),
    "wisp_b200_pack_rows": (_I, [_P, _P, _I, _I, _P, _P, _E]),
    "wisp_b200_dispatch_plan": (_I, [C.POINTER(WispMoeConfig), _P, _P, _P, _P, _P, _P, _P, _E]),
    "wisp_b200_rms_rescale": (_I, [_P, _P, _I, _I, _F, _P, _E]),
    "wisp_b200_combine_rows": (_I, [_P, _P, _P, _I, _I, _P, _P, _E]),
    "wisp_b200_ep_block_bytes": (_SZ, [_I, _I, _I, _I]),
    "wisp_b200_ep_dispatch": (_I, [_P, _I, _I, _P, _I, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P,
                                   _E]),
    "wisp_b200_ep_recv_plan": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _E]),
    "wisp_b200_ep_gather_rows": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _P, _I, _I, _P, _P, _E]),
    "wisp_b200_ep_combine": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _E]),
    "wisp_b200_ep_combine_f16": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _E]),
    "wisp_b200_ep_return_rows": (_I, [_P, _I, _I, _P, _P, _E]),
    "wisp_b200_check_error_flag": (_I, [_P, _P, _E]),
    "wisp_b200_moe_error_word": (_P, [C.POINTER(WispMoeConfig), _P]),
    "wisp_b200_debug_set_counters": (None, [_P]),
    "wisp_b200_version": (C.c_char_p, []),
}


def header_functions() -> list[str]:
    """Function names declared in include/wisp_b200.h."""
    text = HEADER_PATH.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = "\n".join(l for l in text.splitlines() if not l.lstrip().startswith("#"))
    names = re.findall(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", text)
    skip = {"defined", "if", "sizeof"}
    decl = []
    for n in names:
        if n in skip or n.isupper():
            continue
        if n not in decl:
            decl.append(n)
    return decl


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m wisp_b200.build` "
                "(the CUDA path has no fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(code: int, err: WispErrCtx) -> None:
    if code != WISP_OK:
        msg = f"wisp engine error [{code}]: {err.message.decode(errors='replace')}"
        if err.file:
            msg += f" ({err.file.decode()}:{err.line})"
        raise RuntimeError(msg)


def call(name: str, *args) -> None:
    """Call a WispError-returning entry point with a fresh error context as
    its last argument; raise RuntimeError on failure."""
    err = WispErrCtx()
    code = getattr(lib(), name)(*args, C.byref(err))
    check(code, err)
