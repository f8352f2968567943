"""TEST INFRASTRUCTURE ONLY -- ctypes loaders for the parity oracle.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
``--impl reference`` arm) import this module, and only as the checker or the
timed reference CPU path; the product (libwisp_b200.so) never calls it.

* ``Oracle``  -- oracle/_ref/liboracle.so: fp64 restatement (oracle.c).
* ``RefCPU``  -- oracle/_ref/libwisp_ref.so: the reference engine's own
  scalar/OpenMP CPU functions compiled in place (ref_harness.c). The
  ``avx512=True`` variant is the reference's AVX-512 build (timed only; its
  results are wrong, see the notes in ref_harness.c).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"

_P = C.c_void_p
_I = C.c_int
_D = C.c_double


class OrcMat(C.Structure):
    _fields_ = [("packed", _P), ("scales", _P), ("zeros", _P), ("rows", C.c_int32),
                ("cols", C.c_int32)]


class OrcExpert(C.Structure):
    _fields_ = [("mat", OrcMat * 3)]


class OrcMeta(C.Structure):
    _fields_ = [("packed_off", C.c_int64 * 3), ("scales_off", C.c_int64 * 3),
                ("zeros_off", C.c_int64 * 3), ("rows", C.c_int32 * 3), ("cols", C.c_int32 * 3),
                ("group_size", C.c_int32), ("total_bytes", C.c_int64)]


def _ptr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


class Oracle:
    def __init__(self, path: Path | None = None):
        path = path or REF_DIR / "liboracle.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        L = C.CDLL(str(path))
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_parse_header.restype = _I
        L.orc_parse_header.argtypes = [_P, C.c_size_t, _P]
        L.orc_dequant_n.argtypes = [C.POINTER(OrcMat), C.c_int64, _I, _P]
        L.orc_gemv_int4.argtypes = [C.POINTER(OrcMat), _I, _P, _P]
        L.orc_expert_ffn.argtypes = [C.POINTER(OrcExpert), _I, _P, _P, _D]
        L.orc_router_logits.argtypes = [_P, _I, _P, _P, _I, _I, _I, _P]
        L.orc_topk_softmax.argtypes = [_P, _I, _I, _P, _P, _P]
        L.orc_topk_sigmoid_grouped.argtypes = [_P, _I, _I, _I, _I, _D, _P, _P, _P]
        L.orc_moe_tokens.argtypes = [_I, _I, _P, _I, _P, _P, C.POINTER(OrcExpert),
                                     C.POINTER(OrcExpert), _P, _I, _P]
        self.L = L

    # -- building blocks ---------------------------------------------------
    @staticmethod
    def mat(packed, scales, zeros, rows, cols) -> tuple[OrcMat, list]:
        keep = [np.ascontiguousarray(packed, np.uint8), np.ascontiguousarray(scales, np.uint16),
                None if zeros is None else np.ascontiguousarray(zeros, np.uint16)]
        m = OrcMat(_ptr(keep[0]), _ptr(keep[1]), _ptr(keep[2]), rows, cols)
        return m, keep

    def expert(self, mats3) -> tuple[OrcExpert, list]:
        """mats3: three objects with packed/scales/zeros/rows/cols (blob.Int4Matrix)."""
        e = OrcExpert()
        keep = []
        for i, m in enumerate(mats3):
            om, k = self.mat(m.packed, m.scales, m.zeros, m.rows, m.cols)
            e.mat[i] = om
            keep += k
        return e, keep

    def parse_header(self, blob: bytes) -> dict | None:
        m = OrcMeta()
        raw = C.create_string_buffer(blob, len(blob))
        rc = self.L.orc_parse_header(raw, len(blob), C.byref(m))
        if rc != 0:
            return None
        return dict(packed_off=list(m.packed_off), scales_off=list(m.scales_off),
                    zeros_off=list(m.zeros_off), rows=list(m.rows), cols=list(m.cols),
                    group_size=m.group_size, total_bytes=m.total_bytes)

    def dequant(self, m, n: int, gs: int) -> np.ndarray:
        om, keep = self.mat(m.packed, m.scales, m.zeros, m.rows, m.cols)
        out = np.empty(n, np.float32)
        self.L.orc_dequant_n(C.byref(om), n, gs, _ptr(out))
        return out

    def gemv(self, m, gs: int, x: np.ndarray) -> np.ndarray:
        om, keep = self.mat(m.packed, m.scales, m.zeros, m.rows, m.cols)
        x = np.ascontiguousarray(x, np.float64)
        y = np.empty(m.rows, np.float64)
        self.L.orc_gemv_int4(C.byref(om), gs, _ptr(x), _ptr(y))
        return y

    def expert_ffn(self, mats3, gs: int, x: np.ndarray, weight: float = 1.0,
                   acc: np.ndarray | None = None) -> np.ndarray:
        e, keep = self.expert(mats3)
        x = np.ascontiguousarray(x, np.float64)
        acc = np.zeros(mats3[2].rows, np.float64) if acc is None else acc
        self.L.orc_expert_ffn(C.byref(e), gs, _ptr(x), _ptr(acc), weight)
        return acc

    def router_logits(self, W: np.ndarray, wtype: int, bias, x: np.ndarray) -> np.ndarray:
        """W: float32 (wtype 0) or uint16 fp16/bf16 bits (1/2), [E, M]; x [T, M]."""
        E, M = W.shape
        x = np.ascontiguousarray(x, np.float64).reshape(-1, M)
        T = x.shape[0]
        W = np.ascontiguousarray(W)
        b = None if bias is None else np.ascontiguousarray(bias, np.float64)
        out = np.empty((T, E), np.float64)
        self.L.orc_router_logits(_ptr(W), wtype, _ptr(b), _ptr(x), T, E, M, _ptr(out))
        return out

    def topk(self, logits: np.ndarray, k: int, scoring: int = 0, n_groups: int = 1,
             topk_groups: int = 1, scaling: float = 1.0):
        """Per-token routing: (idx [T,k] int32, w [T,k] f64, margin [T] f64)."""
        logits = np.ascontiguousarray(logits, np.float64)
        T, E = logits.shape
        idx = np.empty((T, k), np.int32)
        w = np.empty((T, k), np.float64)
        mg = np.empty(T, np.float64)
        for t in range(T):
            row = logits[t]
            ip, wp, mp = (idx[t].ctypes.data, w[t].ctypes.data,
                          mg[t:t + 1].ctypes.data)
            if scoring == 0:
                self.L.orc_topk_softmax(row.ctypes.data, E, k, ip, wp, mp)
            else:
                self.L.orc_topk_sigmoid_grouped(row.ctypes.data, E, n_groups, topk_groups, k,
                                                scaling, ip, wp, mp)
        return idx, w, mg

    def moe_tokens(self, M: int, gs: int, x: np.ndarray, idx: np.ndarray, w: np.ndarray,
                   experts: list, shared, tokens: list[int]) -> np.ndarray:
        """out[j] = routed + shared expert outputs of token tokens[j] (fp64)."""
        x = np.ascontiguousarray(x, np.float64)
        idx = np.ascontiguousarray(idx, np.int32)
        w = np.ascontiguousarray(w, np.float64)
        k = idx.shape[1]
        arr = (OrcExpert * len(experts))()
        keep = []
        for i, mats in enumerate(experts):
            if mats is None:
                continue
            e, kk = self.expert(mats)
            arr[i] = e
            keep += kk
        sh = None
        if shared is not None:
            sh, kk = self.expert(shared)
            keep += kk
        tok = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((len(tokens), M), np.float64)
        self.L.orc_moe_tokens(M, gs, _ptr(x), k, _ptr(idx), _ptr(w), arr,
                              C.byref(sh) if sh is not None else None, _ptr(tok), len(tokens),
                              _ptr(out))
        return out


class RefCPU:
    """The reference engine's CPU hot path (compiled from its own sources)."""

    def __init__(self, avx512: bool = False, threads: int | None = None):
        """threads: OpenMP threads for the reference's parallel loops; None
        keeps the runtime's default (OMP_NUM_THREADS or all cores)."""
        name = "libwisp_ref_avx512.so" if avx512 else "libwisp_ref.so"
        path = REF_DIR / name
        if not path.exists():
            raise FileNotFoundError(f"{path} missing (built from the reference sources by "
                                    "`make -C oracle` where they are present)")
        L = C.CDLL(str(path))
        L.ref_gemv_int4.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I]
        L.ref_gemv_f16.argtypes = [_P, _P, _P, _I, _I]
        L.ref_swiglu.argtypes = [_P, _P, _P, _I]
        L.ref_scale_accum.argtypes = [_P, _P, C.c_float, _I]
        L.ref_router_topk.argtypes = [_P, _P, _P, _P, _I, _I, _I, _P, _P]
        L.ref_parse_header.restype = _I
        L.ref_parse_header.argtypes = [_P, C.c_size_t, _P]
        L.ref_expert_ffn.restype = _I
        L.ref_expert_ffn.argtypes = [_P, C.c_size_t, _P, _P, C.c_float]
        L.ref_moe_token.restype = _I
        L.ref_moe_token.argtypes = [_P, _P, _P, _I, _I, C.POINTER(_P), C.c_size_t, _P, _P, _P, _P]
        L.ref_half_to_float.restype = C.c_float
        L.ref_half_to_float.argtypes = [C.c_uint16]
        L.ref_omp_threads.restype = _I
        L.ref_set_threads.restype = None
        L.ref_set_threads.argtypes = [_I]
        self.L = L
        if threads is not None:
            L.ref_set_threads(int(threads))

    @staticmethod
    def available(avx512: bool = False) -> bool:
        name = "libwisp_ref_avx512.so" if avx512 else "libwisp_ref.so"
        if not (REF_DIR / name).exists():
            return False
        if avx512:
            try:
                flags = Path("/proc/cpuinfo").read_text()
            except OSError:
                return False
            return "avx512f" in flags and "avx512bw" in flags and "avx512vl" in flags
        return True

    def threads(self) -> int:
        return self.L.ref_omp_threads()

    @staticmethod
    def host_cores() -> int:
        """Cores this process may run on (its CPU affinity set)."""
        try:
            return len(os.sched_getaffinity(0))
        except (AttributeError, OSError):
            return os.cpu_count() or 1

    def parse_header(self, blob: bytes) -> dict | None:
        buf = (C.c_int64 * 20)()
        raw = C.create_string_buffer(blob, len(blob))
        rc = self.L.ref_parse_header(raw, len(blob), buf)
        if rc != 0:
            return None
        v = list(buf)
        return dict(packed_off=v[0:3], scales_off=v[3:6], zeros_off=v[6:9], rows=v[9:12],
                    cols=v[12:15], group_size=v[15], total_bytes=v[16])

    def gemv_int4(self, m, gs: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(m.rows, np.float32)
        z = m.zeros if m.zeros is not None else np.zeros_like(m.scales)
        self.L.ref_gemv_int4(_ptr(np.ascontiguousarray(m.packed)), _ptr(np.ascontiguousarray(m.scales)),
                             _ptr(np.ascontiguousarray(z)), _ptr(x), _ptr(y), m.rows, m.cols, gs)
        return y

    def router_topk(self, W16: np.ndarray, bias16, x: np.ndarray, k: int):
        """W16: fp16 bits [E, M]; x fp32 [M]; returns (idx, w)."""
        E, M = W16.shape
        W16 = np.ascontiguousarray(W16, np.uint16)
        x = np.ascontiguousarray(x, np.float32)
        logits = np.empty(E, np.float32)
        idx = np.empty(k, np.int32)
        w = np.empty(k, np.float32)
        b = None if bias16 is None else np.ascontiguousarray(bias16, np.uint16)
        self.L.ref_router_topk(_ptr(W16), _ptr(b), _ptr(x), _ptr(logits), E, M, k, _ptr(idx), _ptr(w))
        return idx, w

    def expert_ffn(self, blob: bytes, x: np.ndarray, acc: np.ndarray, weight: float) -> None:
        raw = np.frombuffer(blob, np.uint8)
        x = np.ascontiguousarray(x, np.float32)
        rc = self.L.ref_expert_ffn(_ptr(raw), len(blob), _ptr(x), _ptr(acc), weight)
        if rc != 0:
            raise RuntimeError(f"reference expert_ffn failed: {rc}")

    def moe_token(self, W16: np.ndarray, bias16, x: np.ndarray, k: int, blobs: list[np.ndarray],
                  shared: np.ndarray | None):
        """One token through the reference's CPU run_moe branch. blobs: uint8
        arrays (one per routed expert, same size). Returns (out, idx, w)."""
        E, M = W16.shape
        W16 = np.ascontiguousarray(W16, np.uint16)
        x = np.ascontiguousarray(x, np.float32)
        arr = (_P * E)(*[b.ctypes.data for b in blobs])
        out = np.empty(M, np.float32)
        idx = np.empty(k, np.int32)
        w = np.empty(k, np.float32)
        b = None if bias16 is None else np.ascontiguousarray(bias16, np.uint16)
        rc = self.L.ref_moe_token(_ptr(W16), _ptr(b), _ptr(x), E, k, arr, blobs[0].size,
                                  None if shared is None else shared.ctypes.data, _ptr(out),
                                  _ptr(idx), _ptr(w))
        if rc != 0:
            raise RuntimeError(f"reference moe_token failed: {rc}")
        return out, idx, w
