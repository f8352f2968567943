"""Expert parallelism: routed experts sharded across GPUs, tokens exchanged
with NCCL all-to-all (dispatch) and back (combine).

The reference engine binds a single GPU (csrc/core/wisp_engine.c:2045-2053)
and has no expert parallelism; this is new functionality whose results must
equal the single-GPU path's. Layout:

* expert e lives on rank floor(e * N / E) (contiguous blocks of E / N);
  the shared expert and the router are replicated;
* each rank owns a contiguous slice of the tokens.

One layer on rank r:
  route own tokens -> plan (rows grouped by expert, hence by owner rank)
  -> pack rows (fp16) -> exchange per-expert row counts (all_to_all) ->
  dispatch rows (all_to_all_v) -> grouped FFN over the received rows,
  grouped expert-major (mode 1: unweighted fp32 rows) -> return rows
  (all_to_all_v) -> shared expert on own tokens (mode 0) + weighted combine
  of the returned rows.

Collectives go through torch.distributed (NCCL between GPUs); every rank
issues the same collectives in the same order. The compute steps go through
an ``ops`` object -- :class:`CudaOps` (the C ABI) in production; the CPU
tests substitute a host implementation to exercise the exchange logic with
the gloo backend.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

from . import abi
from .synth import LayerWeights, MoeSpec


def block_range(n: int, world: int, rank: int) -> tuple[int, int]:
    return n * rank // world, n * (rank + 1) // world


def send_splits(counts: np.ndarray, n_experts: int, world: int) -> list[int]:
    """Rows this rank sends to each destination (its rows are sorted by expert)."""
    return [int(counts[slice(*block_range(n_experts, world, q))].sum()) for q in range(world)]


def recv_layout(recv_counts: np.ndarray) -> tuple[list[tuple[int, int, int]], list[int]]:
    """recv_counts[s, e]: rows source s sends for local expert e. The receive
    buffer holds source blocks in rank order, each sorted by expert. Returns
    segments (local_expert, row_begin, rows) ordered expert-major (so tiles
    of one expert are adjacent and share its weights in L2) and the per-source
    row counts."""
    world, e_loc = recv_counts.shape
    per_src = recv_counts.sum(axis=1)
    base = np.concatenate([[0], np.cumsum(per_src)[:-1]])
    inner = np.concatenate([np.zeros((world, 1), np.int64), np.cumsum(recv_counts, axis=1)[:, :-1]], axis=1)
    segs = []
    for e in range(e_loc):
        for s in range(world):
            segs.append((e, int(base[s] + inner[s, e]), int(recv_counts[s, e])))
    return segs, [int(v) for v in per_src]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _segments_tensor(segs, device) -> torch.Tensor:
    arr = (abi.WispSegment * max(1, len(segs)))()
    for i, (e, b, r) in enumerate(segs):
        arr[i].expert, arr[i].row_begin, arr[i].rows = e, b, r
    return torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(device, non_blocking=True)


class CudaOps:
    """Compute steps of one EP layer on the GPU, through libwisp_b200.so."""

    def route(self, cfg, lw: LayerWeights, x, idx, w, logits):
        ws = lw.weights_struct()
        abi.call("wisp_b200_route", C.byref(cfg), C.byref(ws), x.data_ptr(), logits.data_ptr(),
                 idx.data_ptr(), w.data_ptr(), _stream())

    def plan(self, cfg, idx, w, counts, segs, row_token, row_weight):
        abi.call("wisp_b200_dispatch_plan", C.byref(cfg), idx.data_ptr(), w.data_ptr(),
                 counts.data_ptr(), segs.data_ptr(), row_token.data_ptr(), row_weight.data_ptr(),
                 _stream())

    def pack(self, x, src, n_rows, xp):
        abi.call("wisp_b200_pack_rows", x.data_ptr(), None if src is None else src.data_ptr(),
                 n_rows, x.shape[1], xp.data_ptr(), _stream())

    def grouped(self, cfg, lw, segs, rows, xp, h, mode, row_token, row_weight, out, tiles, flag):
        dsegs = _segments_tensor(segs, xp.device)
        abi.call("wisp_b200_grouped_ffn", C.byref(cfg), lw.prepare().data_ptr(), lw.table.data_ptr(),
                 lw.n_entries,
                 dsegs.data_ptr(), len(segs),
                 max(rows, 1), xp.data_ptr(), h.data_ptr(), mode,
                 None if row_token is None else row_token.data_ptr(),
                 None if row_weight is None else row_weight.data_ptr(), out.data_ptr(),
                 tiles.data_ptr(), flag.data_ptr(), _stream())

    def combine(self, y, row_token, row_weight, n_rows, out):
        abi.call("wisp_b200_combine_rows", y.data_ptr(), row_token.data_ptr(), row_weight.data_ptr(),
                 n_rows, out.shape[1], out.data_ptr(), _stream())

    def act_dtype(self):
        return torch.float16


class EpLayer:
    """One MoE layer whose routed experts are sharded over the process group.

    ``lw`` holds this rank's experts only: local expert i is global expert
    e0 + i, and the shared expert (if any) is local index E_loc. The router
    weight is the full one."""

    def __init__(self, spec: MoeSpec, lw: LayerWeights, tokens: int, rank: int, world: int,
                 group=None, ops=None, device=None):
        assert spec.n_experts % world == 0, "experts must split evenly over the ranks"
        self.spec, self.lw, self.T, self.rank, self.world = spec, lw, tokens, rank, world
        self.group = group
        self.ops = ops or CudaOps()
        self.dev = device if device is not None else lw.router_w.device
        self.e0, self.e1 = block_range(spec.n_experts, world, rank)
        self.e_loc = self.e1 - self.e0
        k, M, I = spec.top_k, spec.hidden, spec.inter
        T = tokens
        # Routing over the full expert set, without the shared expert (it is
        # computed locally, never dispatched).
        self.cfg_route = spec.cfg(T)
        self.cfg_route.has_shared = 0
        # Local expert table: e_loc routed experts (+ shared at index e_loc).
        self.cfg_loc = spec.cfg(T)
        self.cfg_loc.n_experts = self.e_loc
        dev = self.dev
        adt = self.ops.act_dtype()
        self.idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        self.w = torch.empty((T, k), dtype=torch.float32, device=dev)
        self.logits = torch.empty((T, spec.n_experts), dtype=torch.float32, device=dev)
        self.counts = torch.empty(spec.n_experts, dtype=torch.int32, device=dev)
        self.segs = torch.empty(16 * spec.n_experts, dtype=torch.uint8, device=dev)
        self.row_token = torch.empty(T * k, dtype=torch.int32, device=dev)
        self.row_weight = torch.empty(T * k, dtype=torch.float32, device=dev)
        self.xp = torch.empty((T * k, M), dtype=adt, device=dev)
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        nseg_max = max(self.e_loc * world, 1) + 1
        self.tiles = torch.empty(abi.lib().wisp_b200_tiles_words(nseg_max) if adt == torch.float16 else 1,
                                 dtype=torch.int32, device=dev)
        # Worst case every token of every rank routes all k slots here.
        self.cap = T * k * world
        self.xr = torch.empty((self.cap, M), dtype=adt, device=dev)
        self.hr = torch.empty((max(self.cap, T), I), dtype=adt, device=dev)
        self.yr = torch.empty((self.cap, M), dtype=torch.float32, device=dev)
        self.yret = torch.empty((T * k, M), dtype=torch.float32, device=dev)
        if spec.has_shared:
            self.xs = torch.empty((T, M), dtype=adt, device=dev)
            self.sh_token = torch.arange(T, dtype=torch.int32, device=dev)
            self.sh_weight = torch.ones(T, dtype=torch.float32, device=dev)

    def forward(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """x: bf16 [T, M] (this rank's tokens) -> out fp32 [T, M]."""
        spec, ops, T, k, world = self.spec, self.ops, self.T, self.spec.top_k, self.world
        ops.route(self.cfg_route, self.lw, x, self.idx, self.w, self.logits)
        ops.plan(self.cfg_route, self.idx, self.w, self.counts, self.segs, self.row_token,
                 self.row_weight)
        ops.pack(x, self.row_token, T * k, self.xp)
        # 1. per-expert row counts to the owners (fixed-size exchange)
        cnt_recv = torch.empty(self.e_loc * world, dtype=torch.int32, device=self.dev)
        dist.all_to_all_single(cnt_recv, self.counts, group=self.group)
        counts_h = self.counts.cpu().numpy()
        recv_counts = cnt_recv.cpu().numpy().reshape(world, self.e_loc).astype(np.int64)
        send = send_splits(counts_h, spec.n_experts, world)
        segs, recv = recv_layout(recv_counts)
        R = sum(recv)
        # 2. dispatch rows
        dist.all_to_all_single(self.xr[:R], self.xp[:T * k], output_split_sizes=recv,
                               input_split_sizes=send, group=self.group)
        # 3. local experts over the received rows (unweighted fp32 rows)
        if R > 0:
            ops.grouped(self.cfg_loc, self.lw, segs, R, self.xr, self.hr, 1, None, None,
                        self.yr, self.tiles, self.flag)
        # 4. return rows to their tokens' ranks
        dist.all_to_all_single(self.yret, self.yr[:R], output_split_sizes=send,
                               input_split_sizes=recv, group=self.group)
        # 5. shared expert on own tokens, then the weighted combine
        out.zero_()
        if spec.has_shared:
            ops.pack(x, None, T, self.xs)
            ops.grouped(self.cfg_loc, self.lw, [(self.e_loc, 0, T)], T, self.xs, self.hr, 0,
                        self.sh_token, self.sh_weight, out, self.tiles, self.flag)
        ops.combine(self.yret, self.row_token, self.row_weight, T * k, out)
        return out
