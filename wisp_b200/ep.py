"""Expert parallelism: routed experts sharded across GPUs, tokens exchanged
with NCCL all-to-all (dispatch) and back (combine).

The reference engine binds a single GPU (csrc/core/wisp_engine.c:2045-2053)
and has no expert parallelism; this is new functionality whose results must
equal the single-GPU path's. Layout:

* expert e lives on rank floor(e * N / E) (contiguous blocks of E / N);
  the shared expert and the router are replicated;
* each rank owns a contiguous slice of the tokens.

One layer on rank r, with every count kept on the device (no host round
trip between routing and the expert FFN):
  route own tokens -> plan (rows grouped by expert, hence by owner rank)
  -> pack rows (fp16) into a send buffer of `world` fixed blocks of `cap`
  rows -> exchange per-expert row counts and the row blocks (all_to_all,
  equal splits), meanwhile the shared expert on own tokens (mode 0) -> gather
  the received rows expert-contiguous (one segment per local expert, as on
  one GPU) -> grouped FFN (mode 1: unweighted fp32 rows) -> scatter the
  results into the source blocks -> return the row blocks (all_to_all) ->
  weighted combine of the returned rows.
cap = tokens * top_k, the most rows one rank can send to one destination;
the padding rows are exchanged but never computed or read.

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

    def send_pack(self, x, row_token, plan_segs, n_experts, n_rows, world, cap, xsend, slot):
        abi.call("wisp_b200_ep_send_pack", x.data_ptr(), x.shape[1], row_token.data_ptr(),
                 plan_segs.data_ptr(), n_experts, n_rows, world, cap, xsend.data_ptr(),
                 slot.data_ptr(), _stream())

    def recv_plan(self, recv_counts, world, e_loc, cap, segs, src_pos, total):
        abi.call("wisp_b200_ep_recv_plan", recv_counts.data_ptr(), world, e_loc, cap,
                 segs.data_ptr(), src_pos.data_ptr(), total.data_ptr(), _stream())

    def gather_rows(self, recv, src_pos, total, max_rows, sorted_rows):
        abi.call("wisp_b200_ep_gather_rows", recv.data_ptr(), src_pos.data_ptr(), total.data_ptr(),
                 max_rows, recv.shape[1], sorted_rows.data_ptr(), _stream())

    def scatter_rows(self, sorted_rows, src_pos, total, max_rows, recv):
        abi.call("wisp_b200_ep_scatter_rows", sorted_rows.data_ptr(), src_pos.data_ptr(),
                 total.data_ptr(), max_rows, recv.shape[1], recv.data_ptr(), _stream())

    def grouped_dev(self, cfg, lw, segs, n_segs, rows, xp, h, mode, row_token, row_weight, out,
                    tiles, flag):
        abi.call("wisp_b200_grouped_ffn", C.byref(cfg), lw.prepare().data_ptr(), lw.table.data_ptr(),
                 lw.n_entries, segs.data_ptr(), n_segs, max(rows, 1), xp.data_ptr(), h.data_ptr(),
                 mode, None if row_token is None else row_token.data_ptr(),
                 None if row_weight is None else row_weight.data_ptr(), out.data_ptr(),
                 tiles.data_ptr(), flag.data_ptr(), _stream())

    def ep_combine(self, y, slot, row_token, row_weight, n_rows, out):
        abi.call("wisp_b200_ep_combine", y.data_ptr(), slot.data_ptr(), row_token.data_ptr(),
                 row_weight.data_ptr(), n_rows, out.shape[1], out.data_ptr(), _stream())

    def act_dtype(self):
        return torch.float16


class EpLayer:
    """One MoE layer whose routed experts are sharded over the process group.

    ``lw`` holds this rank's experts only: local expert i is global expert
    e0 + i, and the shared expert (if any) is local index E_loc. The router
    weight is the full one."""

    def __init__(self, spec: MoeSpec, lw: LayerWeights, tokens: int, rank: int, world: int,
                 group=None, ops=None, device=None, max_tokens: int | None = None):
        """``max_tokens``: the largest token count of any rank (the exchange
        blocks must have one size on every rank); when None it is agreed on
        with one all_reduce over the group, so every rank must construct its
        layers in the same order."""
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
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        # Exchange blocks: `cap` rows per rank pair (all of a rank's rows may
        # go to one owner), the same on every rank.
        if max_tokens is None:
            t = torch.tensor([T], dtype=torch.int64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            max_tokens = int(t.item())
        self.cap = max_tokens * k
        R = self.cap * world
        self.slot = torch.empty(T * k, dtype=torch.int32, device=dev)
        self.xsend = torch.empty((R, M), dtype=adt, device=dev)
        self.xrecv = torch.empty((R, M), dtype=adt, device=dev)
        self.hr = torch.empty((max(R, T), I), dtype=adt, device=dev)
        self.yr = torch.empty((R, M), dtype=torch.float32, device=dev)
        self.yback = torch.empty((R, M), dtype=torch.float32, device=dev)
        self.xsorted = torch.empty((R, M), dtype=adt, device=dev)
        self.ysorted = torch.empty((R, M), dtype=torch.float32, device=dev)
        self.src_pos = torch.empty(R, dtype=torch.int32, device=dev)
        self.total = torch.zeros(1, dtype=torch.int32, device=dev)
        self.cnt_recv = torch.empty(self.e_loc * world, dtype=torch.int32, device=dev)
        self.n_rsegs = self.e_loc
        self.rsegs = torch.empty(16 * self.n_rsegs, dtype=torch.uint8, device=dev)
        self.tiles = torch.empty(abi.lib().wisp_b200_tiles_words(self.n_rsegs + 1)
                                 if adt == torch.float16 else 1, dtype=torch.int32, device=dev)
        if spec.has_shared:
            self.xs = torch.empty((T, M), dtype=adt, device=dev)
            self.sh_token = torch.arange(T, dtype=torch.int32, device=dev)
            self.sh_weight = torch.ones(T, dtype=torch.float32, device=dev)
            self.sh_seg = torch.empty(16, dtype=torch.uint8, device=dev)
            seg = abi.WispSegment()
            seg.expert, seg.row_begin, seg.rows = self.e_loc, 0, T
            self.sh_seg.copy_(torch.frombuffer(bytearray(bytes(seg)), dtype=torch.uint8))

    def forward(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """x: bf16 [T, M] (this rank's tokens) -> out fp32 [T, M]."""
        spec, ops, T, k, world = self.spec, self.ops, self.T, self.spec.top_k, self.world
        ops.route(self.cfg_route, self.lw, x, self.idx, self.w, self.logits)
        ops.plan(self.cfg_route, self.idx, self.w, self.counts, self.segs, self.row_token,
                 self.row_weight)
        ops.send_pack(x, self.row_token, self.segs, spec.n_experts, T * k, world, self.cap,
                      self.xsend, self.slot)
        # 1. per-expert row counts to the owners, then the row blocks; the
        #    shared expert runs on this rank's own tokens while they travel
        w_cnt = dist.all_to_all_single(self.cnt_recv, self.counts, group=self.group,
                                       async_op=True)
        w_rows = dist.all_to_all_single(self.xrecv, self.xsend, group=self.group, async_op=True)
        out.zero_()
        if spec.has_shared:
            ops.pack(x, None, T, self.xs)
            ops.grouped_dev(self.cfg_loc, self.lw, self.sh_seg, 1, T, self.xs, self.hr, 0,
                            self.sh_token, self.sh_weight, out, self.tiles, self.flag)
        w_cnt.wait()
        w_rows.wait()
        # 2. local experts over the received rows, gathered so that each
        #    expert is one segment (unweighted fp32 rows), then scattered
        #    back into the source blocks
        R = self.cap * world
        ops.recv_plan(self.cnt_recv, world, self.e_loc, self.cap, self.rsegs, self.src_pos,
                      self.total)
        ops.gather_rows(self.xrecv, self.src_pos, self.total, R, self.xsorted)
        ops.grouped_dev(self.cfg_loc, self.lw, self.rsegs, self.n_rsegs, R, self.xsorted,
                        self.hr, 1, None, None, self.ysorted, self.tiles, self.flag)
        ops.scatter_rows(self.ysorted, self.src_pos, self.total, R, self.yr)
        # 3. rows back to their tokens' ranks, then the weighted combine
        dist.all_to_all_single(self.yback, self.yr, group=self.group)
        ops.ep_combine(self.yback, self.slot, self.row_token, self.row_weight, T * k, out)
        return out
