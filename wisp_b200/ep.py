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
  route own tokens -> plan (rows grouped by expert) -> one fixed-size block
  per destination rank: a token's row once per destination that owns any of
  its experts, plus the (row, weight) entries of its experts there
  (wisp_b200_ep_dispatch, which also packs the rank's own rows) -> all_to_all
  of the blocks -> gather the received rows expert-contiguous (one
  segment per local expert, as on one GPU), the own rows after them as the
  shared expert's segment -> one grouped FFN in mode 0 with the routing
  weights, into one fp32 row per received token (and one per own token for
  the shared expert) -> the return rows rounded to fp16 and sent back with
  one all_to_all -> out[t] = the shared expert's row + the rows from the
  owners, in rank order.
cap = the most tokens any rank holds (a token fills at most one row of a
block); padding rows are exchanged but never computed or read.

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


class BlockLayout:
    """Byte layout of one exchange block (mirrors ep.cu; elem = bytes per
    row element: 2 for the fp16 rows of the CUDA path)."""

    def __init__(self, hidden: int, e_loc: int, cap: int, top_k: int, elem: int = 2):
        a16 = lambda v: (v + 15) & ~15  # noqa: E731
        self.cap, self.k, self.e_loc, self.hidden, self.elem = cap, top_k, e_loc, hidden, elem
        self.off_cnt = 16
        self.off_ent = a16(16 + 4 * e_loc)
        self.off_w = self.off_ent + 4 * cap * top_k
        self.off_rows = a16(self.off_w + 4 * cap * top_k)
        self.bytes = a16(self.off_rows + cap * hidden * elem)


def dispatch_reference(idx: np.ndarray, n_experts: int, world: int):
    """Host statement of the dispatch layout: slot[t, q] (row of token t in
    the block for rank q, tokens in order, -1 if none of t's experts is on
    q) and, per destination, the entries (row, k-index) expert-major then
    token-ascending."""
    T, k = idx.shape
    e_loc = n_experts // world
    slot = -np.ones((T, world), np.int64)
    for q in range(world):
        n = 0
        for t in range(T):
            if any(int(e) // e_loc == q for e in idx[t]):
                slot[t, q] = n
                n += 1
    entries = []
    for q in range(world):
        ent = []
        for e in range(q * e_loc, (q + 1) * e_loc):
            for t in range(T):
                for j in range(k):
                    if int(idx[t, j]) == e:
                        ent.append((int(slot[t, q]), t, j))
        entries.append(ent)
    return slot, entries


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _segments_tensor(segs, device) -> torch.Tensor:
    arr = (abi.WispSegment * max(1, len(segs)))()
    for i, (e, b, r) in enumerate(segs):
        arr[i].expert, arr[i].row_begin, arr[i].rows = e, b, r
    return torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(device, non_blocking=True)


class CudaOps:
    """Compute steps of one EP layer on the GPU, through libwisp_b200.so."""

    def route_scratch(self, cfg, device):
        """Split-K partial sums of the router logits (wisp_b200_route_ws)."""
        n = abi.lib().wisp_b200_route_workspace_bytes(C.byref(cfg))
        if n == 0:
            raise RuntimeError(f"wisp engine error [{abi.WISP_ERR_INVALID_ARG}]: route workspace query failed")
        return torch.empty(n, dtype=torch.uint8, device=device)

    def route(self, cfg, lw: LayerWeights, x, idx, w, scratch):
        ws = lw.weights_struct()
        abi.call("wisp_b200_route_ws", C.byref(cfg), C.byref(ws), x.data_ptr(), None,
                 idx.data_ptr(), w.data_ptr(), scratch.data_ptr(), scratch.numel(), _stream())

    def plan(self, cfg, idx, w, counts, segs, row_token, row_weight):
        abi.call("wisp_b200_dispatch_plan", C.byref(cfg), idx.data_ptr(), w.data_ptr(),
                 counts.data_ptr(), segs.data_ptr(), row_token.data_ptr(), row_weight.data_ptr(),
                 _stream())

    def pack(self, x, src, n_rows, xp):
        abi.call("wisp_b200_pack_rows", x.data_ptr(), None if src is None else src.data_ptr(),
                 n_rows, x.shape[1], xp.data_ptr(), _stream())

    def grouped(self, cfg, lw, segs, rows, xp, h, mode, row_token, row_weight, out, ws, flag):
        dsegs = _segments_tensor(segs, xp.device)
        abi.call("wisp_b200_grouped_ffn", C.byref(cfg), lw.prepare().data_ptr(), lw.table.data_ptr(),
                 lw.n_entries,
                 dsegs.data_ptr(), len(segs),
                 max(rows, 1), xp.data_ptr(), h.data_ptr(), mode,
                 None if row_token is None else row_token.data_ptr(),
                 None if row_weight is None else row_weight.data_ptr(), out.data_ptr(),
                 ws.data_ptr(), ws.numel(), flag.data_ptr(), _stream())

    def combine(self, y, row_token, row_weight, n_rows, out):
        abi.call("wisp_b200_combine_rows", y.data_ptr(), row_token.data_ptr(), row_weight.data_ptr(),
                 n_rows, out.shape[1], out.data_ptr(), _stream())

    def dispatch(self, x, idx, plan_segs, row_token, row_weight, n_experts, world, cap, send, slot,
                 own_rows=None):
        abi.call("wisp_b200_ep_dispatch", x.data_ptr(), x.shape[0], x.shape[1], idx.data_ptr(),
                 idx.shape[1], plan_segs.data_ptr(), row_token.data_ptr(), row_weight.data_ptr(),
                 n_experts, world, cap, send.data_ptr(), slot.data_ptr(),
                 None if own_rows is None else own_rows.data_ptr(), _stream())

    def recv_plan(self, recv, world, e_loc, cap, k, hidden, own, segs, src_pos, weight, total):
        abi.call("wisp_b200_ep_recv_plan", recv.data_ptr(), world, e_loc, cap, k, hidden, own,
                 segs.data_ptr(), src_pos.data_ptr(), weight.data_ptr(), total.data_ptr(), _stream())

    def gather_rows(self, recv, world, e_loc, cap, k, hidden, src_pos, total, own_rows, own,
                    max_rows, sorted_rows):
        abi.call("wisp_b200_ep_gather_rows", recv.data_ptr(), world, e_loc, cap, k, hidden,
                 src_pos.data_ptr(), total.data_ptr(),
                 None if own_rows is None else own_rows.data_ptr(), own, max_rows,
                 sorted_rows.data_ptr(), _stream())

    def grouped_dev(self, cfg, lw, segs, n_segs, rows, xp, h, mode, row_token, row_weight, out,
                    ws, flag):
        abi.call("wisp_b200_grouped_ffn", C.byref(cfg), lw.prepare().data_ptr(), lw.table.data_ptr(),
                 lw.n_entries, segs.data_ptr(), n_segs, max(rows, 1), xp.data_ptr(), h.data_ptr(),
                 mode, None if row_token is None else row_token.data_ptr(),
                 None if row_weight is None else row_weight.data_ptr(), out.data_ptr(),
                 ws.data_ptr(), ws.numel(), flag.data_ptr(), _stream())

    def workspace(self, cfg, n_segs, rows, device):
        n = abi.lib().wisp_b200_grouped_workspace_bytes(C.byref(cfg), n_segs, max(rows, 1))
        if n == 0:
            raise RuntimeError(f"wisp engine error [{abi.WISP_ERR_INVALID_ARG}]: grouped workspace query failed")
        return torch.empty(n, dtype=torch.uint8, device=device)

    def clear_flag(self, flag):
        flag.zero_()

    def check_flag(self, flag):
        abi.call("wisp_b200_check_error_flag", flag.data_ptr(), _stream())

    def ep_combine(self, yback, slot, local, tokens, world, cap, out):
        abi.call("wisp_b200_ep_combine_f16", yback.data_ptr(), slot.data_ptr(),
                 None if local is None else local.data_ptr(), tokens, world, cap, out.shape[1],
                 out.data_ptr(), _stream())

    def return_rows(self, yr, yr16):
        abi.call("wisp_b200_ep_return_rows", yr.data_ptr(), yr.shape[0], yr.shape[1],
                 yr16.data_ptr(), _stream())

    def ret_dtype(self):
        return torch.float16

    def block_layout(self, hidden, e_loc, cap, k):
        lay = BlockLayout(hidden, e_loc, cap, k, 2)
        assert lay.bytes == abi.lib().wisp_b200_ep_block_bytes(hidden, e_loc, cap, k)
        return lay

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
        self.route_scratch = self.ops.route_scratch(self.cfg_route, dev)
        self.counts = torch.empty(spec.n_experts, dtype=torch.int32, device=dev)
        self.segs = torch.empty(16 * spec.n_experts, dtype=torch.uint8, device=dev)
        self.row_token = torch.empty(T * k, dtype=torch.int32, device=dev)
        self.row_weight = torch.empty(T * k, dtype=torch.float32, device=dev)
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        # Exchange blocks: one per rank pair, `cap` token rows each (a token
        # fills at most one row of a block), the same on every rank.
        if max_tokens is None:
            t = torch.tensor([T], dtype=torch.int64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            max_tokens = int(t.item())
        self.cap = max(1, max_tokens)
        self.layout = self.ops.block_layout(M, self.e_loc, self.cap, k)
        nb = self.layout.bytes
        RK = world * self.cap * k          # most (token, local expert) rows received
        # The shared expert runs in the same grouped call as the local experts:
        # this rank's own T token rows follow the received rows as one more
        # segment, and its output rows follow the return rows in yr.
        self.own = T if spec.has_shared else 0
        self.rk = RK + self.own
        self.slot = torch.empty((T, world), dtype=torch.int32, device=dev)
        self.send = torch.zeros(world * nb, dtype=torch.uint8, device=dev)
        self.recv = torch.zeros(world * nb, dtype=torch.uint8, device=dev)
        self.xsorted = torch.empty((self.rk, M), dtype=adt, device=dev)
        self.hr = torch.empty((self.rk, I), dtype=adt, device=dev)
        # return rows (then the shared expert's own rows): fp32 where the FFN
        # accumulates them, the return rows then in the exchange dtype (fp16
        # on GPUs) for the trip back
        nret = world * self.cap
        self.yr = torch.empty((nret + self.own, M), dtype=torch.float32, device=dev)
        self.yr_ret = self.yr[:nret]
        self.yr_own = self.yr[nret:] if self.own else None
        self.yr16 = torch.empty((nret, M), dtype=self.ops.ret_dtype(), device=dev)
        self.yback = torch.empty((nret, M), dtype=self.ops.ret_dtype(), device=dev)
        self.src_pos = torch.empty(self.rk, dtype=torch.int32, device=dev)
        self.gw = torch.empty(self.rk, dtype=torch.float32, device=dev)
        self.total = torch.zeros(1, dtype=torch.int32, device=dev)
        self.n_rsegs = self.e_loc + (1 if self.own else 0)
        self.rsegs = torch.empty(16 * self.n_rsegs, dtype=torch.uint8, device=dev)
        self.gws = self.ops.workspace(self.cfg_loc, max(self.n_rsegs, 1), self.rk, dev)
        self.xs = torch.empty((T, M), dtype=adt, device=dev) if self.own else None

    # One layer is four local phases around two all-to-alls; forward() runs
    # them over the process group, and a single-process caller can run the
    # phases of several ranks itself with the exchanges done as copies
    # (loopback_forward).

    def dispatch_phase(self, x: torch.Tensor, out: torch.Tensor) -> None:
        """Route this rank's tokens and fill the send blocks (and, with a
        shared expert, this rank's own rows in the FFN's input form); clear
        the device error word."""
        spec, ops = self.spec, self.ops
        ops.clear_flag(self.flag)
        ops.route(self.cfg_route, self.lw, x, self.idx, self.w, self.route_scratch)
        ops.plan(self.cfg_route, self.idx, self.w, self.counts, self.segs, self.row_token,
                 self.row_weight)
        ops.dispatch(x, self.idx, self.segs, self.row_token, self.row_weight, spec.n_experts,
                     self.world, self.cap, self.send, self.slot, self.xs)

    def expert_phase(self, mark=None) -> None:
        """Local experts over the received rows, gathered so that each expert
        is one segment, and the shared expert over this rank's own rows as one
        more segment, in one grouped call: the FFN adds w * y of every local
        expert of a received token into that token's fp32 return row, and the
        shared expert's output of own token t into row world * cap + t.
        ``mark(name)``, if given, is called after the receive plan and
        gather."""
        ops, k, M = self.ops, self.spec.top_k, self.spec.hidden
        ops.recv_plan(self.recv, self.world, self.e_loc, self.cap, k, M, self.own, self.rsegs,
                      self.src_pos, self.gw, self.total)
        ops.gather_rows(self.recv, self.world, self.e_loc, self.cap, k, M, self.src_pos, self.total,
                        self.xs, self.own, self.rk, self.xsorted)
        if mark:
            mark("gather")
        self.yr.zero_()
        ops.grouped_dev(self.cfg_loc, self.lw, self.rsegs, self.n_rsegs, self.rk, self.xsorted,
                        self.hr, 0, self.src_pos, self.gw, self.yr, self.gws, self.flag)
        ops.return_rows(self.yr_ret, self.yr16)

    def combine_phase(self, out: torch.Tensor) -> None:
        """out = the shared expert's row (if any) + the returned rows from the
        owners, in rank order."""
        if self.own:
            self.ops.ep_combine(self.yback, self.slot, self.yr_own, self.T, self.world, self.cap,
                                out)
        else:
            out.zero_()
            self.ops.ep_combine(self.yback, self.slot, None, self.T, self.world, self.cap, out)

    def forward(self, x: torch.Tensor, out: torch.Tensor, mark=None) -> torch.Tensor:
        """x: bf16 [T, M] (this rank's tokens) -> out fp32 [T, M].

        ``mark(name)``, if given, is called on the host after each phase has
        been issued (for per-phase CUDA events on the current stream): after
        route + plan + dispatch ("dispatch"), the first exchange
        ("exchange"), the receive plan and
        gather ("gather"), the FFN of the local and shared experts ("ffn"), the
        return exchange ("return") and the combine ("combine")."""
        m = mark or (lambda name: None)
        self.dispatch_phase(x, out)
        m("dispatch")
        # 1. the blocks to the owners
        dist.all_to_all_single(self.recv, self.send, group=self.group)
        m("exchange")
        # 2. local experts over the received rows and the shared expert over
        #    the own rows, one grouped call
        self.expert_phase(mark)
        m("ffn")
        # 3. the rows back to their tokens' ranks, added in rank order
        dist.all_to_all_single(self.yback, self.yr16, group=self.group)
        m("return")
        self.combine_phase(out)
        m("combine")
        return out

    def check(self) -> None:
        """Raise (WISP_ERR_TIMEOUT) if a kernel of the last forward gave up a
        bounded wait; synchronises the current stream."""
        self.ops.check_flag(self.flag)


def loopback_forward(layers: list, xs: list, outs: list) -> None:
    """Runs one layer of every rank of an expert-parallel group inside one
    process: layers[r] / xs[r] / outs[r] belong to rank r. The two
    all-to-alls become copies with all_to_all_single's block semantics
    (block q of rank r's send buffer is block r of rank q's receive
    buffer), so every device kernel of the exchange runs exactly as it does
    across GPUs."""
    W = len(layers)
    for r in range(W):
        layers[r].dispatch_phase(xs[r], outs[r])
    nb = layers[0].layout.bytes
    for r in range(W):
        for q in range(W):
            layers[q].recv[r * nb:(r + 1) * nb].copy_(layers[r].send[q * nb:(q + 1) * nb])
    for r in range(W):
        layers[r].expert_phase()
    cap = layers[0].cap
    for r in range(W):
        for q in range(W):
            layers[q].yback[r * cap:(r + 1) * cap].copy_(layers[r].yr16[q * cap:(q + 1) * cap])
    for r in range(W):
        layers[r].combine_phase(outs[r])
