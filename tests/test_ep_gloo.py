"""Expert-parallel exchange logic on CPU ranks (gloo, world size 2).

EpLayer's dispatch/combine plumbing (count exchange, send/receive splits,
expert-major receive layout, all-to-all ordering, weighted combine) runs for
real over torch.distributed; the compute steps are a host implementation
built on the fp64 oracle. The result must equal the single-process oracle
output for every token. Also: a rank that dies before the collective makes
the others fail within the process-group timeout instead of hanging.
"""
from __future__ import annotations

import os
import socket
import tempfile
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wisp_b200 import synth
from wisp_b200.ep import BlockLayout, EpLayer, block_range, dispatch_reference

SPEC = synth.MoeSpec("ep_cpu", 256, 128, 8, 2, group_size=64, has_shared=True, tokens=10, seed=21)


class CpuOps:
    """Host stand-in for CudaOps: same contract, fp64 oracle arithmetic."""

    def __init__(self, orc, lw):
        self.orc, self.lw = orc, lw

    def act_dtype(self):
        return torch.float64

    def route_scratch(self, cfg, device):
        return torch.empty(1)

    def route(self, cfg, lw, x, idx, w, scratch):
        from helpers import oracle_route
        i, ww, _ = oracle_route(self.orc, lw, x)
        idx.copy_(torch.from_numpy(i))
        w.copy_(torch.from_numpy(ww).float())

    def plan(self, cfg, idx, w, counts, segs, row_token, row_weight):
        ii, ww = idx.numpy(), w.numpy()
        T, k = ii.shape
        sv = segs.numpy().view(np.int32).reshape(-1, 4)
        p = 0
        for e in range(cfg.n_experts):
            sv[e] = (e, p, 0, 0)
            n = 0
            for t in range(T):
                for j in range(k):
                    if ii[t, j] == e:
                        row_token[p] = t
                        row_weight[p] = float(ww[t, j])
                        p += 1
                        n += 1
            counts[e] = n
            sv[e, 2] = n

    def block_layout(self, hidden, e_loc, cap, k):
        self.lay = BlockLayout(hidden, e_loc, cap, k, 8)   # float64 rows
        return self.lay

    def _views(self, buf, q, lay):
        b = buf.numpy()[q * lay.bytes:(q + 1) * lay.bytes]
        hdr = b[:lay.off_ent].view(np.int32)
        ent = b[lay.off_ent:lay.off_w].view(np.int32)
        ew = b[lay.off_w:lay.off_w + 4 * lay.cap * lay.k].view(np.float32)
        rows = b[lay.off_rows:lay.off_rows + lay.cap * lay.hidden * 8].view(np.float64)
        return hdr, ent, ew, rows.reshape(lay.cap, lay.hidden)

    def dispatch(self, x, idx, plan_segs, row_token, row_weight, n_experts, world, cap, send, slot,
                 own_rows=None):
        lay = self.lay
        if own_rows is not None:
            own_rows[:x.shape[0]] = x.double()
        T = x.shape[0]
        slot_ref, entries = dispatch_reference(idx.numpy(), n_experts, world)
        slot.copy_(torch.from_numpy(slot_ref).int())
        e_loc = n_experts // world
        sv = plan_segs.numpy().view(np.int32).reshape(-1, 4)
        wv = row_weight.numpy()
        xd = x.double().numpy()
        for q in range(world):
            hdr, ent, ew, rows = self._views(send, q, lay)
            hdr[0] = int((slot_ref[:, q] >= 0).sum())
            hdr[4:4 + e_loc] = sv[q * e_loc:(q + 1) * e_loc, 2]
            first = int(sv[q * e_loc, 1])
            # the plan rows of q's experts, in plan order, are the entries
            for i, (r, t, j) in enumerate(entries[q]):
                p = first + i
                assert int(row_token[p]) == t
                ent[i] = r
                ew[i] = wv[p]
            for t in range(T):
                if slot_ref[t, q] >= 0:
                    rows[slot_ref[t, q]] = xd[t]

    def recv_plan(self, recv, world, e_loc, cap, k, hidden, own, segs, src_pos, weight, total):
        lay = self.lay
        sv = segs.numpy().view(np.int32).reshape(-1, 4)
        views = [self._views(recv, s, lay) for s in range(world)]
        off = [np.concatenate([[0], np.cumsum(v[0][4:4 + e_loc])[:-1]]) for v in views]
        j = 0
        for e in range(e_loc):
            b = j
            for s in range(world):
                hdr, ent, ew, _ = views[s]
                for i in range(int(hdr[4 + e])):
                    src_pos[j] = s * cap + int(ent[off[s][e] + i])
                    weight[j] = float(ew[off[s][e] + i])
                    j += 1
            sv[e] = (e, b, j - b, 0)
        total[0] = j
        if own:   # the rank's own rows, the shared expert's segment
            sv[e_loc] = (e_loc, j, own, 0)
            for t in range(own):
                src_pos[j + t] = world * cap + t
                weight[j + t] = 1.0

    def gather_rows(self, recv, world, e_loc, cap, k, hidden, src_pos, total, own_rows, own,
                    max_rows, sorted_rows):
        lay = self.lay
        for j in range(int(total[0]) + own):
            r = int(src_pos[j])
            if r >= world * cap:
                sorted_rows[j] = own_rows[r - world * cap]
            else:
                sorted_rows[j] = torch.from_numpy(self._views(recv, r // cap, lay)[3][r % cap].copy())

    def workspace(self, cfg, n_segs, rows, device):
        return torch.empty(1, dtype=torch.uint8)

    def clear_flag(self, flag):
        flag.zero_()

    def check_flag(self, flag):
        assert int(flag[0]) == 0

    def grouped_dev(self, cfg, lw, segs, n_segs, rows, xp, h, mode, row_token, row_weight, out,
                    tiles, flag):
        sv = segs.numpy().view(np.int32).reshape(-1, 4)[:n_segs]
        self.grouped(cfg, lw, [(int(e), int(b), int(r)) for e, b, r, _ in sv], rows, xp, h, mode,
                     row_token, row_weight, out, tiles, flag)

    def ret_dtype(self):
        return torch.float64

    def return_rows(self, yr, yr16):
        yr16.copy_(yr)

    def ep_combine(self, yback, slot, local, tokens, world, cap, out):
        sl = slot.numpy()
        if local is not None:
            out[:tokens] = local[:tokens]
        for t in range(tokens):
            for q in range(world):
                if sl[t, q] >= 0:
                    out[t] += yback[q * cap + int(sl[t, q])]

    def pack(self, x, src, n_rows, xp):
        xd = x.double()
        xp[:n_rows] = xd if src is None else xd[src[:n_rows].long()]

    def grouped(self, cfg, lw, segs, rows, xp, h, mode, row_token, row_weight, out, tiles, flag):
        for e, b, r in segs:
            mats = self.lw.expert_host(e)
            for p in range(b, b + r):
                y = self.orc.expert_ffn(mats, self.lw.spec.group_size, xp[p].numpy(), 1.0)
                if mode == 1:
                    out[p] = torch.from_numpy(y).float()
                else:
                    t = int(row_token[p])
                    out[t] += float(row_weight[p]) * torch.from_numpy(y).float()

    def combine(self, y, row_token, row_weight, n_rows, out):
        for p in range(n_rows):
            out[int(row_token[p])] += float(row_weight[p]) * y[p]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, outdir, spec, mode):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
    try:
        from oracle.oracle import Oracle
        orc = Oracle()
        keep = range(*block_range(spec.n_experts, world, rank))
        layers, x = synth.make_model(spec, "cpu", keep=keep)
        lw = layers[0]
        t0, t1 = block_range(spec.tokens, world, rank)
        t_max = max(b - a for a, b in (block_range(spec.tokens, world, q) for q in range(world)))
        layer = EpLayer(spec, lw, t1 - t0, rank, world, ops=CpuOps(orc, lw), device=torch.device("cpu"),
                        max_tokens=t_max)
        if mode == "die" and rank == 1:
            raise SystemExit(3)          # leaves before the first collective
        out = torch.zeros((t1 - t0, spec.hidden), dtype=torch.float32)
        try:
            layer.forward(x[t0:t1].contiguous(), out)
            np.save(os.path.join(outdir, f"out{rank}.npy"), out.numpy())
        except Exception as exc:  # noqa: BLE001 - reported to the parent
            with open(os.path.join(outdir, f"err{rank}.txt"), "w") as f:
                f.write(type(exc).__name__ + ": " + str(exc))
    finally:
        if mode != "die":
            dist.destroy_process_group()


def test_dispatch_layout():
    """A token is sent once per owner rank; entries are expert-major, then
    token order; the Python block layout matches the library's."""
    idx = np.array([[0, 5], [1, 2], [7, 4], [3, 3]])   # 4 tokens, k=2, 8 experts
    slot, entries = dispatch_reference(idx, 8, 2)       # ranks own experts 0-3 / 4-7
    assert slot.tolist() == [[0, 0], [1, -1], [-1, 1], [2, -1]]
    assert entries[0] == [(0, 0, 0), (1, 1, 0), (1, 1, 1), (2, 3, 0), (2, 3, 1)]
    assert entries[1] == [(1, 2, 1), (0, 0, 1), (1, 2, 0)]
    from wisp_b200 import abi
    for hidden, e_loc, cap, k in [(7168, 48, 32, 8), (256, 4, 5, 2), (4096, 1, 1, 1)]:
        assert BlockLayout(hidden, e_loc, cap, k).bytes == \
            abi.lib().wisp_b200_ep_block_bytes(hidden, e_loc, cap, k)


@pytest.mark.parametrize("world,spec", [(2, SPEC), (2, synth.small(SPEC, skew=True, seed=4, tokens=7)),
                                        (4, synth.small(SPEC, seed=9, tokens=11)),
                                        (8, synth.small(SPEC, seed=12, tokens=13))])
def test_ep_ranks_match_single_process(orc, world, spec):
    from helpers import oracle_outputs, oracle_route
    port = _free_port()
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(world, port, td, spec, "ok"), nprocs=world, join=True,
                           start_method="spawn")
        for r in range(world):
            assert not os.path.exists(os.path.join(td, f"err{r}.txt")), open(os.path.join(td, f"err{r}.txt")).read()
        got = np.concatenate([np.load(os.path.join(td, f"out{r}.npy")) for r in range(world)])
    layers, x = synth.make_model(spec, "cpu")
    lw = layers[0]
    idx, w, _ = oracle_route(orc, lw, x)
    ref = oracle_outputs(orc, lw, x, idx, w, list(range(spec.tokens)))
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())


def test_ep_rank_failure_is_detected_not_hung():
    port = _free_port()
    with tempfile.TemporaryDirectory() as td:
        ctx = mp.start_processes(_worker, args=(2, port, td, SPEC, "die"), nprocs=2, join=False,
                                 start_method="spawn")
        import time
        deadline = time.time() + 60
        while time.time() < deadline:
            try:
                if ctx.join(timeout=1):
                    break
            except Exception:  # noqa: BLE001 - rank 1 exits with an error on purpose
                pass
            if all(not p.is_alive() for p in ctx.processes):
                break
        alive = [p.is_alive() for p in ctx.processes]
        for p in ctx.processes:
            if p.is_alive():
                p.kill()
        assert not any(alive), "a surviving rank hung on the collective"
        assert os.path.exists(os.path.join(td, "err0.txt")), "rank 0 did not report the failure"
