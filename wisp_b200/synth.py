"""Seeded synthetic MoE layers with the shapes and value distributions of the
benchmark configurations (no checkpoints or datasets are involved).

Distributions: int4 values uniform in [-8, 7] (nibbles uniform in 0..15,
packed two per byte along K, low nibble first), fp16 scales uniform in
[0.004, 0.02] per group of ``group_size`` along K, symmetric (zero = 0)
unless ``zeros=True``; router weight bf16 ~ N(0, 0.02); activations bf16 ~
N(0, 1). The skewed prefill configuration adds an N(0, 1) offset per expert
to the router logits (passed as the router bias, added before scoring).

Draw order from one torch.Generator per configuration (seeded with the
configuration's seed): for each layer: router weight, the logit offsets
(skewed configs only), then per expert (routed experts in order, then the
shared expert) gate packed, gate scales, up packed, up scales, down packed,
down scales [, zeros when requested]; finally the activations.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, replace

import torch

from . import abi


@dataclass(frozen=True)
class MoeSpec:
    name: str
    hidden: int
    inter: int
    n_experts: int
    top_k: int
    group_size: int = 128
    scoring: int = abi.WISP_SCORE_SOFTMAX
    n_groups: int = 1
    topk_groups: int = 1
    routed_scaling: float = 1.0
    has_shared: bool = False
    tokens: int = 1
    layers: int = 1
    seed: int = 0
    skew: bool = False

    @property
    def n_virtual(self) -> int:
        return self.n_experts + (1 if self.has_shared else 0)

    def cfg(self, tokens: int | None = None) -> abi.WispMoeConfig:
        c = abi.WispMoeConfig()
        c.tokens = self.tokens if tokens is None else tokens
        c.hidden, c.inter, c.n_experts, c.top_k = self.hidden, self.inter, self.n_experts, self.top_k
        c.group_size, c.scoring = self.group_size, self.scoring
        c.n_groups, c.topk_groups = self.n_groups, self.topk_groups
        c.routed_scaling = self.routed_scaling
        c.has_shared = 1 if self.has_shared else 0
        c.router_fp16 = 0
        return c

    def expert_bytes(self) -> int:
        """Algorithmic bytes of one expert: int4 packed + fp16 scales."""
        n = 3 * self.hidden * self.inter
        return n // 2 + 2 * (n // self.group_size)


_DS = dict(hidden=7168, inter=2048, n_experts=256, top_k=8,
           scoring=abi.WISP_SCORE_SIGMOID_GROUPED, n_groups=8, topk_groups=4,
           routed_scaling=2.5, has_shared=True)

# The benchmark configurations (BASELINE.json "configs", in order).
CONFIGS: dict[str, MoeSpec] = {
    "mixtral_b1": MoeSpec("mixtral_b1", 4096, 14336, 8, 2, tokens=1, seed=0),
    "mixtral_b64": MoeSpec("mixtral_b64", 4096, 14336, 8, 2, tokens=64, seed=0),
    "ds_b1": MoeSpec("ds_b1", tokens=1, seed=1, **_DS),
    "ds_b128": MoeSpec("ds_b128", tokens=128, seed=1, **_DS),
    "ds_prefill": MoeSpec("ds_prefill", tokens=4096, seed=2, skew=True, **_DS),
    "ep_stack": MoeSpec("ep_stack", 7168, 2048, 384, 8, has_shared=True, tokens=256, layers=4,
                        seed=3),
    # One layer of the ep_stack shape with 64 experts (~1.5 GB of weights,
    # still larger than L2): the small case for ncu captures.
    "ep_profile": MoeSpec("ep_profile", 7168, 2048, 64, 8, has_shared=True, tokens=40, layers=1,
                          seed=3),
    # The DeepSeek b1 decode layer with 16 routed experts (+ shared): the
    # same 9 touched experts and register-path launches as ds_b1 with
    # 386 MB of weights on the device, the small case for ncu captures.
    "ds_b1_profile": MoeSpec("ds_b1_profile", tokens=1, seed=1, **dict(_DS, n_experts=16)),
    # A prefill-shaped layer small enough for ncu: 64 DeepSeek-shaped experts
    # (1.45 GB), 1024 skewed tokens -> segments of ~100-600 rows.
    "prefill_profile": MoeSpec("prefill_profile", tokens=1024, seed=2, skew=True,
                               **dict(_DS, n_experts=64)),
}


@dataclass
class Int4Arena:
    """All experts' copies of one matrix kind: V x rows x cols."""
    packed: torch.Tensor          # uint8 [V, rows, cols // 2]
    scales: torch.Tensor          # fp16  [V, rows, cols // gs]
    zeros: torch.Tensor | None    # fp16  [V, rows, cols // gs] or None

    def mat_ptrs(self, v: int) -> abi.WispInt4Mat:
        m = abi.WispInt4Mat()
        m.packed = self.packed[v].data_ptr()
        m.scales = self.scales[v].data_ptr()
        m.zeros = self.zeros[v].data_ptr() if self.zeros is not None else None
        return m


@dataclass
class LayerWeights:
    spec: MoeSpec
    router_w: torch.Tensor              # bf16 [E, M]
    router_bias: torch.Tensor | None    # fp32 [E]
    gate: Int4Arena
    up: Int4Arena
    down: Int4Arena
    table: torch.Tensor = field(default=None)     # uint8 device copy of WispInt4Expert[V]
    prepared: torch.Tensor = field(default=None)  # from wisp_b200_prepare_experts

    def build_table(self) -> None:
        V = self.gate.packed.shape[0]
        arr = (abi.WispInt4Expert * V)()
        for v in range(V):
            arr[v].gate = self.gate.mat_ptrs(v)
            arr[v].up = self.up.mat_ptrs(v)
            arr[v].down = self.down.mat_ptrs(v)
        raw = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
        self.table = raw.to(self.gate.packed.device)

    @property
    def n_entries(self) -> int:
        return self.gate.packed.shape[0]

    def prepare(self) -> torch.Tensor:
        """Run wisp_b200_prepare_experts once (device weights only)."""
        if self.prepared is None:
            cfg = self.spec.cfg()
            n = self.n_entries
            nbytes = abi.lib().wisp_b200_prepared_bytes(C.byref(cfg), n)
            if nbytes == 0:
                raise RuntimeError("wisp engine error [4]: shapes not supported by the tensor-core path")
            self.prepared = torch.empty(nbytes, dtype=torch.uint8, device=self.table.device)
            abi.call("wisp_b200_prepare_experts", C.byref(cfg), self.table.data_ptr(), n,
                     self.prepared.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream)
        return self.prepared

    def weights_struct(self) -> abi.WispMoeWeights:
        w = abi.WispMoeWeights()
        w.router_w = self.router_w.data_ptr()
        w.router_bias = self.router_bias.data_ptr() if self.router_bias is not None else None
        w.experts = self.table.data_ptr()
        w.prepared = self.prepared.data_ptr() if self.prepared is not None else None
        return w

    def expert_host(self, v: int):
        """(gate, up, down) of virtual expert v as numpy-backed blob matrices."""
        from .blob import Int4Matrix
        out = []
        for a in (self.gate, self.up, self.down):
            p = a.packed[v].cpu()
            rows, half = p.shape
            out.append(Int4Matrix(
                packed=p.reshape(-1).numpy(),
                scales=a.scales[v].cpu().reshape(-1).view(torch.int16).numpy().view("uint16"),
                zeros=None if a.zeros is None else
                a.zeros[v].cpu().reshape(-1).view(torch.int16).numpy().view("uint16"),
                rows=rows, cols=2 * half))
        return out


def _arena(g: torch.Generator, V: int, rows: int, cols: int, gs: int, device, zeros: bool):
    packed = torch.empty((V, rows, cols // 2), dtype=torch.uint8, device=device)
    scales = torch.empty((V, rows, cols // gs), dtype=torch.float16, device=device)
    zs = torch.empty_like(scales) if zeros else None
    return Int4Arena(packed, scales, zs)


def make_layer(spec: MoeSpec, g: torch.Generator, device, zeros: bool = False,
               keep: range | None = None) -> LayerWeights:
    """One layer. ``keep``: the routed experts this process holds (an
    expert-parallel shard); the others are still drawn, into a scratch
    buffer, so every shard sees the same random stream as the full model.
    The shared expert is always kept (local index len(keep))."""
    M, I, E, gs = spec.hidden, spec.inter, spec.n_experts, spec.group_size
    keep = range(E) if keep is None else keep
    local = {e: i for i, e in enumerate(keep)}
    if spec.has_shared:
        local[E] = len(keep)
    V = len(local)
    router_w = (torch.randn((E, M), generator=g, device=device) * 0.02).to(torch.bfloat16)
    bias = torch.randn((E,), generator=g, device=device) if spec.skew else None
    gate = _arena(g, V, I, M, gs, device, zeros)
    up = _arena(g, V, I, M, gs, device, zeros)
    down = _arena(g, V, M, I, gs, device, zeros)
    scratch = None
    for v in range(spec.n_virtual):
        for a in (gate, up, down):
            shape_p, shape_s = a.packed.shape[1:], a.scales.shape[1:]
            if v in local:
                i = local[v]
                dst_p, dst_s = a.packed[i], a.scales[i]
                dst_z = a.zeros[i] if a.zeros is not None else None
            else:
                if scratch is None:
                    scratch = {}
                key = tuple(shape_p)
                if key not in scratch:
                    scratch[key] = (torch.empty(shape_p, dtype=torch.uint8, device=device),
                                    torch.empty(shape_s, dtype=torch.float16, device=device),
                                    torch.empty(shape_s, dtype=torch.float16, device=device))
                dst_p, dst_s, dst_z = scratch[key]
                if a.zeros is None:
                    dst_z = None
            dst_p.copy_(torch.randint(0, 256, shape_p, generator=g, device=device, dtype=torch.uint8))
            dst_s.copy_(torch.empty(shape_s, device=device).uniform_(0.004, 0.02, generator=g)
                        .to(torch.float16))
            if dst_z is not None:
                dst_z.copy_(torch.empty(shape_s, device=device).uniform_(-0.01, 0.01, generator=g)
                            .to(torch.float16))
    lw = LayerWeights(spec, router_w.contiguous(), bias, gate, up, down)
    lw.build_table()
    return lw


def make_model(spec: MoeSpec, device="cuda", zeros: bool = False, tokens: int | None = None,
               keep: range | None = None):
    """All layers of a configuration plus its activations x (bf16 [T, M])."""
    g = torch.Generator(device=device)
    g.manual_seed(spec.seed)
    layers = [make_layer(spec, g, device, zeros, keep) for _ in range(spec.layers)]
    T = spec.tokens if tokens is None else tokens
    x = torch.randn((T, spec.hidden), generator=g, device=device).to(torch.bfloat16)
    return layers, x


def small(spec: MoeSpec, **kw) -> MoeSpec:
    """A reduced copy of a configuration (for tests)."""
    return replace(spec, **kw)
