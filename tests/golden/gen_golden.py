"""Generate the golden fixtures in tests/golden/ from the REFERENCE itself.

Run in a container where the reference project is importable:

    python tests/golden/gen_golden.py --reference /path/to/reference

It imports the reference's own Python int4 quantizer and expert-file writer
(wisp/converter/quantizer.py, wisp/converter/partitioner.py) and calls the
reference engine's own compiled CPU hot path (oracle/_ref/libwisp_ref.so,
built by `make -C oracle` from the reference's csrc/core sources). Nothing
here is needed at test time: the outputs are committed as .npz files.

Fixtures:
  format_vectors.npz  the reference's int4 format known answers: the constant
                      group packs to 0x88 and dequantises exactly
                      (tests/test_adapters.py:262-267), the round-trip case
                      (:250-259), a 16x32 / 32x16 gs=16 expert blob and its
                      Python dequantisation (:281-345).
  moe_small.npz       a 4-expert (+1 shared) MoE layer quantised by the
                      reference quantizer (asymmetric, gs=64, M=256, I=128),
                      serialised by the reference writer, with per-token
                      outputs, top-k indices and weights computed by the
                      reference's CPU run_moe branch (router_topk +
                      cpu_expert_ffn) for 6 tokens.
"""
from __future__ import annotations

import argparse
import sys
import os
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("WISP_REFERENCE_DIR"),
                    help="the reference project's checkout (or $WISP_REFERENCE_DIR)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference <path> or set WISP_REFERENCE_DIR")
    sys.path.insert(0, a.reference)
    sys.path.insert(0, str(ROOT))
    from wisp.converter.quantizer import quantize_int4, dequantize_int4  # reference code
    from wisp.converter.partitioner import write_expert_file  # reference code
    from oracle.oracle import RefCPU

    # ---- format known answers -------------------------------------------
    w = torch.full((2, 64), 1.0)
    qc = quantize_int4(w, group_size=64)
    torch.manual_seed(0)
    wr = torch.randn(64, 128) * 0.02
    qr = quantize_int4(wr, group_size=64)
    torch.manual_seed(7)
    hidden, inter, gs = 32, 16, 16
    mats = {
        "gate_proj": quantize_int4(torch.randn(inter, hidden), gs),
        "up_proj": quantize_int4(torch.randn(inter, hidden), gs),
        "down_proj": quantize_int4(torch.randn(hidden, inter), gs),
    }
    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "L005_E00123.bin"
        write_expert_file(p, 5, 123, mats)
        blob = np.frombuffer(p.read_bytes(), np.uint8).copy()
    fv = dict(
        const_packed=qc.packed.numpy(), const_scales=qc.scales.view(torch.int16).numpy(),
        const_zeros=qc.zeros.view(torch.int16).numpy(),
        const_dequant=dequantize_int4(qc).float().numpy(),
        rt_weight=wr.numpy(), rt_packed=qr.packed.numpy(),
        rt_scales=qr.scales.view(torch.int16).numpy(), rt_zeros=qr.zeros.view(torch.int16).numpy(),
        rt_dequant=dequantize_int4(qr).float().numpy(),
        small_blob=blob,
    )
    for i, key in enumerate(("gate_proj", "up_proj", "down_proj")):
        fv[f"small_dequant_{i}"] = dequantize_int4(mats[key]).float().numpy().reshape(-1)
    np.savez_compressed(HERE / "format_vectors.npz", **fv)

    # ---- small MoE layer through the reference CPU path ------------------
    ref = RefCPU()
    g = torch.Generator().manual_seed(1234)
    M, I, E, k, gs, T = 256, 128, 4, 2, 64, 6
    blobs = []
    with tempfile.TemporaryDirectory() as td:
        for e in range(E + 1):  # the last one is the shared expert
            ms = {
                "gate_proj": quantize_int4(torch.randn(I, M, generator=g) * 0.05, gs),
                "up_proj": quantize_int4(torch.randn(I, M, generator=g) * 0.05, gs),
                "down_proj": quantize_int4(torch.randn(M, I, generator=g) * 0.05, gs),
            }
            p = Path(td) / f"L000_E{e:05d}.bin"
            write_expert_file(p, 0, e, ms)
            blobs.append(np.frombuffer(p.read_bytes(), np.uint8).copy())
    router_w16 = (torch.randn(E, M, generator=g) * 0.05).half()
    x = torch.randn(T, M, generator=g).to(torch.bfloat16).float()
    outs, idxs, ws, outs_noshared = [], [], [], []
    for t in range(T):
        o, i, wt = ref.moe_token(router_w16.view(torch.int16).numpy().view(np.uint16), None,
                                 x[t].numpy(), k, blobs[:E], blobs[E])
        o2, _, _ = ref.moe_token(router_w16.view(torch.int16).numpy().view(np.uint16), None,
                                 x[t].numpy(), k, blobs[:E], None)
        outs.append(o)
        outs_noshared.append(o2)
        idxs.append(i)
        ws.append(wt)
    np.savez_compressed(
        HERE / "moe_small.npz",
        blobs=np.stack(blobs), router_w16=router_w16.view(torch.int16).numpy(),
        x=x.numpy(), out=np.stack(outs), out_noshared=np.stack(outs_noshared),
        idx=np.stack(idxs), w=np.stack(ws),
        dims=np.array([M, I, E, k, gs, T], np.int64))
    print("wrote", HERE / "format_vectors.npz", HERE / "moe_small.npz")


if __name__ == "__main__":
    main()
